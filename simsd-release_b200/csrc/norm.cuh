// Layer ops around the verify forward's linears: RMSNorm (optionally fused
// with the residual add before it) and the attention front end (per-head q/k
// RMSNorm, rotary embedding, K/V cache write).
//
// Reference math (sdar/modeling_sdar.py with the fp32 RMSNorm the runners
// install, sdar/run_native_tp2.py:34-51; rotary sdar/modeling_sdar.py:129-153;
// q/k norms over head_dim :197-302):
//   rmsnorm(x) = w * bf16(x_f32 * rsqrt(mean(x_f32^2) + eps))   (the product w * .
//                rounded to the input type)
//   rope(x)    = bf16(bf16(x * cos) + bf16(rotate_half(x) * sin)),
//                rotate_half(x)[i] = -x[i + D/2] (i < D/2), x[i - D/2] (i >= D/2)
// Every elementwise step rounds where the torch expressions round, so given the
// same mean square the outputs are the reference's bits; the mean square is an
// fp32 sum in this kernel's order (torch's reduction order is its own), then
// multiplied by 1/n as torch's mean does.
#pragma once
#include "sm100.cuh"
#include "moe.cuh"   // unpack8

namespace simsd {

constexpr int NORM_THREADS = 256;

__device__ __forceinline__ float round16(float v, int dtype) {
  return dtype == 0 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

// y[r] = rmsnorm(h[r]) with h = x (res == nullptr) or h = round(x + res)
// (then also written to h_out when that is not nullptr).  One CTA per row; the
// row's values stay in shared memory between the sum and the scaling.
struct RmsNormArgs {
  const void* x;
  const void* res;
  void* h_out;
  const void* w;
  void* y;
  long long ldx, ldres, ldh, ldy;
  int rows, n, dtype;
  float eps;
};

__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_kernel(const RmsNormArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ float nsh[];   // the row's h values (fp32) [n], then NORM_THREADS/32 partial sums
  float* hv = nsh;
  float* part = nsh + p.n;
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const char* xr = reinterpret_cast<const char*>(p.x) + (long long)r * p.ldx * 2;
  const char* rr = p.res ? reinterpret_cast<const char*>(p.res) + (long long)r * p.ldres * 2 : nullptr;
  float ss = 0.0f;
  for (int i = tid; i < p.n; i += NORM_THREADS) {
    float v = load_f(xr, i, p.dtype);
    if (rr) v = round16(__fadd_rn(v, load_f(rr, i, p.dtype)), p.dtype);
    hv[i] = v;
    ss = __fadd_rn(ss, __fmul_rn(v, v));   // x^2 rounded, then summed (torch's pow(2).mean)
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int j = 0; j < NORM_THREADS / 32; ++j) tot = __fadd_rn(tot, part[j]);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / (float)p.n), p.eps));
  char* yr = reinterpret_cast<char*>(p.y) + (long long)r * p.ldy * 2;
  char* hr = p.h_out ? reinterpret_cast<char*>(p.h_out) + (long long)r * p.ldh * 2 : nullptr;
  for (int i = tid; i < p.n; i += NORM_THREADS) {
    const float v = hv[i];
    if (hr) store_f(hr, i, v, p.dtype);
    const float nv = round16(__fmul_rn(v, inv), p.dtype);
    store_f(yr, i, __fmul_rn(load_f(p.w, i, p.dtype), nv), p.dtype);
  }
}

// The same RMSNorm for rows whose length is a multiple of 8 with 16-byte
// aligned rows: thread t holds the 8-element vectors t, t + 256, ... of its row
// in registers (VPT of them), so the row is read once with 16-byte loads, all
// issued before the first use, and never staged in shared memory.  Mean-square
// order: each thread sums its vectors' squares in element order, then the
// warp's xor butterfly, then the warps in order.
__device__ __forceinline__ uint4 pack8(const float (&f)[8], int dtype) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = (uint32_t)f32_to_16bit(f[2 * i], dtype) | ((uint32_t)f32_to_16bit(f[2 * i + 1], dtype) << 16);
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <int VPT>
__global__ void __launch_bounds__(NORM_THREADS) rmsnorm_vec_kernel(const RmsNormArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ float part[NORM_THREADS / 32];
  const int r = blockIdx.x;
  const int tid = threadIdx.x;
  const int nvec = p.n >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(p.x) + (long long)r * p.ldx * 2);
  const uint4* rr =
      p.res ? reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(p.res) + (long long)r * p.ldres * 2)
            : nullptr;
  uint4 xa[VPT], ra[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int vi = tid + j * NORM_THREADS;
    xa[j] = vi < nvec ? xr[vi] : make_uint4(0, 0, 0, 0);
    ra[j] = (rr && vi < nvec) ? rr[vi] : make_uint4(0, 0, 0, 0);
  }
  float h[VPT][8];
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    unpack8(xa[j], p.dtype, h[j]);
    if (rr) {
      float b[8];
      unpack8(ra[j], p.dtype, b);
#pragma unroll
      for (int e = 0; e < 8; ++e) h[j][e] = round16(__fadd_rn(h[j][e], b[e]), p.dtype);
    }
    if (tid + j * NORM_THREADS < nvec) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = __fadd_rn(ss, __fmul_rn(h[j][e], h[j][e]));
    }
  }
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
  if ((tid & 31) == 0) part[tid >> 5] = ss;
  __syncthreads();
  float tot = 0.0f;
#pragma unroll
  for (int j = 0; j < NORM_THREADS / 32; ++j) tot = __fadd_rn(tot, part[j]);
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(tot, 1.0f / (float)p.n), p.eps));
  uint4* yr = reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.y) + (long long)r * p.ldy * 2);
  uint4* hr = p.h_out ? reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.h_out) + (long long)r * p.ldh * 2)
                      : nullptr;
  const uint4* wv = reinterpret_cast<const uint4*>(p.w);
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int vi = tid + j * NORM_THREADS;
    if (vi >= nvec) break;
    if (hr) hr[vi] = pack8(h[j], p.dtype);
    float wf[8], o[8];
    unpack8(wv[vi], p.dtype, wf);
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = __fmul_rn(wf[e], round16(__fmul_rn(h[j][e], inv), p.dtype));
    yr[vi] = pack8(o, p.dtype);
  }
}

// Attention front end for L tokens of one sequence, head_dim D = 128:
//   qkv [L, (Hq + 2 Hk) * D] (row stride ldqkv): q heads, then k heads, then v;
//   q_out[h, t, :]           = rope(rmsnorm_qw(q[t, h]))      [Hq, L, D] contiguous
//   k_cache[g, pos + t, :]   = rope(rmsnorm_kw(k[t, g]))      [Hk, cap, D]
//   v_cache[g, pos + t, :]   = v[t, g]
// cos/sin [L, D] in the activation type.  One warp per (token, head): lane l
// holds elements l, l+32, l+64, l+96, so both rotary pairs (i, i + 64) are in
// the lane.
struct QkRopeArgs {
  const void* qkv;
  const void* qw;
  const void* kw;
  const void* cos;
  const void* sin;
  void* q_out;
  void* k_cache;
  void* v_cache;
  long long ldqkv, cache_cap;
  int L, Hq, Hk, pos, dtype;
  float eps;
};

constexpr int QKR_WARPS = 8;

__global__ void __launch_bounds__(QKR_WARPS * 32) qk_norm_rope_kernel(const QkRopeArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int D = 128;
  const int lane = threadIdx.x & 31;
  const long long unit = (long long)blockIdx.x * QKR_WARPS + (threadIdx.x >> 5);
  const int H = p.Hq + 2 * p.Hk;
  if (unit >= (long long)p.L * H) return;
  const int t = (int)(unit / H);
  const int h = (int)(unit - (long long)t * H);
  const char* src = reinterpret_cast<const char*>(p.qkv) + ((long long)t * p.ldqkv + (long long)h * D) * 2;
  float v[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = load_f(src, lane + 32 * j, p.dtype);
  if (h >= p.Hq + p.Hk) {
    // v: straight into the cache
    const int g = h - p.Hq - p.Hk;
    char* dst = reinterpret_cast<char*>(p.v_cache) + (((long long)g * p.cache_cap + p.pos + t) * D) * 2;
#pragma unroll
    for (int j = 0; j < 4; ++j) store_f(dst, lane + 32 * j, v[j], p.dtype);
    return;
  }
  const bool is_q = h < p.Hq;
  const void* w = is_q ? p.qw : p.kw;
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; ++j) ss = __fadd_rn(ss, __fmul_rn(v[j], v[j]));
#pragma unroll
  for (int m = 16; m > 0; m >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, m));
  const float inv = rsqrtf(__fadd_rn(__fmul_rn(ss, 1.0f / (float)D), p.eps));
  float nv[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    nv[j] = round16(__fmul_rn(load_f(w, lane + 32 * j, p.dtype), round16(__fmul_rn(v[j], inv), p.dtype)), p.dtype);
  const char* cr = reinterpret_cast<const char*>(p.cos) + (long long)t * D * 2;
  const char* sr = reinterpret_cast<const char*>(p.sin) + (long long)t * D * 2;
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int i = lane + 32 * j;
    const float rot = j < 2 ? -nv[j + 2] : nv[j - 2];   // rotate_half: pairs (i, i + 64)
    const float a = round16(__fmul_rn(nv[j], load_f(cr, i, p.dtype)), p.dtype);
    const float b = round16(__fmul_rn(rot, load_f(sr, i, p.dtype)), p.dtype);
    o[j] = __fadd_rn(a, b);
  }
  char* dst;
  if (is_q) {
    dst = reinterpret_cast<char*>(p.q_out) + (((long long)h * p.L + t) * D) * 2;
  } else {
    const int g = h - p.Hq;
    dst = reinterpret_cast<char*>(p.k_cache) + (((long long)g * p.cache_cap + p.pos + t) * D) * 2;
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) store_f(dst, lane + 32 * j, o[j], p.dtype);
}

}  // namespace simsd
