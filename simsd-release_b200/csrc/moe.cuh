// MoE dispatch kernels: top-k router, expert align (histogram, offsets, stable
// permutation), token-row gather and the fp32 weighted combine.
//
// Reference: kernels/moe_dispatch_fused.py:93-132 (`_align`), :165-192
// (`moe_dispatch`), and the synthetic router of
// kernels/workspace/moe_dispatch/build_oracle.py:71-90 (sigmoid scores, top-k,
// renormalise, routed scale).  The real LLaDA2 gate is remote code that is not
// part of the reference; the router here selects on sigmoid(logit) + bias.
//
// Routing is integer work downstream of fp32 logits, so it can only be
// bit-exact against a checker that computes the same logits bit for bit.  The
// router therefore fixes its arithmetic completely:
//   logit[t,e]: lane l (0..31) of a warp accumulates, with fp32 fma, the
//     8-element chunks c = l, l+32, l+64, ... of x[t,:] . w[e,:] in increasing
//     element order; the 32 lane sums are combined by the xor butterfly
//     (16, 8, 4, 2, 1), v_l <- v_l + v_{l^m};
//   score = 1 / (1 + exp(-logit)) with exp_fixed() below;
//   choice = score + bias[e]; top-k by choice, ties to the lower expert id,
//     NaN ranked below every number;
//   weight_j = score[id_j]; if renormalising and k > 1:
//     weight_j /= (((w_0 + w_1) + w_2) + ...) + 1e-20; then weight_j *= scale.
// Every operation is an explicitly rounded fp32 op, so the C oracle
// (oracle/simsd_oracle.c) reproduces it exactly.
#pragma once
#include "sm100.cuh"

namespace simsd {

// exp(x) in fp32 by Cody-Waite reduction x = n ln2 + r (ln2 split into a high
// part with 11 trailing zero bits and the remainder), |r| <= ln2/2, and the
// degree-7 Taylor polynomial of e^r in Horner form (truncation error below
// 2^-24 relative); 2^n is applied in two exact power-of-two steps.
__device__ __forceinline__ float exp_fixed(float x) {
  if (!(x == x)) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.97208404541015625f) return 0.0f;
  const float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.428606765330187045037746429443359375e-06f, r);
  float q = 1.98412701138295233249664306640625e-04f;  // 1/5040
  q = __fmaf_rn(q, r, 1.3888889225199818611145019531250e-03f);  // 1/720
  q = __fmaf_rn(q, r, 8.3333337679505348205566406250000e-03f);  // 1/120
  q = __fmaf_rn(q, r, 4.1666667908430099487304687500000e-02f);  // 1/24
  q = __fmaf_rn(q, r, 1.6666667163372039794921875000000e-01f);  // 1/6
  q = __fmaf_rn(q, r, 0.5f);
  q = __fmaf_rn(q, r, 1.0f);
  q = __fmaf_rn(q, r, 1.0f);
  const int ni = (int)n;
  const int n1 = ni >> 1;   // floor(n/2)
  const int n2 = ni - n1;
  q = __fmul_rn(q, __int_as_float((n1 + 127) << 23));
  q = __fmul_rn(q, __int_as_float((n2 + 127) << 23));
  return q;
}

__device__ __forceinline__ float sigmoid_fixed(float z) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_fixed(-z)));
}

// ------------------------------------------------------------------ router
struct RouteArgs {
  const void* x;          // [T, H], row stride ldx
  const void* w;          // [E, H], row stride ldw
  const float* bias;      // [E] or nullptr
  long long* topk_ids;    // [T, k]
  float* topk_weight;     // [T, k]
  float* logits;          // [T, E] or nullptr (debug / parity)
  long long ldx, ldw;
  int T, H, E, k;
  int x_dtype, w_dtype;   // 0 bf16, 1 fp16, 2 fp32
  int renorm;
  float scale;
  int ldo;                // row stride of topk_ids / topk_weight (>= k)
  int extra_id;           // >= 0: column k of every row gets this id with weight 1 (an always-on expert)
};

constexpr int ROUTE_TOK = 16;    // tokens per CTA
constexpr int ROUTE_EXP = 4;     // experts per warp pass
constexpr int ROUTE_WARPS = 8;

__device__ __forceinline__ void load8(const void* base, long long idx, int dtype, int n_valid, float (&v)[8]) {
  if (n_valid == 8 && dtype != 2 && ((reinterpret_cast<uintptr_t>(base) + idx * 2) & 15) == 0) {
    const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(base) + idx * 2);
    const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == 0) {
        v[2 * i] = __uint_as_float(w4[i] << 16);
        v[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
      } else {
        __half2 h = *reinterpret_cast<const __half2*>(&w4[i]);
        const float2 f = __half22float2(h);
        v[2 * i] = f.x;
        v[2 * i + 1] = f.y;
      }
    }
    return;
  }
  if (n_valid == 8 && dtype == 2 && ((reinterpret_cast<uintptr_t>(base) + idx * 4) & 15) == 0) {
    const float4 a = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx);
    const float4 b = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(base) + idx + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = (i < n_valid) ? load_f(base, idx + i, dtype) : 0.0f;
}

// top-k per token, one warp per token; lane l owns experts l, l+32, ... (NC
// per lane, held in registers).  Each round takes the largest remaining choice
// (ties to the lower expert id, NaN below every number); lane j keeps round
// j's pick.  The weights are then normalised with the sum taken in round
// order, (((w_0 + w_1) + w_2) + ...) + 1e-20, and lane j writes output j.
template <int NC>
__device__ __forceinline__ void route_topk_nc(const RouteArgs& p, const float* s_score, const float* s_choice,
                                              int t0, int ntok) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int t = warp; t < ntok; t += nwarps) {
    const float* ch = s_choice + t * p.E;
    float cv[NC];
#pragma unroll
    for (int i = 0; i < NC; ++i) {
      const int e = lane + 32 * i;
      float v = e < p.E ? ch[e] : 0.0f;
      if (v != v) v = -__int_as_float(0x7f800000);
      cv[i] = v;
    }
    unsigned taken = 0u;
    int my_id = -1;
    float my_w = 0.0f;
    for (int j = 0; j < p.k; ++j) {
      float bb = 0.0f;
      int be = -1;
#pragma unroll
      for (int i = 0; i < NC; ++i) {
        const int e = lane + 32 * i;
        if (e < p.E && !((taken >> i) & 1u) && (be < 0 || cv[i] > bb)) { bb = cv[i]; be = e; }
      }
#pragma unroll
      for (int m = 16; m > 0; m >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, bb, m);
        const int oe = __shfl_xor_sync(0xffffffffu, be, m);
        const bool take = (be < 0) || (oe >= 0 && (ob > bb || (ob == bb && oe < be)));
        if (take) { bb = ob; be = oe; }
      }
      if (be >= 0 && (be & 31) == lane) taken |= 1u << (be >> 5);
      if (lane == j) {
        my_id = be;
        my_w = (be >= 0) ? s_score[t * p.E + be] : 0.0f;
      }
    }
    const bool norm = p.renorm && p.k > 1;
    float denom = 1.0f;
    if (norm) {
      float sum = __shfl_sync(0xffffffffu, my_w, 0);
      for (int j = 1; j < p.k; ++j) sum = __fadd_rn(sum, __shfl_sync(0xffffffffu, my_w, j));
      denom = __fadd_rn(sum, 1e-20f);
    }
    if (lane < p.k) {
      float wj = my_w;
      if (norm) wj = __fdiv_rn(wj, denom);
      wj = __fmul_rn(wj, p.scale);
      p.topk_ids[(long long)(t0 + t) * p.ldo + lane] = my_id;
      p.topk_weight[(long long)(t0 + t) * p.ldo + lane] = wj;
    }
    if (p.extra_id >= 0 && lane == 0) {
      p.topk_ids[(long long)(t0 + t) * p.ldo + p.k] = p.extra_id;
      p.topk_weight[(long long)(t0 + t) * p.ldo + p.k] = 1.0f;
    }
    __syncwarp();
  }
}

__device__ __forceinline__ void route_topk(const RouteArgs& p, const float* s_score, const float* s_choice, int t0,
                                           int ntok) {
  if (p.E <= 256) route_topk_nc<8>(p, s_score, s_choice, t0, ntok);
  else route_topk_nc<32>(p, s_score, s_choice, t0, ntok);
}

__global__ void __launch_bounds__(ROUTE_WARPS * 32) route_kernel(const RouteArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ float sh[];
  float* s_score = sh;                          // [ROUTE_TOK][E]
  float* s_choice = sh + ROUTE_TOK * p.E;       // [ROUTE_TOK][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * ROUTE_TOK;
  const int ntok = min(ROUTE_TOK, p.T - t0);
  const int nchunks = (p.H + 7) / 8;

  for (int e0 = warp * ROUTE_EXP; e0 < p.E; e0 += ROUTE_WARPS * ROUTE_EXP) {
    float acc[ROUTE_TOK][ROUTE_EXP];
#pragma unroll
    for (int t = 0; t < ROUTE_TOK; ++t)
#pragma unroll
      for (int j = 0; j < ROUTE_EXP; ++j) acc[t][j] = 0.0f;
    for (int c = lane; c < nchunks; c += 32) {
      const int k0 = c * 8;
      const int nv = min(8, p.H - k0);
      float wv[ROUTE_EXP][8];
#pragma unroll
      for (int j = 0; j < ROUTE_EXP; ++j) {
        if (e0 + j < p.E) load8(p.w, (long long)(e0 + j) * p.ldw + k0, p.w_dtype, nv, wv[j]);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) wv[j][i] = 0.0f;
        }
      }
#pragma unroll
      for (int t = 0; t < ROUTE_TOK; ++t) {
        if (t < ntok) {
          float xv[8];
          load8(p.x, (long long)(t0 + t) * p.ldx + k0, p.x_dtype, nv, xv);
#pragma unroll
          for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < ROUTE_EXP; ++j) acc[t][j] = __fmaf_rn(xv[i], wv[j][i], acc[t][j]);
        }
      }
    }
#pragma unroll
    for (int t = 0; t < ROUTE_TOK; ++t)
#pragma unroll
      for (int j = 0; j < ROUTE_EXP; ++j) {
        float v = acc[t][j];
#pragma unroll
        for (int m = 16; m > 0; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
        acc[t][j] = v;
      }
    if (lane == 0) {
#pragma unroll
      for (int t = 0; t < ROUTE_TOK; ++t)
#pragma unroll
        for (int j = 0; j < ROUTE_EXP; ++j)
          if (t < ntok && e0 + j < p.E) {
            const int e = e0 + j;
            const float lg = acc[t][j];
            if (p.logits) p.logits[(long long)(t0 + t) * p.E + e] = lg;
            const float s = sigmoid_fixed(lg);
            s_score[t * p.E + e] = s;
            s_choice[t * p.E + e] = p.bias ? __fadd_rn(s, p.bias[e]) : s;
          }
    }
  }
  __syncthreads();

  route_topk(p, s_score, s_choice, t0, ntok);
}

// Fast router for 16-bit activations with H % 8 == 0 and 16-byte aligned rows.
// A CTA of ROUTE_FAST_WARPS warps stages TT token rows in shared memory as
// fp32, four tokens to a 16-byte vector: xs[(i * TT/4 + q) * nchunks + c]
// holds element 8c + i of tokens 4q .. 4q+3, so the lanes of a warp
// (consecutive chunks c) read consecutive vectors and the inner loop converts
// no activations.  Each warp pass computes the TT x (32/TT) logits of TT
// tokens and 32/TT experts with the same per-lane chunk order as route_kernel;
// the fp32 fmas of a token pair run as one packed __ffma2_rn, which rounds
// each half exactly like __fmaf_rn, so every accumulator sees the same
// sequence of correctly rounded fmas.  A reduce-scatter butterfly then leaves
// logit q of the pass in lane q; its pairing tree is the one of the xor
// butterfly (v_l + v_{l^m} for m = 16, 8, 4, 2, 1), so the logits are
// bit-identical to route_kernel's and to the oracle's.  The activation and
// weight types are template parameters (XDT: 0 bf16, 1 fp16; WDT: 0 bf16,
// 1 fp16, 2 fp32) so the loop carries no per-element type dispatch.  The
// weight chunks are fetched one step ahead, across a warp's passes too, and
// each block walks its experts from a different starting group so the blocks
// do not all read the same router rows at once.  TT adapts to T so small
// batches still spread over many SMs.
constexpr int ROUTE_FAST_WARPS = 16;

template <int WDT>
__device__ __forceinline__ float route_w_elem(const uint4 (&r)[WDT == 2 ? 2 : 1], int i) {
  if constexpr (WDT == 2) {
    const uint4 u = r[i >> 2];
    const uint32_t b = (i & 3) == 0 ? u.x : (i & 3) == 1 ? u.y : (i & 3) == 2 ? u.z : u.w;
    return __uint_as_float(b);
  } else {
    const uint4 u = r[0];
    const int h = i >> 1;
    const uint32_t b = h == 0 ? u.x : h == 1 ? u.y : h == 2 ? u.z : u.w;
    if constexpr (WDT == 0) return __uint_as_float((i & 1) ? (b & 0xffff0000u) : (b << 16));
    else return __half2float(__ushort_as_half((unsigned short)((i & 1) ? (b >> 16) : (b & 0xffffu))));
  }
}

// WSM: the block's router rows are first copied into shared memory with all
// loads in flight at once (the expert-split launch for few tokens, where a
// warp's chain of dependent per-chunk weight loads would otherwise set the
// time); the arithmetic is unchanged.
template <int TT, int XDT, int WDT, bool WSM>
__global__ void __launch_bounds__(ROUTE_FAST_WARPS * 32) route_fast_kernel(const RouteArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  constexpr int EE = 32 / TT;
  constexpr int TQ = TT / 4;                       // 4-token vectors
  extern __shared__ __align__(16) unsigned char rsh[];
  float4* xs = reinterpret_cast<float4*>(rsh);                            // [8][TQ][nchunks]
  float* s_score = reinterpret_cast<float*>(rsh + (size_t)TT * p.H * 4);  // [TT][E]
  float* s_choice = s_score + TT * p.E;
  uint4* wsm = reinterpret_cast<uint4*>(s_choice + TT * p.E);             // WSM: [per][nchunks][WV]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * TT;
  const int ntok = min(TT, p.T - t0);
  const int E = p.E;
  const int nchunks = p.H / 8;

  // stage the token rows as fp32 (rows past T are zero)
  {
    float* xf = reinterpret_cast<float*>(xs);
    for (int idx = threadIdx.x; idx < TT * nchunks; idx += blockDim.x) {
      const int t = idx / nchunks, c = idx - t * nchunks;
      uint4 u = make_uint4(0, 0, 0, 0);
      if (t < ntok)
        u = *reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p.x) + (long long)(t0 + t) * p.ldx + c * 8);
      const uint32_t x4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        float lo, hi;
        if constexpr (XDT == 0) {
          lo = __uint_as_float(x4[h] << 16);
          hi = __uint_as_float(x4[h] & 0xffff0000u);
        } else {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&x4[h]));
          lo = f.x;
          hi = f.y;
        }
        xf[(((2 * h) * TQ + (t >> 2)) * nchunks + c) * 4 + (t & 3)] = lo;
        xf[(((2 * h + 1) * TQ + (t >> 2)) * nchunks + c) * 4 + (t & 3)] = hi;
      }
    }
  }
  __syncthreads();

  // experts of this block: all of them, or (grid.y > 1) a slice whose logits go
  // to p.logits for route_topk_kernel
  const int per = gridDim.y > 1 ? ((E + gridDim.y - 1) / gridDim.y + EE - 1) / EE * EE : E;
  const int ebeg = blockIdx.y * per, eend = min(E, ebeg + per);
  constexpr int WV = WDT == 2 ? 2 : 1;             // uint4 per 8-element chunk
  auto gload_w = [&](int e, int c, int q) {
    return *reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(p.w) +
                                           ((long long)e * p.ldw + c * 8) * (WDT == 2 ? 4 : 2) + q * 16);
  };
  if constexpr (WSM) {
    const int total = (eend - ebeg) * nchunks * WV;
    constexpr int UNR = 8;
    for (int base = threadIdx.x; base < total; base += UNR * blockDim.x) {
      uint4 tmp[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int idx = base + u * blockDim.x;
        if (idx < total) {
          const int el = idx / (nchunks * WV), r = idx - el * (nchunks * WV);
          tmp[u] = gload_w(ebeg + el, r / WV, r % WV);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int idx = base + u * blockDim.x;
        if (idx < total) wsm[idx] = tmp[u];
      }
    }
    __syncthreads();
  }
  // (fp32 weights of eight experts would not leave registers for a prefetch;
  // staged weights need none)
  constexpr bool PREFETCH = !WSM && !(WDT == 2 && EE > 4);
  uint4 wraw[EE][WV], wnext[EE][WV];
  auto load_w = [&](int e0, int c, uint4 (&dst)[EE][WV]) {
#pragma unroll
    for (int j = 0; j < EE; ++j) {
      const int e = e0 + j;
#pragma unroll
      for (int q = 0; q < WV; ++q) {
        if (e < eend && c < nchunks) {
          if constexpr (WSM) dst[j][q] = wsm[((e - ebeg) * nchunks + c) * WV + q];
          else dst[j][q] = gload_w(e, c, q);
        } else {
          dst[j][q] = make_uint4(0, 0, 0, 0);
        }
      }
    }
  };
  // The block's experts form NG groups of EE; warp w takes groups w, w + NW,
  // ... rotated by a per-block offset.  Which warp computes a logit does not
  // change its arithmetic.
  const int NG = (eend - ebeg + EE - 1) / EE;
  const int rot = NG > 0 ? (int)((blockIdx.x * 7u) % (unsigned)NG) : 0;
  auto group_e0 = [&](int gi) { return ebeg + ((gi + rot) % NG) * EE; };
  if (PREFETCH && warp < NG) load_w(group_e0(warp), lane, wraw);
  for (int gi = warp; gi < NG; gi += ROUTE_FAST_WARPS) {
    const int e0 = group_e0(gi);
    float2 acc[EE][TT / 2];                          // (token 2u, token 2u+1) of expert e0 + j
#pragma unroll
    for (int j = 0; j < EE; ++j)
#pragma unroll
      for (int u = 0; u < TT / 2; ++u) acc[j][u] = make_float2(0.0f, 0.0f);
    for (int c = lane; c < nchunks; c += 32) {
      if (PREFETCH) {
        // the next chunk of this pass, or the first chunk of the next pass
        if (c + 32 < nchunks) load_w(e0, c + 32, wnext);
        else if (gi + ROUTE_FAST_WARPS < NG) load_w(group_e0(gi + ROUTE_FAST_WARPS), lane, wnext);
      } else {
        load_w(e0, c, wraw);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        float2 w2[EE];
#pragma unroll
        for (int j = 0; j < EE; ++j) {
          const float w = route_w_elem<WDT>(wraw[j], i);
          w2[j] = make_float2(w, w);
        }
#pragma unroll
        for (int q = 0; q < TQ; ++q) {
          const float4 xq = xs[(i * TQ + q) * nchunks + c];
#pragma unroll
          for (int j = 0; j < EE; ++j) {
            acc[j][2 * q] = __ffma2_rn(make_float2(xq.x, xq.y), w2[j], acc[j][2 * q]);
            acc[j][2 * q + 1] = __ffma2_rn(make_float2(xq.z, xq.w), w2[j], acc[j][2 * q + 1]);
          }
        }
      }
      if (PREFETCH) {
#pragma unroll
        for (int j = 0; j < EE; ++j)
#pragma unroll
          for (int q = 0; q < WV; ++q) wraw[j][q] = wnext[j][q];
      }
    }
    // v[t * EE + j] = lane partial of token t, expert e0 + j
    float v[32];
#pragma unroll
    for (int t = 0; t < TT; ++t)
#pragma unroll
      for (int j = 0; j < EE; ++j) v[t * EE + j] = (t & 1) ? acc[j][t >> 1].y : acc[j][t >> 1].x;
    // reduce-scatter: after the step with offset m, a lane keeps the half of
    // its values whose index bit log2(m) equals its own lane bit
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < m; ++i) {
        const float send = upper ? v[i] : v[i + m];
        const float keep = upper ? v[i + m] : v[i];
        const float recv = __shfl_xor_sync(0xffffffffu, send, m);
        v[i] = __fadd_rn(keep, recv);
      }
    }
    const int t = lane / EE, e = e0 + (lane % EE);
    if (t < ntok && e < eend) {
      const float lg = v[0];
      if (p.logits) p.logits[(long long)(t0 + t) * E + e] = lg;
      if (gridDim.y == 1) {
        const float sc = sigmoid_fixed(lg);
        s_score[t * E + e] = sc;
        s_choice[t * E + e] = p.bias ? __fadd_rn(sc, p.bias[e]) : sc;
      }
    }
  }
  if (gridDim.y > 1) return;   // route_topk_kernel selects from p.logits
  __syncthreads();
  route_topk(p, s_score, s_choice, t0, ntok);
}

// Top-k over logits that route_fast_kernel wrote with its experts split over
// blocks (few tokens, so that the logits use many SMs): the same sigmoid, bias
// and selection as its fused path, ROUTE_WARPS tokens per block.
__global__ void __launch_bounds__(ROUTE_WARPS * 32) route_topk_kernel(const RouteArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ float tsh[];
  float* s_score = tsh;                        // [ROUTE_WARPS][E]
  float* s_choice = tsh + ROUTE_WARPS * p.E;   // [ROUTE_WARPS][E]
  const int t0 = blockIdx.x * ROUTE_WARPS;
  const int ntok = min(ROUTE_WARPS, p.T - t0);
  // the block's logits are contiguous: load UNR of them per thread before
  // any arithmetic, so the loads are in flight together
  const int n = ntok * p.E;
  const float* lg = p.logits + (long long)t0 * p.E;
  constexpr int UNR = 8;
  for (int base = threadIdx.x; base < n; base += UNR * blockDim.x) {
    float v[UNR], b[UNR];
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int i = base + u * blockDim.x;
      v[u] = i < n ? lg[i] : 0.0f;
      b[u] = (i < n && p.bias) ? p.bias[i % p.E] : 0.0f;
    }
#pragma unroll
    for (int u = 0; u < UNR; ++u) {
      const int i = base + u * blockDim.x;
      if (i < n) {
        const float sc = sigmoid_fixed(v[u]);
        s_score[i] = sc;
        s_choice[i] = p.bias ? __fadd_rn(sc, b[u]) : sc;
      }
    }
  }
  __syncthreads();
  route_topk(p, s_score, s_choice, t0, ntok);
}

// ------------------------------------------------------------------ align
// Stable counting sort of the T*k slots (slot = t*k + j) by expert, in one CTA:
// per-warp histograms over contiguous slot ranges, a scan over (warp, expert),
// then each warp re-walks its range in order and ranks equal experts inside
// each 32-slot step with __match_any_sync.  The permutation equals
// torch.argsort(ids.flatten(), stable=True) (kernels/moe_dispatch_fused.py:121).
struct AlignArgs {
  const long long* ids;   // [S]
  int* counts;            // [E]
  int* offsets;           // [E+1]
  int* sorted_slots;      // [S]  row -> slot
  int* slot_to_row;       // [S]  slot -> row, -1 for an id outside [0, E)
  int* slots_padded;      // reference layout [num_tiles*block_m] or nullptr
  int* tile_expert;       // reference layout [num_tiles] or nullptr
  int* err;
  int S, E, block_m, num_tiles;
  int ids_in_smem;        // 1: the launch reserved S ints of shared memory for the ids
};

constexpr int ALIGN_THREADS = 1024;

__global__ void __launch_bounds__(ALIGN_THREADS, 1) align_kernel(const AlignArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ int ash[];
  int* hist = ash;                       // [32][E]
  int* s_off = ash + 32 * p.E;           // [E+1]
  int* s_pad = s_off + p.E + 1;          // [E+1] padded ends (reference layout)
  __shared__ int s_wsum[32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int E = p.E, S = p.S;
  const int L = (S + 31) / 32;
  const int lo = warp * L, hi = min(S, lo + L);

  // the ids are read twice below; keep an int32 copy in shared memory when it fits
  int* s_ids = s_pad + E + 1;
  const bool cache_ids = p.ids_in_smem != 0;
  for (int i = tid; i < 32 * E; i += ALIGN_THREADS) hist[i] = 0;
  if (cache_ids)
    for (int i = tid; i < S; i += ALIGN_THREADS) {
      const long long e = p.ids[i];
      s_ids[i] = (e >= 0 && e < E) ? (int)e : (e < 0 ? -1 : E);   // E: out of range
    }
  __syncthreads();
  auto id_at = [&](int s) -> long long { return cache_ids ? (long long)s_ids[s] : p.ids[s]; };
  for (int s = lo + lane; s < hi; s += 32) {
    const long long e = id_at(s);
    if (e >= 0 && e < E) atomicAdd(&hist[warp * E + (int)e], 1);
  }
  __syncthreads();
  // per expert: exclusive scan over warps; counts
  for (int e = tid; e < E; e += ALIGN_THREADS) {
    int run = 0;
    for (int w = 0; w < 32; ++w) {
      const int v = hist[w * E + e];
      hist[w * E + e] = run;
      run += v;
    }
    s_off[e + 1] = run;
    p.counts[e] = run;
  }
  __syncthreads();
  // exclusive scan of counts over experts (E <= 1024 = one element per thread)
  {
    int v = (tid < E) ? s_off[tid + 1] : 0;
    int x = v;
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) s_wsum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = s_wsum[lane];
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      s_wsum[lane] = w;  // inclusive
    }
    __syncthreads();
    const int incl = x + (warp > 0 ? s_wsum[warp - 1] : 0);
    __syncthreads();
    if (tid < E) s_off[tid + 1] = incl;
    if (tid == 0) s_off[0] = 0;
    __syncthreads();
  }
  for (int e = tid; e <= E; e += ALIGN_THREADS) p.offsets[e] = s_off[e];
  for (int i = tid; i < 32 * E; i += ALIGN_THREADS) hist[i] += s_off[i % E];
  __syncthreads();
  // stable scatter
  const unsigned lt = (1u << lane) - 1u;
  for (int base = lo; base < hi; base += 32) {
    const int s = base + lane;
    int e = -2;
    bool valid = false;
    if (s < hi) {
      const long long ev = id_at(s);
      if (ev >= 0 && ev < E) { e = (int)ev; valid = true; }
      else { e = -1; }
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    int row = -1;
    if (valid) row = hist[warp * E + e] + __popc(peers & lt);
    __syncwarp();
    if (valid && lane == __ffs(peers) - 1) hist[warp * E + e] += __popc(peers);
    __syncwarp();
    if (s < hi) {
      p.slot_to_row[s] = row;
      if (valid) p.sorted_slots[row] = s;
      else if (id_at(s) >= 0) atomicOr(p.err, SIMSD_DEV_ERR_BAD_INDEX);   // id >= E; negative = no expert
    }
  }
  // rows left over by invalid ids hold no slot
  for (int row = s_off[E] + tid; row < S; row += ALIGN_THREADS) p.sorted_slots[row] = -1;
  if (p.slots_padded == nullptr) return;
  __syncthreads();
  // reference layout: groups padded to block_m rows, -1 = padding
  const int bm = p.block_m;
  if (tid == 0) {
    int run = 0;
    for (int e = 0; e < E; ++e) {
      const int c = s_off[e + 1] - s_off[e];
      run += ((c + bm - 1) / bm) * bm;
      s_pad[e + 1] = run;
    }
    s_pad[0] = 0;
  }
  const long long npad = (long long)p.num_tiles * bm;
  for (long long i = tid; i < npad; i += ALIGN_THREADS) p.slots_padded[i] = -1;
  __syncthreads();
  for (int row = tid; row < s_off[E]; row += ALIGN_THREADS) {
    // expert of this sorted row: largest e with s_off[e] <= row
    int a = 0, b = E - 1;
    while (a < b) {
      const int mid = (a + b + 1) >> 1;
      if (s_off[mid] <= row) a = mid; else b = mid - 1;
    }
    const long long dst = (long long)s_pad[a] + (row - s_off[a]);
    if (dst < npad) p.slots_padded[dst] = p.sorted_slots[row];
    else atomicOr(p.err, SIMSD_DEV_ERR_BAD_INDEX);
  }
  for (int t = tid; t < p.num_tiles; t += ALIGN_THREADS) {
    const long long v = (long long)t * bm;
    // number of padded group ends <= v  (torch.searchsorted(..., right=True))
    int a = 0, b = E;
    while (a < b) {
      const int mid = (a + b) >> 1;
      if (s_pad[mid + 1] <= v) a = mid + 1; else b = mid;
    }
    p.tile_expert[t] = a;
  }
}

// ------------------------------------------------------------------ gather
// xs[row, :] = x[sorted_slots[row] / k, :]
__global__ void gather_rows_kernel(const void* x, long long ldx, const int* sorted_slots, void* xs, long long ldxs,
                                   int S, int k, int H, int esz) {
  griddep_launch_dependents();
  griddep_wait();
  const int row = blockIdx.x;
  if (row >= S) return;
  const int slot = sorted_slots[row];
  if (slot < 0) return;  // no token (an invalid expert id left this row empty)
  const int tok = slot / k;
  const char* src = reinterpret_cast<const char*>(x) + (long long)tok * ldx * esz;
  char* dst = reinterpret_cast<char*>(xs) + (long long)row * ldxs * esz;
  const long long nbytes = (long long)H * esz;
  if (((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0 && (nbytes & 15) == 0) {
    for (long long i = threadIdx.x; i < nbytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
  } else {
    for (long long i = threadIdx.x; i < nbytes; i += blockDim.x) dst[i] = src[i];
  }
}

// ------------------------------------------------------------------ expert-parallel exchange
// The expert-parallel layer's two exchanges as plain stores into every rank's
// receive blocks (NVLink peer mappings; the own rank's block is local).
// Bucket entry e = p * cap + i of this rank (p: the rank it goes to, i: its
// position in the fixed-capacity bucket) lands in row rank * cap + i of rank
// p's block, the layout an all-to-all of [world * cap] rows gives.
//   send   (mode 0): row x[sel[e] / k] when sel[e] >= 0 (sel = the bucket's
//          slots), and the local expert id expert[e] for every entry (-1 for
//          an empty one), so the receiver's ids are all rewritten each call;
//   return (mode 1): row y[e] when sel[e] >= 0 (sel = the received expert
//          ids), back to the rank p it came from.
// Only occupied entries move a row.  One warp per entry, 16-byte stores.
constexpr int EP_XCH_MAX_WORLD = 8;   // ranks of a peer-store exchange (a node)
struct EpExchangeArgs {
  const void* src;            // x (send) or the experts' output y (return)
  long long src_row_bytes;    // row stride of src in bytes
  const int* sel;             // [entries]
  const int* expert;          // [entries] (send only)
  void* rows[EP_XCH_MAX_WORLD];   // every rank's row block [world * cap, H]
  int* ids[EP_XCH_MAX_WORLD];     // every rank's id block [world * cap] (send only)
  int entries, cap, k, rank, mode, row_bytes;
};

__global__ void __launch_bounds__(256) ep_exchange_kernel(const __grid_constant__ EpExchangeArgs a) {
  griddep_launch_dependents();
  griddep_wait();
  const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (e >= a.entries) return;
  const int p = e / a.cap;
  const long long drow = (long long)a.rank * a.cap + (e - p * a.cap);
  const int s = a.sel[e];
  if (a.mode == 0 && lane == 0) a.ids[p][drow] = a.expert[e];
  if (s < 0) return;
  const long long srow = a.mode == 0 ? s / a.k : e;
  const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a.src) + srow * a.src_row_bytes);
  uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a.rows[p]) + drow * a.row_bytes);
  const int n16 = a.row_bytes >> 4;
#pragma unroll 4
  for (int c = lane; c < n16; c += 32) dst[c] = src[c];
}

// ------------------------------------------------------------------ combine
// out[t, h] = cast( sum_j  fp32(ys[row(t,j), h]) * w[t, j] )  (j in order, each
// product rounded to fp32 before the add, as `.mul_(w).sum(dim=1)` does:
// kernels/moe_dispatch_fused.py:189-192); with `add` (the shared expert's
// output) the result is cast(fp32(cast(sum)) + fp32(add[t, h])), i.e. the
// x.dtype addition `moe_out + shared_out`.
__global__ void combine_kernel(const void* ys, long long ldys, const int* slot_to_row, const float* w, void* out,
                               long long ld_out, const void* add, long long ld_add, int T, int k, int H, int dtype,
                               int shared_last) {
  griddep_launch_dependents();
  griddep_wait();
  const int t = blockIdx.x;
  if (t >= T) return;
  const int kr = shared_last ? k - 1 : k;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.0f;
    for (int j = 0; j < kr; ++j) {
      const int row = slot_to_row[(long long)t * k + j];
      if (row < 0) continue;
      const float y = load_f(ys, (long long)row * ldys + h, dtype);
      acc = __fadd_rn(acc, __fmul_rn(y, w[(long long)t * k + j]));
    }
    if (shared_last) {
      const int row = slot_to_row[(long long)t * k + k - 1];
      if (row >= 0) {
        float r = acc;
        if (dtype == 0) r = __bfloat162float(__float2bfloat16_rn(acc));
        else if (dtype == 1) r = __half2float(__float2half_rn(acc));
        acc = __fadd_rn(r, load_f(ys, (long long)row * ldys + h, dtype));
      }
    }
    if (add) {
      float r = acc;
      if (dtype == 0) r = __bfloat162float(__float2bfloat16_rn(acc));
      else if (dtype == 1) r = __half2float(__float2half_rn(acc));
      acc = __fadd_rn(r, load_f(add, (long long)t * ld_add + h, dtype));
    }
    store_f(out, (long long)t * ld_out + h, acc, dtype);
  }
}

// combine_kernel for 16-bit outputs with H % 8 == 0: a thread owns 8 adjacent
// columns (16-byte loads and stores); same arithmetic, same order.
__device__ __forceinline__ void unpack8(uint4 u, int dtype, float (&v)[8]) {
  const uint32_t w4[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if (dtype == 0) {
      v[2 * i] = __uint_as_float(w4[i] << 16);
      v[2 * i + 1] = __uint_as_float(w4[i] & 0xffff0000u);
    } else {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[i]));
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

__device__ __forceinline__ float round_to_dtype(float v, int dtype) {
  return dtype == 0 ? __bfloat162float(__float2bfloat16_rn(v)) : __half2float(__float2half_rn(v));
}

// shared_last: column k-1 is an always-on (shared) expert, added unweighted to
// the rounded sum of the other columns, as `add` is.
__global__ void combine_vec_kernel(const void* ys, long long ldys, const int* slot_to_row, const float* w, void* out,
                                   long long ld_out, const void* add, long long ld_add, int T, int k, int H,
                                   int dtype, int shared_last) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int s_row[32];
  __shared__ float s_w[32];
  const int t = blockIdx.x;
  if (t >= T) return;
  if (threadIdx.x < k) {
    s_row[threadIdx.x] = slot_to_row[(long long)t * k + threadIdx.x];
    s_w[threadIdx.x] = w[(long long)t * k + threadIdx.x];
  }
  __syncthreads();
  const uint16_t* yb = reinterpret_cast<const uint16_t*>(ys);
  for (int h8 = threadIdx.x; h8 < H / 8; h8 += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    const int kr = shared_last ? k - 1 : k;
    for (int j = 0; j < kr; ++j) {
      const int row = s_row[j];
      if (row < 0) continue;
      float y[8];
      unpack8(*reinterpret_cast<const uint4*>(yb + (long long)row * ldys + h8 * 8), dtype, y);
      const float wj = s_w[j];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(acc[i], __fmul_rn(y[i], wj));
    }
    if (shared_last && s_row[k - 1] >= 0) {
      float a[8];
      unpack8(*reinterpret_cast<const uint4*>(yb + (long long)s_row[k - 1] * ldys + h8 * 8), dtype, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(round_to_dtype(acc[i], dtype), a[i]);
    }
    if (add) {
      float a[8];
      unpack8(*reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(add) + (long long)t * ld_add + h8 * 8),
              dtype, a);
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = __fadd_rn(round_to_dtype(acc[i], dtype), a[i]);
    }
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (dtype == 0) {
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i]));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i + 1]));
        o[i] = lo | (hi << 16);
      } else {
        const uint32_t lo = __half_as_ushort(__float2half_rn(acc[2 * i]));
        const uint32_t hi = __half_as_ushort(__float2half_rn(acc[2 * i + 1]));
        o[i] = lo | (hi << 16);
      }
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + (long long)t * ld_out + h8 * 8) =
        make_uint4(o[0], o[1], o[2], o[3]);
  }
}


// ------------------------------------------------------------------ expert-parallel buckets
// Expert e lives on rank e / (E / world) as its local expert e % (E / world).
// Slot s = t*k + j of this rank's tokens goes to bucket peer(ids[s]) at the
// next free position, in slot order (stable): send_slot[peer*cap + i] = s,
// send_expert[...] = local expert id, slot_pos[s] = peer*cap + i.  Unused
// bucket entries hold -1; a slot beyond `cap` or with an id outside [0, E) gets
// slot_pos -1 (BAD_INDEX / CAPACITY in the error word).  counts[peer] = slots
// bound for the peer.  One CTA; stable ranks come from warp match masks and a
// per-chunk scan over warps.
struct EpPlanArgs {
  const long long* ids;  // [S]
  int* send_slot;        // [world * cap]
  int* send_expert;      // [world * cap]
  int* slot_pos;         // [S]
  int* counts;           // [world]
  int* err;
  int S, E, world, cap;
};

constexpr int EP_THREADS = 1024;
constexpr int EP_MAX_WORLD = 64;

__global__ void __launch_bounds__(EP_THREADS, 1) ep_plan_kernel(const EpPlanArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int s_warp[32][EP_MAX_WORLD];
  __shared__ int s_base[EP_MAX_WORLD];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int epr = p.E / p.world;
  const long long nb = (long long)p.world * p.cap;
  for (long long i = tid; i < nb; i += EP_THREADS) {
    p.send_slot[i] = -1;
    p.send_expert[i] = -1;
  }
  if (tid < p.world) s_base[tid] = 0;
  const unsigned lt = (1u << lane) - 1u;
  for (int base = 0; base < p.S; base += EP_THREADS) {
    for (int i = tid; i < 32 * EP_MAX_WORLD; i += EP_THREADS) (&s_warp[0][0])[i] = 0;
    __syncthreads();
    const int s = base + tid;
    int peer = -1, lid = -1;
    if (s < p.S) {
      const long long e = p.ids[s];
      if (e >= 0 && e < p.E) {
        peer = (int)(e / epr);
        lid = (int)(e - (long long)peer * epr);
      } else if (e >= p.E) {
        atomicOr(p.err, SIMSD_DEV_ERR_BAD_INDEX);
      }
    }
    const unsigned same = __match_any_sync(0xffffffffu, peer);
    const int rank_in_warp = __popc(same & lt);
    if (peer >= 0 && lane == __ffs(same) - 1) s_warp[warp][peer] = __popc(same);
    __syncthreads();
    if (tid < p.world) {
      int run = s_base[tid];
      for (int w = 0; w < 32; ++w) {
        const int v = s_warp[w][tid];
        s_warp[w][tid] = run;
        run += v;
      }
      s_base[tid] = run;
    }
    __syncthreads();
    if (s < p.S) {
      int slot_pos = -1;
      if (peer >= 0) {
        const int pos = s_warp[warp][peer] + rank_in_warp;
        if (pos < p.cap) {
          slot_pos = peer * p.cap + pos;
          p.send_slot[slot_pos] = s;
          p.send_expert[slot_pos] = lid;
        } else {
          atomicOr(p.err, SIMSD_DEV_ERR_CAPACITY);
        }
      }
      p.slot_pos[s] = slot_pos;
    }
    __syncthreads();
  }
  if (tid < p.world) p.counts[tid] = s_base[tid];
}

}  // namespace simsd
