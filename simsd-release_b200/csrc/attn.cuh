// Verify attention over a static KV cache with native GQA (no expanded K/V):
// o[t, h, :] = softmax_j(scale * q[h, t] . k[g, j] | mask[t, j]) v[g, j],
// g = h / (Hq / Hk), keys j < Lk.  Split over keys (flash decoding): CTA (c, g)
// takes keys [c KC, (c + 1) KC) for the G = Hq / Hk query heads of KV head g,
// i.e. a tile of R = G * L query rows (row = head_in_group * L + t), computes
// S = Q K^T and O = P V on the tensor cores (mma.sync m16n8k16, bf16 in, fp32
// accumulate), and leaves the chunk's (O, row max, row sum) in the workspace;
// attn_combine_kernel merges the chunks of each row and writes o in the
// [L, Hq, D] layout the output projection reads.
//
// Softmax in fp32 with exp2 on log2-scaled scores; P rounded to bf16 for the
// second product (as flash attention does); a masked key (or one past Lk)
// scores -inf, and a chunk with every key of a row masked contributes nothing.
// A row with every key masked comes out as zeros.
//
// Replaces torch SDPA with enable_gqa over the 4x-expanded KV of the
// reference's verify (speculative_decoding/cache_aware.py:195-215, the
// multi-block mask of sdar/new_attn_multi_block.py).
#pragma once
#include "sm100.cuh"

namespace simsd {

constexpr int ATT_D = 128;        // head dim
constexpr int ATT_KC = 128;       // keys per CTA
constexpr int ATT_R = 128;        // query rows per CTA (G * L <= 128)
constexpr int ATT_THREADS = 256;  // 8 warps x 16 rows

struct AttnArgs {
  const void* q;        // [Hq, L, D] bf16 contiguous
  const void* k;        // [Hk, cap, D] bf16 contiguous
  const void* v;        // [Hk, cap, D]
  const uint8_t* mask;  // [L, ldm] (nonzero = attend)
  void* o;              // [L, Hq, D] bf16 contiguous
  float* part_o;        // [Hk][nchunks][R][D]
  float* part_ml;       // [Hk][nchunks][R][2]  (row max in log2 units, row sum)
  long long cap, ldm;
  int Hq, Hk, L, Lk, nchunks;
  float scale_log2;     // softmax scale * log2(e)
};

// 16-byte chunk c of row r of a [rows][128] bf16 tile: XOR-swizzled so that the
// 8 rows an ldmatrix phase reads fall in 8 different bank groups
__device__ __forceinline__ uint32_t att_off(int r, int c) { return (uint32_t)(r * 256 + ((c ^ (r & 7)) << 4)); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& a, uint32_t& b, uint32_t& c, uint32_t& d) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d) : "r"(addr));
}
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  const uint32_t l = __bfloat16_as_ushort(__float2bfloat16_rn(lo));
  const uint32_t h = __bfloat16_as_ushort(__float2bfloat16_rn(hi));
  return l | (h << 16);
}

// rows [0, nrows) of a [*][128] bf16 global matrix into a swizzled tile; the
// rest of the tile's 128 rows zero
__device__ __forceinline__ void att_load_tile(uint8_t* tile, const uint8_t* src, int nrows) {
  for (int i = threadIdx.x; i < 128 * 16; i += ATT_THREADS) {
    const int r = i >> 4, c = i & 15;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (r < nrows) v = *reinterpret_cast<const uint4*>(src + (long long)r * 256 + c * 16);
    *reinterpret_cast<uint4*>(tile + att_off(r, c)) = v;
  }
}

__global__ void __launch_bounds__(ATT_THREADS) attn_split_kernel(const AttnArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  extern __shared__ __align__(128) uint8_t att_smem[];
  uint8_t* Qs = att_smem;
  uint8_t* Ks = att_smem + 32768;
  uint8_t* Vs = att_smem + 65536;
  const int c = blockIdx.x, g = blockIdx.y;
  const int G = p.Hq / p.Hk;
  const int R = G * p.L;
  const int k0 = c * ATT_KC;
  const int nk = min(ATT_KC, p.Lk - k0);
  const uint8_t* qsrc = reinterpret_cast<const uint8_t*>(p.q) + (long long)g * G * p.L * ATT_D * 2;
  const uint8_t* ksrc = reinterpret_cast<const uint8_t*>(p.k) + ((long long)g * p.cap + k0) * ATT_D * 2;
  const uint8_t* vsrc = reinterpret_cast<const uint8_t*>(p.v) + ((long long)g * p.cap + k0) * ATT_D * 2;
  att_load_tile(Qs, qsrc, R);
  att_load_tile(Ks, ksrc, nk);
  att_load_tile(Vs, vsrc, nk);
  __syncthreads();

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int r0 = warp * 16;
  if (r0 >= R) return;
  const uint32_t qs = smem_u32(Qs), ks = smem_u32(Ks), vs = smem_u32(Vs);
  const int lr = lane & 7, lm = lane >> 3;   // ldmatrix: row within matrix, matrix index

  // S = Q K^T for rows r0..r0+15, keys 0..127: 16 n8 tiles
  float s[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
    uint32_t a0, a1, a2, a3;
    // A: matrices (rows 0-7, k 0-7), (rows 8-15, k 0-7), (rows 0-7, k 8-15), (rows 8-15, k 8-15)
    ldsm_x4(qs + att_off(r0 + (lm & 1) * 8 + lr, 2 * kk + (lm >> 1)), a0, a1, a2, a3);
#pragma unroll
    for (int j2 = 0; j2 < 8; ++j2) {
      uint32_t b0, b1, b2, b3;
      // B from K rows (keys): (keys 0-7, k 0-7), (keys 0-7, k 8-15), (keys 8-15, k 0-7), (keys 8-15, k 8-15)
      ldsm_x4(ks + att_off(16 * j2 + (lm >> 1) * 8 + lr, 2 * kk + (lm & 1)), b0, b1, b2, b3);
      mma_bf16(s[2 * j2], a0, a1, a2, a3, b0, b1);
      mma_bf16(s[2 * j2 + 1], a0, a1, a2, a3, b2, b3);
    }
  }

  // scale, mask, row max (rows r0 + gid and r0 + gid + 8)
  const int rowA = r0 + gid, rowB = rowA + 8;
  const int tA = rowA % p.L, tB = rowB % p.L;
  const uint8_t* mA = p.mask + (long long)tA * p.ldm + k0;
  const uint8_t* mB = p.mask + (long long)tB * p.ldm + k0;
  const float NEG = -__int_as_float(0x7f800000);
  float mxA = NEG, mxB = NEG;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int key = 8 * j + 2 * tig + e;
      const bool okA = key < nk && rowA < R && mA[key] != 0;
      const bool okB = key < nk && rowB < R && mB[key] != 0;
      s[j][e] = okA ? __fmul_rn(s[j][e], p.scale_log2) : NEG;
      s[j][2 + e] = okB ? __fmul_rn(s[j][2 + e], p.scale_log2) : NEG;
      mxA = fmaxf(mxA, s[j][e]);
      mxB = fmaxf(mxB, s[j][2 + e]);
    }
  }
#pragma unroll
  for (int m = 1; m <= 2; m <<= 1) {
    mxA = fmaxf(mxA, __shfl_xor_sync(0xffffffffu, mxA, m));
    mxB = fmaxf(mxB, __shfl_xor_sync(0xffffffffu, mxB, m));
  }
  const float bA = mxA == NEG ? 0.0f : mxA, bB = mxB == NEG ? 0.0f : mxB;
  float lA = 0.0f, lB = 0.0f;
  uint32_t pa[8][4];   // P as A fragments: k16 block kk from S tiles 2kk, 2kk+1
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float p0 = exp2f(s[j][0] - bA), p1 = exp2f(s[j][1] - bA);
    const float p2 = exp2f(s[j][2] - bB), p3 = exp2f(s[j][3] - bB);
    lA += p0 + p1;
    lB += p2 + p3;
    const int kk = j >> 1;
    if ((j & 1) == 0) {
      pa[kk][0] = pack_bf16(p0, p1);
      pa[kk][1] = pack_bf16(p2, p3);
    } else {
      pa[kk][2] = pack_bf16(p0, p1);
      pa[kk][3] = pack_bf16(p2, p3);
    }
  }
#pragma unroll
  for (int m = 1; m <= 2; m <<= 1) {
    lA += __shfl_xor_sync(0xffffffffu, lA, m);
    lB += __shfl_xor_sync(0xffffffffu, lB, m);
  }

  // O = P V for rows r0..r0+15, dims 0..127: 16 n8 tiles
  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.0f;
#pragma unroll
  for (int kk = 0; kk < 8; ++kk) {
#pragma unroll
    for (int j2 = 0; j2 < 8; ++j2) {
      uint32_t b0, b1, b2, b3;
      // B = V[keys 16kk.., dims 16j2..] transposed: (keys 0-7, d 0-7), (keys 8-15, d 0-7),
      // (keys 0-7, d 8-15), (keys 8-15, d 8-15)
      ldsm_x4_t(vs + att_off(16 * kk + (lm & 1) * 8 + lr, 2 * j2 + (lm >> 1)), b0, b1, b2, b3);
      mma_bf16(o[2 * j2], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
      mma_bf16(o[2 * j2 + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
    }
  }

  // the chunk's partials
  float* po = p.part_o + (((long long)g * p.nchunks + c) * ATT_R) * ATT_D;
  float* pml = p.part_ml + (((long long)g * p.nchunks + c) * ATT_R) * 2;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * tig;
    if (rowA < R) *reinterpret_cast<float2*>(po + (long long)rowA * ATT_D + d) = make_float2(o[j][0], o[j][1]);
    if (rowB < R) *reinterpret_cast<float2*>(po + (long long)rowB * ATT_D + d) = make_float2(o[j][2], o[j][3]);
  }
  if (tig == 0) {
    if (rowA < R) *reinterpret_cast<float2*>(pml + rowA * 2) = make_float2(mxA, lA);
    if (rowB < R) *reinterpret_cast<float2*>(pml + rowB * 2) = make_float2(mxB, lB);
  }
}

// One warp per (KV head, row): o = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.
__global__ void __launch_bounds__(256) attn_combine_kernel(const AttnArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  const int G = p.Hq / p.Hk;
  const int R = G * p.L;
  const long long unit = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (unit >= (long long)p.Hk * R) return;
  const int lane = threadIdx.x & 31;
  const int g = (int)(unit / R), row = (int)(unit - (long long)g * R);
  const float NEG = -__int_as_float(0x7f800000);
  float M = NEG;
  for (int c = 0; c < p.nchunks; ++c)
    M = fmaxf(M, p.part_ml[(((long long)g * p.nchunks + c) * ATT_R + row) * 2]);
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float den = 0.0f;
  if (M != NEG) {
    for (int c = 0; c < p.nchunks; ++c) {
      const long long base = ((long long)g * p.nchunks + c) * ATT_R + row;
      const float2 ml = *reinterpret_cast<const float2*>(p.part_ml + base * 2);
      if (ml.x == NEG) continue;
      const float w = exp2f(ml.x - M);
      den += w * ml.y;
      const float4 ov = reinterpret_cast<const float4*>(p.part_o + base * ATT_D)[lane];
      acc.x += w * ov.x;
      acc.y += w * ov.y;
      acc.z += w * ov.z;
      acc.w += w * ov.w;
    }
  }
  const float inv = den > 0.0f ? 1.0f / den : 0.0f;
  const int h = g * G + row / p.L, t = row % p.L;
  uint8_t* dst = reinterpret_cast<uint8_t*>(p.o) + (((long long)t * p.Hq + h) * ATT_D + lane * 4) * 2;
  uint2 pk;
  pk.x = pack_bf16(acc.x * inv, acc.y * inv);
  pk.y = pack_bf16(acc.z * inv, acc.w * inv);
  *reinterpret_cast<uint2*>(dst) = pk;
}

}  // namespace simsd
