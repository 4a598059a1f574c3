// Stride-generic CUDA-core path of the thin GEMM, for what the tcgen05 kernel
// cannot take: fp32 inputs (the reference requires IEEE fp32, not TF32:
// kernels/thin_linear_fused.py:310, kernels/thin_linear_fused_test.py:65-71),
// strides TMA cannot describe (inner stride != 1, rows not 16-byte aligned:
// kernels/thin_linear_fused_test.py:87-92) and K below one 64-wide block.
//
// One warp owns one output column and up to 8 rows: lanes stride over K with
// fp32 FMA, then a fixed xor-butterfly sums the 32 lane partials, so results
// are bit-reproducible.  Grouped mode (MoE experts) uses the same per-group row
// tables as the tensor-core kernel.
#pragma once
#include "sm100.cuh"

namespace simsd {

constexpr int SIMT_ROWS = 8;
constexpr int SIMT_WARPS = 8;

struct SimtGemmArgs {
  const void* a;            // activations: row r at a + r*lda_m, element stride lda_k
  const void* w;            // weights [groups][rows][K]
  const void* w_up;         // SiLU-mul: up weights (same strides) or nullptr
  const void* bias;         // [N] or nullptr
  void* out;                // out + r*ld_out + col
  const int* group_counts;  // grouped mode rows per group, or nullptr
  int* err;
  long long lda_m, lda_k, ldw_n, ldw_k, ldw_g, ld_out;
  int rows;                 // single mode: M
  int num_groups;
  int N, K;                 // output columns, reduction length
  int dtype;                // 0 bf16, 1 fp16, 2 fp32 (inputs and output)
  int silu;
  int max_chunks;           // gridDim.y bound (grouped mode)
};

__global__ void __launch_bounds__(SIMT_WARPS * 32) simt_gemm_kernel(const SimtGemmArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ int s_row_prefix[1025];
  __shared__ int s_chunk_prefix[1025];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * SIMT_WARPS + warp;
  const int chunk = blockIdx.y;

  int group = 0, row0, nrows;
  if (p.group_counts == nullptr) {
    row0 = chunk * SIMT_ROWS;
    nrows = min(SIMT_ROWS, p.rows - row0);
  } else {
    const int G = p.num_groups;
    if (threadIdx.x < 32) {
      int run_r = 0, run_c = 0;
      for (int base = 0; base < G; base += 32) {
        const int g = base + lane;
        int c = (g < G) ? p.group_counts[g] : 0;
        if (c < 0) c = 0;
        int ch = (c + SIMT_ROWS - 1) / SIMT_ROWS;
        for (int o = 1; o < 32; o <<= 1) {
          const int c2 = __shfl_up_sync(0xffffffffu, c, o);
          const int h2 = __shfl_up_sync(0xffffffffu, ch, o);
          if (lane >= o) { c += c2; ch += h2; }
        }
        if (g < G) { s_row_prefix[g + 1] = run_r + c; s_chunk_prefix[g + 1] = run_c + ch; }
        run_r += __shfl_sync(0xffffffffu, c, 31);
        run_c += __shfl_sync(0xffffffffu, ch, 31);
      }
      if (lane == 0) { s_row_prefix[0] = 0; s_chunk_prefix[0] = 0; }
    }
    __syncthreads();
    if (chunk >= s_chunk_prefix[G]) return;
    int lo = 0, hi = G - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_chunk_prefix[mid] <= chunk) lo = mid; else hi = mid - 1;
    }
    group = lo;
    row0 = s_row_prefix[lo] + (chunk - s_chunk_prefix[lo]) * SIMT_ROWS;
    nrows = min(SIMT_ROWS, s_row_prefix[lo + 1] - row0);
  }
  if (col >= p.N || nrows <= 0) return;

  const long long wbase = (long long)group * p.ldw_g + (long long)col * p.ldw_n;
  float acc[SIMT_ROWS], acu[SIMT_ROWS];
#pragma unroll
  for (int r = 0; r < SIMT_ROWS; ++r) { acc[r] = 0.0f; acu[r] = 0.0f; }
  for (int k = lane; k < p.K; k += 32) {
    const long long wi = wbase + (long long)k * p.ldw_k;
    const float wv = load_f(p.w, wi, p.dtype);
    const float uv = p.silu ? load_f(p.w_up, wi, p.dtype) : 0.0f;
#pragma unroll
    for (int r = 0; r < SIMT_ROWS; ++r) {
      if (r < nrows) {
        const float xv = load_f(p.a, (long long)(row0 + r) * p.lda_m + (long long)k * p.lda_k, p.dtype);
        acc[r] = __fmaf_rn(xv, wv, acc[r]);
        if (p.silu) acu[r] = __fmaf_rn(xv, uv, acu[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < SIMT_ROWS; ++r) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc[r] = __fadd_rn(acc[r], __shfl_xor_sync(0xffffffffu, acc[r], o));
      if (p.silu) acu[r] = __fadd_rn(acu[r], __shfl_xor_sync(0xffffffffu, acu[r], o));
    }
  }
  const float bv = p.bias ? load_f(p.bias, col, p.dtype) : 0.0f;
#pragma unroll
  for (int r = 0; r < SIMT_ROWS; ++r) {
    if (lane == r && r < nrows) {
      const float v = p.silu ? silu_mul(acc[r], acu[r]) : __fadd_rn(acc[r], bv);
      store_f(p.out, (long long)(row0 + r) * p.ld_out + col, v, p.dtype);
    }
  }
}

}  // namespace simsd
