// Weight-streaming tcgen05 GEMM for thin activations (the B200 path of
// `_thin_gemv_kernel` in kernels/thin_linear_fused.py:67-136 and of
// `_grouped_gemm_kernel` in kernels/moe_dispatch_fused.py:32-90).
//
//   out[row, col] = sum_k  B[row, k] * A[col, k]          (y = x W^T, nn.Linear layout)
//
// The weight A is the large operand and the activation B has 1..256 rows, so
// the roles are swapped relative to a square GEMM: 128 weight rows fill the
// MMA's M dimension and the activation rows are the MMA's N dimension
// (16..BMAX, a runtime field of the instruction descriptor).  Weight tiles
// (128 rows x 64 K, 16 KiB, 128-byte swizzle) and activation tiles (16-row
// boxes) are staged by TMA into a STAGES-deep shared-memory ring, one elected
// thread issues tcgen05.mma into a double-buffered TMEM accumulator, and four
// epilogue warps read TMEM back with tcgen05.ld.
//
// Work split (stream-K): the iteration space (tile, k-block) is cut into
// gridDim.x contiguous, equal ranges, one per CTA, so every SM streams the same
// number of weight bytes whatever the shape.  A tile that lies inside one CTA's
// range is finished by that CTA's epilogue.  A tile whose K range is spread over
// several CTAs is reduced deterministically by tc_fixup_kernel, launched right
// after: each CTA parks its fp32 partial in a fixed slot, and the fixup sums the
// slots of each split tile in K order, every tile in parallel.  No CTA waits on
// another and no atomics are involved, and the sum order depends only on the
// shape and grid size, so results are bit-identical across calls and graph
// replays (the property tested at kernels/thin_linear_fused_test.py:130-151).
//
// Grouped mode: B rows are grouped (MoE experts, rows sorted by expert);
// group g owns rows [offset_g, offset_g + count_g) of B and of the output, and
// A is a 3-D tensor [groups, rows, K].  Tiles never straddle groups.
//
// SiLU-mul mode: A rows 0-63 of a tile come from the gate weight and rows
// 64-127 from the up weight (same output columns), so the epilogue writes
// silu(x Wg^T) * (x Wu^T) without a DRAM round trip for the two halves.
#pragma once
#include "sm100.cuh"

namespace simsd {

constexpr int TC_THREADS = 192;            // warps 0-3 epilogue, 4 TMA, 5 MMA
constexpr int TC_A_BYTES = 128 * 128;      // 128 weight rows x 64 bf16
constexpr int TC_BOX_ROWS = 16;            // activation rows per MMA N step (tcgen05 N granularity)
// The activation tile of a stage atom is one TMA box of BMAX rows x 64 K
// (128-byte rows, SW128); rows past the valid ones (beyond M, or the next
// expert's rows in grouped mode) are loaded or zero-filled and never stored.
constexpr int TC_MAX_GROUPS = 1024;
constexpr int TC_MAX_GRID = 1024;          // CTAs per launch (segments per tile <= this)
constexpr int WS_COUNTER_BYTES = 256 * 1024;          // head of every workspace (reserved)
constexpr int WS_ERR_OFFSET = WS_COUNTER_BYTES - 64;  // device error word
constexpr int WS_ARGMAX_OFFSET = WS_COUNTER_BYTES - 4096;    // argmax keys [64] u64, then its launch counter
constexpr int WS_MAX_COUNTERS = WS_ARGMAX_OFFSET / 4;          // per-tile arrival counters from offset 0
constexpr int TC_TABLE_INTS = 2 * (TC_MAX_GROUPS + 1);

struct alignas(64) TcGemmArgs {
  CUtensorMap tmA0;          // weights (gate weights in SiLU-mul mode)
  CUtensorMap tmA1;          // up weights (SiLU-mul mode only)
  CUtensorMap tmB;           // activations: 2-D {K, rows}
  void* out;                 // output, row stride ld_out elements
  const void* bias;          // [rows_out] or nullptr (single mode only)
  float* partials;           // [2 * gridDim.x][128 weight rows][BMAX activation rows] fp32
  int* tables;               // grouped mode: row and chunk prefixes for tc_fixup_kernel
  int* counters;             // per-tile arrival counters (zero on entry and exit); nullptr =
                             // split tiles are left to tc_fixup_kernel
  int* err;                  // device error word
  const int* group_counts;   // grouped mode: rows per group; nullptr = single mode
  long long ld_out;
  int num_groups;
  // grouped mode: only groups with cls_lo < rows <= cls_hi take tiles here
  // (cls_hi 0: no upper bound); the others keep their rows but get no chunks,
  // so two launches with different tile heights can split the groups by size
  int cls_lo, cls_hi;
  int single_rows;           // single mode: rows of B (M)
  int kb;                    // number of 64-wide K blocks
  int rows_out;              // valid output columns (N, or I in SiLU-mul mode)
  int row_tiles;             // output-column tiles per group
  int silu;
  int three_d;
  int is_bf16;
  int pdl;                   // launched as a programmatic dependent (see griddep_wait)
  int prefetch;              // ring stages of weights fetched before griddep_wait (single mode, pdl)
  unsigned long long* trace; // optional: 8 %globaltimer stamps per CTA (diagnostics)
};

// KS = 64-wide K atoms per ring stage: each stage reads KS*128 contiguous bytes
// of every weight row it covers, which keeps HBM pages open for longer runs.
// RING_KB bounds the ring: 196 KB gives one CTA per SM the deepest ring; 96 KB
// lets the next launch's CTA share the SM (programmatic dependent launch
// then overlaps its weight prefetch with this kernel's tail).
template <int BMAX, int KS, int RING_KB = 196>
struct TcConfig {
  static constexpr int A_ATOM = TC_A_BYTES;
  static constexpr int B_ATOM = BMAX * 128;
  static constexpr int A_STAGE = KS * A_ATOM;
  static constexpr int B_STAGE = KS * B_ATOM;
  static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
  // the small ring gives up 8 KB so that two CTAs' tails still fit an SM
  static constexpr int RING_BYTES = (RING_KB >= 196 ? RING_KB : RING_KB - 8) * 1024;
  static constexpr int STAGES_RAW = RING_BYTES / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 10 ? 10 : STAGES_RAW;
  static constexpr int TMEM_COLS = (2 * BMAX) < 32 ? 32 : 2 * BMAX;
  // tail: barriers (2*STAGES + 5) x 8, misc ints 16, prefixes 2 x (MAX_GROUPS+1), xbuf 64x16 fp32,
  // output staging 2 x 16 x 128 16-bit
  static constexpr int TAIL_BYTES =
      (2 * STAGES + 5) * 8 + 64 + 2 * (TC_MAX_GROUPS + 1) * 4 + 16 + 64 * 16 * 4 + 16 + 2 * 16 * 128 * 2;
  static constexpr int SMEM_BYTES = 1024 /*align slack*/ + STAGES * STAGE_BYTES + TAIL_BYTES;
  static_assert(STAGES >= 2, "ring needs two stages");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
};

struct TileInfo {
  int group, rtile, row0, nrows;
  bool reread;   // a later row chunk of this tile reads the same weight tile
};

// Tile j -> (group, output-column tile, first B row, B rows).  Tiles are
// ordered (group, column tile, row chunk): the row chunks that share a weight
// tile (a busy expert's rows beyond BMAX, or M > BMAX in single mode) run back
// to back, mostly on one CTA, so the weight tile streams from HBM once and the
// later chunks re-read it from L2.  The activation chunks are small and stay
// L2-resident (evict_last), so walking them per column tile costs no HBM.
template <int BMAX>
__device__ __forceinline__ TileInfo decode_tile(int j, const TcGemmArgs& p,
                                                const int* row_prefix, const int* chunk_prefix) {
  TileInfo ti;
  if (p.group_counts == nullptr) {
    const int nch = (p.single_rows + BMAX - 1) / BMAX;
    ti.rtile = j / nch;
    const int chunk = j - ti.rtile * nch;
    ti.group = 0;
    ti.row0 = chunk * BMAX;
    ti.nrows = min(BMAX, p.single_rows - ti.row0);
    ti.reread = chunk + 1 < nch;
  } else {
    // group g holds tiles [chunk_prefix[g], chunk_prefix[g+1]) x row_tiles, so
    // g is the largest with chunk_prefix[g] <= j / row_tiles (groups with zero
    // chunks are skipped)
    const int pc = j / p.row_tiles;
    int lo = 0, hi = p.num_groups - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (chunk_prefix[mid] <= pc) lo = mid; else hi = mid - 1;
    }
    ti.group = lo;
    const int nch = chunk_prefix[lo + 1] - chunk_prefix[lo];
    const int local = j - chunk_prefix[lo] * p.row_tiles;
    ti.rtile = local / nch;
    const int lc = local - ti.rtile * nch;
    ti.row0 = row_prefix[lo] + lc * BMAX;
    ti.nrows = min(BMAX, row_prefix[lo + 1] - ti.row0);
    ti.reread = lc + 1 < nch;
  }
  return ti;
}

// Work split of a grouped (MoE) GEMM with at least two tiles per CTA: whole
// tiles, balanced by count (the experts' tiles are many and alike, so this
// loses little balance and needs no split-K partials).  Otherwise, and always
// in single mode, the stream-K split below.
__host__ __device__ __forceinline__ bool tc_whole_tiles(bool grouped, int total_tiles, int grid) {
  return grouped && total_tiles >= 2 * grid;
}

// Stream-K partition of `iters` (tile, k-block) iterations over G CTAs: the
// first r = iters % G CTAs take q + 1 = iters / G + 1 iterations, the others q.
// 32-bit throughout (the host keeps iters below 2^31): these run on every CTA's
// start-up path, where 64-bit divisions cost close to a microsecond.
struct SkSplit {
  int q, r;
  __host__ __device__ __forceinline__ SkSplit(int iters, int G) : q(iters / G), r(iters - (iters / G) * G) {}
  __host__ __device__ __forceinline__ int start(int c) const { return c * q + (c < r ? c : r); }
  // CTA whose range holds iteration i
  __host__ __device__ __forceinline__ int owner(int i) const {
    const int t = r * (q + 1);
    return i < t ? i / (q + 1) : r + (i - t) / q;
  }
};

// Sum the nseg partial slots of split tile `tile` (contributors c_first ..
// c_first + nseg - 1, in K order) for activation rows ch*16 .. ch*16+15 and
// apply the epilogue: bias, or SiLU(gate) * up across the two 64-row halves
// (threads 0-63 then take rows 0-7 of the chunk and threads 64-127 rows 8-15).
// Called by 128 threads, `row` = thread index; used by the GEMM's last
// contributor and by tc_fixup_kernel, so both produce the same bits.
template <int BMAX>
__device__ __forceinline__ void reduce_split_chunk(const float* partials, const SkSplit& sk, int kb, int tile,
                                                   int c_first, int nseg, const TileInfo& ti, int ch, int row,
                                                   char* outp, long long ld_out, const void* bias, int rows_out,
                                                   int silu, int odt) {
  auto slot_of = [&](int i) -> long long {
    const int cc = c_first + i;
    return 2LL * cc + ((tile == sk.start(cc) / kb) ? 0 : 1);
  };
  if (!silu) {
    const int col = ti.rtile * 128 + row;
    float acc[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
    for (int i0 = 0; i0 < nseg; i0 += 8) {
      float4 buf[8][4];
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (i0 + q < nseg) {
          const float4* src = reinterpret_cast<const float4*>(
              partials + slot_of(i0 + q) * (BMAX * 128) + (long long)row * BMAX + ch * 16);
#pragma unroll
          for (int u = 0; u < 4; ++u) buf[q][u] = __ldcg(src + u);
        }
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (i0 + q < nseg) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc[4 * u] = __fadd_rn(acc[4 * u], buf[q][u].x);
            acc[4 * u + 1] = __fadd_rn(acc[4 * u + 1], buf[q][u].y);
            acc[4 * u + 2] = __fadd_rn(acc[4 * u + 2], buf[q][u].z);
            acc[4 * u + 3] = __fadd_rn(acc[4 * u + 3], buf[q][u].w);
          }
        }
    }
    if (col < rows_out) {
      const float bv = bias ? load_f(bias, col, odt) : 0.0f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int t = ch * 16 + j;
        if (t < ti.nrows) store_f(outp, (long long)(ti.row0 + t) * ld_out + col, __fadd_rn(acc[j], bv), odt);
      }
    }
  } else {
    // 64 gate rows and their 64 up rows; threads 0-63 take activation rows
    // 0-7 of the chunk, threads 64-127 rows 8-15
    const int i = row & 63;
    const int half = row >> 6;
    const int col = ti.rtile * 64 + i;
    float ag[8], au[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) { ag[j] = 0.0f; au[j] = 0.0f; }
    for (int i0 = 0; i0 < nseg; i0 += 4) {
      float4 bg[4][2], bu[4][2];
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i0 + q < nseg) {
          const float* base = partials + slot_of(i0 + q) * (BMAX * 128) + ch * 16 + half * 8;
          const float4* sg = reinterpret_cast<const float4*>(base + (long long)i * BMAX);
          const float4* su = reinterpret_cast<const float4*>(base + (long long)(64 + i) * BMAX);
#pragma unroll
          for (int u = 0; u < 2; ++u) { bg[q][u] = __ldcg(sg + u); bu[q][u] = __ldcg(su + u); }
        }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        if (i0 + q < nseg) {
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            ag[4 * u] = __fadd_rn(ag[4 * u], bg[q][u].x);
            ag[4 * u + 1] = __fadd_rn(ag[4 * u + 1], bg[q][u].y);
            ag[4 * u + 2] = __fadd_rn(ag[4 * u + 2], bg[q][u].z);
            ag[4 * u + 3] = __fadd_rn(ag[4 * u + 3], bg[q][u].w);
            au[4 * u] = __fadd_rn(au[4 * u], bu[q][u].x);
            au[4 * u + 1] = __fadd_rn(au[4 * u + 1], bu[q][u].y);
            au[4 * u + 2] = __fadd_rn(au[4 * u + 2], bu[q][u].z);
            au[4 * u + 3] = __fadd_rn(au[4 * u + 3], bu[q][u].w);
          }
        }
    }
    if (col < rows_out) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int t = ch * 16 + half * 8 + j;
        if (t < ti.nrows) store_f(outp, (long long)(ti.row0 + t) * ld_out + col, silu_mul(ag[j], au[j]), odt);
      }
    }
  }
}

template <int BMAX, int KS, int RING_KB>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_kernel(const __grid_constant__ TcGemmArgs p) {
  using Cfg = TcConfig<BMAX, KS, RING_KB>;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_STAGE;
  uint8_t* tail = sB + STAGES * Cfg::B_STAGE;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(tail);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint64_t* drain_bar = acce_bar + 2;       // [1]
  int* misc = reinterpret_cast<int*>(drain_bar + 1);  // 16 ints
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort_flag = misc + 1;
  int* sh_total_chunks = misc + 3;
  volatile int* sh_last = misc + 4;         // epilogue: this CTA reduces the tile it just left
  int* row_prefix = misc + 16;                       // [num_groups + 1]
  int* chunk_prefix = row_prefix + (TC_MAX_GROUPS + 1);
  float* xbuf = reinterpret_cast<float*>(chunk_prefix + (TC_MAX_GROUPS + 1) + 4);  // [16][64]
  uint16_t* sout = reinterpret_cast<uint16_t*>((reinterpret_cast<uintptr_t>(xbuf + 16 * 64) + 15) &
                                               ~uintptr_t(15));                      // [2][16][128]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (p.trace && tid == 0) p.trace[blockIdx.x * 8 + 0] = globaltimer_ns();

  // ---- set-up: barriers, TMEM, group tables
  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&accf_bar[a]), 1);
      mbar_init(smem_u32(&acce_bar[a]), 128);
    }
    mbar_init(smem_u32(drain_bar), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&p.tmA0);
    if (p.silu) prefetch_tmap(&p.tmA1);
    prefetch_tmap(&p.tmB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) griddep_launch_dependents();
  long long total_tiles;
  if (p.group_counts != nullptr) {
    // the counts come from the align kernel just before this one
    if (p.pdl) griddep_wait();
    const int G = p.num_groups;
    for (int g = tid; g < G; g += TC_THREADS) row_prefix[g + 1] = p.group_counts[g];
    __syncthreads();
    if (warp == 0) {
      // inclusive scans of counts and of chunk counts, 32 groups at a time
      int run_rows = 0, run_chunks = 0;
      for (int base = 0; base < G; base += 32) {
        const int g = base + lane;
        int c = (g < G) ? row_prefix[g + 1] : 0;
        int ch = (c > p.cls_lo && (p.cls_hi == 0 || c <= p.cls_hi)) ? (c + BMAX - 1) / BMAX : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int c2 = __shfl_up_sync(0xffffffffu, c, o);
          const int h2 = __shfl_up_sync(0xffffffffu, ch, o);
          if (lane >= o) { c += c2; ch += h2; }
        }
        if (g < G) {
          row_prefix[g + 1] = run_rows + c;
          chunk_prefix[g + 1] = run_chunks + ch;
        }
        run_rows += __shfl_sync(0xffffffffu, c, 31);
        run_chunks += __shfl_sync(0xffffffffu, ch, 31);
      }
      if (lane == 0) {
        row_prefix[0] = 0;
        chunk_prefix[0] = 0;
        *sh_total_chunks = run_chunks;
      }
    }
    tc_fence_before();
    __syncthreads();
    total_tiles = (long long)(*sh_total_chunks) * p.row_tiles;
    if (blockIdx.x == 0 && p.tables != nullptr)
      for (int g = tid; g <= G; g += TC_THREADS) {
        p.tables[g] = row_prefix[g];
        p.tables[TC_MAX_GROUPS + 1 + g] = chunk_prefix[g];
      }
  } else {
    tc_fence_before();
    __syncthreads();
    total_tiles = (long long)((p.single_rows + BMAX - 1) / BMAX) * p.row_tiles;
  }
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (p.trace && tid == 0) p.trace[blockIdx.x * 8 + 1] = globaltimer_ns();

  // Partition over G = min(gridDim.x, iters) CTAs so that every partition is
  // non-empty (the tile count is data-dependent in grouped mode); CTAs beyond
  // G have no work.
  const int kb = p.kb;
  const int iters = (int)total_tiles * kb;
  const int G = min((int)gridDim.x, iters);
  const int c = blockIdx.x;
  const SkSplit sk(iters, G > 0 ? G : 1);
  int it_begin = 0, it_end = 0;
  int tstride = 1;   // tiles between one tile of this CTA and its next
  if (tc_whole_tiles(p.group_counts != nullptr, (int)total_tiles, (int)gridDim.x)) {
    // grouped GEMM with at least two tiles per CTA: whole tiles dealt round
    // robin (tile c, c + grid, ...) — no split tile, so no partials and nothing
    // for the fixup.  Dealing rather than cutting contiguous runs spreads the
    // tall row chunks of a busy group (the shared expert is the last group) over
    // all CTAs, and the row chunks that share a weight tile run at the same time
    // on neighbouring CTAs, so the weight tile still streams from HBM once.
    it_begin = c * kb;
    it_end = (int)total_tiles * kb;
    tstride = (int)gridDim.x;
  } else if (c < G) {
    it_begin = sk.start(c);
    it_end = sk.start(c + 1);
  }
  // the iteration after tile `tile` whose K blocks end at kb1: the rest of a
  // split range, or the first K block of this CTA's next tile
  auto next_it = [&](int tile, int kb1) -> int {
    if (kb1 < kb) return tile * kb + kb1;
    const long long nx = (long long)(tile + tstride) * kb;
    return nx < it_end ? (int)nx : it_end;
  };

  if (warp == 4) {
    // ================= TMA producer
    if (lane == 0) {
      // weights stream through L2 evict-first, except for a tile that a later
      // row chunk reads again (normal priority keeps it for that re-read)
      const uint64_t pol_w_last = policy_evict_first();
      const uint64_t pol_w_keep = policy_evict_normal();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;        // stages that have ever been armed
      uint32_t last_parity = 0;        // parity of each stage's last arming
      bool ok = true;
      // Programmatic dependent launch, single mode: the weights are not written
      // by the kernel before this one, so the first ring of weight tiles is
      // fetched before griddep_wait(); the activation boxes of those stages are
      // issued right after the wait.  Everything that reads the activations or
      // writes memory (MMA, epilogue, fixup) sits behind those loads.
      bool dep_ready = !(p.pdl && p.group_counts == nullptr);
      int npend = 0;
      bool traced_first = false;
      uint32_t pend_dst[Cfg::STAGES], pend_bar[Cfg::STAGES];
      int pend_k0[Cfg::STAGES], pend_na[Cfg::STAGES], pend_row0[Cfg::STAGES];
      auto flush_pending = [&]() {
        griddep_wait();
        dep_ready = true;
        for (int q = 0; q < npend; ++q)
          for (int at = 0; at < pend_na[q]; ++at)
            tma_load_2d(pend_dst[q] + at * Cfg::B_ATOM, &p.tmB, pend_bar[q], pend_k0[q] + at * 64, pend_row0[q], pol_x);
        npend = 0;
      };
      for (int it = it_begin; ok && it < it_end;) {
        const int tile = it / kb;
        const int kb0 = it - tile * kb;
        const int kb1 = min(kb, it_end - tile * kb);
        const TileInfo ti = decode_tile<BMAX>(tile, p, row_prefix, chunk_prefix);
        const uint64_t pol_w = ti.reread ? pol_w_keep : pol_w_last;
        for (int k = kb0; k < kb1; k += KS) {
          const int na = min(KS, kb1 - k);
          if (!dep_ready && npend >= min(STAGES, p.prefetch)) flush_pending();
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, na * (TC_A_BYTES + Cfg::B_ATOM));
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          const uint32_t b_dst = smem_u32(sB + stage * Cfg::B_STAGE);
          for (int at = 0; at < na; ++at) {
            const uint32_t a_dst = smem_u32(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM);
            const int k0 = (k + at) * 64;
            if (p.silu) {
              const int r0 = ti.rtile * 64;
              if (p.three_d) {
                tma_load_3d(a_dst, &p.tmA0, fb, k0, r0, ti.group, pol_w);
                tma_load_3d(a_dst + 8192, &p.tmA1, fb, k0, r0, ti.group, pol_w);
              } else {
                tma_load_2d(a_dst, &p.tmA0, fb, k0, r0, pol_w);
                tma_load_2d(a_dst + 8192, &p.tmA1, fb, k0, r0, pol_w);
              }
            } else {
              const int r0 = ti.rtile * 128;
              if (p.three_d) tma_load_3d(a_dst, &p.tmA0, fb, k0, r0, ti.group, pol_w);
              else tma_load_2d(a_dst, &p.tmA0, fb, k0, r0, pol_w);
            }
            if (dep_ready) tma_load_2d(b_dst + at * Cfg::B_ATOM, &p.tmB, fb, k0, ti.row0, pol_x);
          }
          if (p.trace && !traced_first) { p.trace[blockIdx.x * 8 + 2] = globaltimer_ns(); traced_first = true; }
          if (!dep_ready) {
            pend_dst[npend] = b_dst;
            pend_bar[npend] = fb;
            pend_k0[npend] = k * 64;
            pend_na[npend] = na;
            pend_row0[npend] = ti.row0;
            ++npend;
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        it = next_it(tile, kb1);
      }
      // fewer iterations than ring stages, or aborting with weight-only stages
      // armed: their activation boxes still have to land
      if (!dep_ready) flush_pending();
      if (p.trace) p.trace[blockIdx.x * 8 + 4] = globaltimer_ns();
      if (!ok) {
        // aborting: make sure no TMA copy is still landing in shared memory
        for (int s = 0; s < STAGES; ++s)
          if (issued_mask & (1u << s))
            mbar_wait_drain(smem_u32(&full_bar[s]), (last_parity >> s) & 1u, 100000000ull);
      }
    }
  } else if (warp == 5) {
    // ================= MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc_iter = 0;
      bool ok = true;
      bool issued_any = false;
      for (int it = it_begin; ok && it < it_end;) {
        const int tile = it / kb;
        const int kb0 = it - tile * kb;
        const int kb1 = min(kb, it_end - tile * kb);
        const TileInfo ti = decode_tile<BMAX>(tile, p, row_prefix, chunk_prefix);
        const int nb = (ti.nrows + TC_BOX_ROWS - 1) / TC_BOX_ROWS;
        const uint32_t idesc = make_idesc_f16(p.is_bf16, 128, nb * TC_BOX_ROWS);
        const int a = acc_iter & 1;
        const uint32_t aphase = (acc_iter >> 1) & 1;
        if (!mbar_wait(smem_u32(&acce_bar[a]), aphase ^ 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BMAX;
        for (int k = kb0; k < kb1; k += KS) {
          const int na = min(KS, kb1 - k);
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          if (p.trace && !issued_any) p.trace[blockIdx.x * 8 + 3] = globaltimer_ns();
          for (int at = 0; at < na; ++at) {
            const uint64_t adesc = make_sw128_desc(smem_u32(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM));
            const uint64_t bdesc = make_sw128_desc(smem_u32(sB + stage * Cfg::B_STAGE + at * Cfg::B_ATOM));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (k > kb0 || at > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          tc_commit(smem_u32(&empty_bar[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(smem_u32(&accf_bar[a]));
        ++acc_iter;
        it = next_it(tile, kb1);
      }
      if (p.trace) p.trace[blockIdx.x * 8 + 5] = globaltimer_ns();
      if (!ok && issued_any) {
        // aborting: wait for the MMAs already issued before TMEM is released
        tc_commit(smem_u32(drain_bar));
        mbar_wait_drain(smem_u32(drain_bar), 0, 100000000ull);
      }
    }
  } else {
    // ================= epilogue warps 0-3: TMEM lanes 32*warp .. 32*warp+31
    const int row = tid;  // 0..127 == TMEM lane == tile row
    // 16-byte output pieces need a 16-byte aligned base and row stride
    const bool out_vec = (reinterpret_cast<uintptr_t>(p.out) & 15) == 0 && (p.ld_out & 7) == 0;
    int acc_iter = 0;
    for (int it = it_begin; it < it_end;) {
      const int tile = it / kb;
      const int kb0 = it - tile * kb;
      const int kb1 = min(kb, it_end - tile * kb);
      const TileInfo ti = decode_tile<BMAX>(tile, p, row_prefix, chunk_prefix);
      const int nb = (ti.nrows + TC_BOX_ROWS - 1) / TC_BOX_ROWS;
      const int a = acc_iter & 1;
      const uint32_t aphase = (acc_iter >> 1) & 1;
      // One decision for all 128 epilogue threads (they share named barriers
      // below, and tcgen05.ld is .sync.aligned): leave together if any gave up.
      const bool got = named_bar_and(1, 128, mbar_wait(smem_u32(&accf_bar[a]), aphase, abort_flag, p.err));
      if (!got) break;
      tc_fence_after();
      const uint32_t t_base = tmem_base + ((uint32_t)(warp * 32) << 16) + a * BMAX;
      const bool whole = (kb0 == 0 && kb1 == kb);
      const int out_col0 = p.silu ? ti.rtile * 64 : ti.rtile * 128;
      char* outp = reinterpret_cast<char*>(p.out);

      if (whole) {
        // Each 16-row chunk of the accumulator is rounded into a shared staging
        // buffer laid out like the output ([activation row][column], 16-bit),
        // then written as 16-byte row pieces: a warp store covers whole output
        // rows instead of one 2-byte column per thread.  Two staging buffers
        // alternate, so one barrier per chunk orders writes and reads (the
        // SiLU*mul path has a second one for the up half in xbuf).
        const int odt = p.is_bf16 ? 0 : 1;
        const int ncols = p.silu ? 64 : 128;
        for (int ch = 0; ch < nb; ++ch) {
          float v[16];
          tmem_ld16(t_base + ch * 16, v);
          tmem_wait_ld();
          if (ch == nb - 1) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce_bar[a]));
          }
          uint16_t* sb = sout + (ch & 1) * (16 * 128);
          if (!p.silu) {
            const int col = out_col0 + row;
            const float bv = (p.bias && col < p.rows_out) ? load_f(p.bias, col, odt) : 0.0f;
#pragma unroll
            for (int j = 0; j < 16; ++j) sb[j * 128 + row] = f32_to_16bit(__fadd_rn(v[j], bv), odt);
          } else {
            // gate row i (thread i) and up row i (thread 64 + i) meet through
            // xbuf; thread i computes activation rows 0-7 of pair i and thread
            // 64 + i rows 8-15, so all four warps share the SiLU*mul work
            float* xg = xbuf;            // [8][64] gate values of rows 8-15
            float* xu = xbuf + 8 * 64;   // [8][64] up values of rows 0-7
            const int pr = row & 63;
            if (row < 64) {
#pragma unroll
              for (int j = 0; j < 8; ++j) xg[j * 64 + pr] = v[8 + j];
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) xu[j * 64 + pr] = v[j];
            }
            named_bar_sync(1, 128);
            if (row < 64) {
#pragma unroll
              for (int j = 0; j < 8; ++j) sb[j * 64 + pr] = f32_to_16bit(silu_mul(v[j], xu[j * 64 + pr]), odt);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                sb[(8 + j) * 64 + pr] = f32_to_16bit(silu_mul(xg[j * 64 + pr], v[8 + j]), odt);
            }
          }
          named_bar_sync(1, 128);
          // row pieces of 8 columns: ncols / 8 per activation row, 16 rows
          const int per_row = ncols >> 3;
          for (int pc = row; pc < 16 * per_row; pc += 128) {
            const int j = pc / per_row, q = pc - j * per_row;
            const int t = ch * 16 + j;
            if (t >= ti.nrows) continue;
            const int col = out_col0 + q * 8;
            const uint16_t* src = sb + j * ncols + q * 8;
            uint16_t* dst = reinterpret_cast<uint16_t*>(outp) + (long long)(ti.row0 + t) * p.ld_out + col;
            if (out_vec && col + 8 <= p.rows_out) {
              *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
            } else {
              for (int e = 0; e < 8 && col + e < p.rows_out; ++e) dst[e] = src[e];
            }
          }
        }
      } else {
        // partial K range of this tile: park the fp32 partial in this CTA's slot,
        // laid out [weight row][activation row].  The tile's last contributor
        // to arrive (counted per tile) sums all its slots in K order and writes
        // the output, so no CTA waits for another; without counters
        // tc_fixup_kernel does the same right after this kernel.
        const int first_tile_of_cta = it_begin / kb;
        const long long slot = 2LL * c + (tile == first_tile_of_cta ? 0 : 1);
        float* P = p.partials + slot * (long long)(BMAX * 128) + (long long)row * BMAX;
        for (int ch = 0; ch < nb; ++ch) {
          float v[16];
          tmem_ld16(t_base + ch * 16, v);
          tmem_wait_ld();
          float4* d = reinterpret_cast<float4*>(P + ch * 16);
#pragma unroll
          for (int u = 0; u < 4; ++u) __stcg(d + u, make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]));
        }
        tc_fence_before();
        mbar_arrive(smem_u32(&acce_bar[a]));
        if (p.counters != nullptr) {
          __threadfence();                       // this CTA's partial before its arrival
          named_bar_sync(1, 128);
          const int c_first = sk.owner(tile * kb);
          const int nseg = sk.owner(tile * kb + kb - 1) - c_first + 1;
          if (row == 0) {
            const int prev = atomicAdd(&p.counters[tile], 1);
            const bool last = prev == nseg - 1;
            if (last) atomicExch(&p.counters[tile], 0);   // ready for the next launch
            *sh_last = last ? 1 : 0;
          }
          named_bar_sync(1, 128);
          if (*sh_last) {
            __threadfence();                     // the other contributors' partials
            for (int ch = 0; ch < nb; ++ch)
              reduce_split_chunk<BMAX>(p.partials, sk, kb, tile, c_first, nseg, ti, ch, row, outp, p.ld_out,
                                       p.bias, p.rows_out, p.silu, p.is_bf16 ? 0 : 1);
          }
        }
      }
      ++acc_iter;
      it = next_it(tile, kb1);
    }
  }

  if (p.trace && tid == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    p.trace[blockIdx.x * 8 + 6] = smid;
  }
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
  if (p.trace && tid == 0) p.trace[blockIdx.x * 8 + 7] = globaltimer_ns();
}

// Deterministic split-K reduction for tc_gemm_kernel.  A tile is split exactly
// where a CTA boundary falls strictly inside it, so block (b, chunk) looks at
// boundary b+1: if it is the first boundary inside its tile, the block sums that
// tile's partial slots in K order for 16 activation rows and applies the
// epilogue (bias, or SiLU*mul across the gate/up halves).  The grid is therefore
// (gemm grid - 1) x (BMAX / 16) whatever the tile count, and whole tiles (written
// by the GEMM itself) cost nothing here.
struct TcFixupArgs {
  const float* partials;
  void* out;
  const void* bias;
  const int* group_counts;   // grouped mode (tables then come from `tables`)
  const int* tables;
  long long ld_out;
  int single_rows, num_groups, kb, rows_out, row_tiles, silu, is_bf16, grid;
};

template <int BMAX>
__global__ void __launch_bounds__(128) tc_fixup_kernel(const TcFixupArgs p) {
  griddep_launch_dependents();
  griddep_wait();
  // grouped mode only: the GEMM's prefix tables, 2 x (num_groups + 1) ints of
  // dynamic shared memory (none in single mode, so that these blocks never
  // keep the next GEMM's CTAs off an SM)
  extern __shared__ int s_tab[];
  const int row = threadIdx.x;
  const int ch = blockIdx.y;
  const int* row_prefix = s_tab;
  const int* chunk_prefix = s_tab + p.num_groups + 1;
  int total_tiles;
  if (p.group_counts != nullptr) {
    for (int g = row; g <= p.num_groups; g += 128) {
      s_tab[g] = p.tables[g];
      s_tab[p.num_groups + 1 + g] = p.tables[TC_MAX_GROUPS + 1 + g];
    }
    __syncthreads();
    total_tiles = chunk_prefix[p.num_groups] * p.row_tiles;
  } else {
    total_tiles = ((p.single_rows + BMAX - 1) / BMAX) * p.row_tiles;
  }
  const int kb = p.kb;
  const int iters = total_tiles * kb;
  if (iters == 0) return;
  if (tc_whole_tiles(p.group_counts != nullptr, total_tiles, p.grid)) return;   // no split tiles
  const int G = min(p.grid, iters);
  const int cb = blockIdx.x + 1;                       // CTA boundary: start of CTA cb
  if (cb >= G) return;
  const SkSplit sk(iters, G);
  const int ib = sk.start(cb);
  if (ib % kb == 0) return;                            // on a tile edge: splits nothing
  const int tile = ib / kb;
  if (cb > 1) {
    const int ip = sk.start(cb - 1);
    if (ip / kb == tile && ip % kb != 0) return;       // an earlier boundary owns this tile
  }
  const int c_first = sk.owner(tile * kb);
  const int c_last = sk.owner(tile * kb + kb - 1);
  TcGemmArgs ta;                                       // decode_tile reads only these fields
  ta.group_counts = p.group_counts;
  ta.row_tiles = p.row_tiles;
  ta.single_rows = p.single_rows;
  ta.num_groups = p.num_groups;
  const TileInfo ti = decode_tile<BMAX>(tile, ta, row_prefix, chunk_prefix);
  if (ch * 16 >= ti.nrows) return;
  const int nseg = c_last - c_first + 1;
  const int odt = p.is_bf16 ? 0 : 1;
  char* outp = reinterpret_cast<char*>(p.out);
  reduce_split_chunk<BMAX>(p.partials, sk, kb, tile, c_first, nseg, ti, ch, row, outp, p.ld_out, p.bias,
                           p.rows_out, p.silu, odt);
}

}  // namespace simsd
