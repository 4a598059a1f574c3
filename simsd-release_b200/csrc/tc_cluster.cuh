// Thin-M GEMM with the split-K reduction done inside a thread-block cluster.
//
// y[m, n] = sum_k x[m, k] w[n, k] (+ bias[n]) or, with the SiLU*mul epilogue,
// y[m, i] = silu(x . w_gate[i]) * (x . w_up[i]), for M <= 64 activation rows.
// Same tensor-core pipeline as tc_gemm_kernel (TMA ring of 128 weight rows x
// 64 K and the activation box, tcgen05 MMA with the weights as the M = 128
// operand and the activation rows as N, fp32 accumulators in TMEM), but the
// work is split differently:
//
// * the grid is C clusters of S CTAs (S = 1..8); cluster c takes output tiles
//   c, c + C, c + 2C, ... and CTA rank q of a cluster takes K blocks
//   [q kb / S, (q + 1) kb / S) of each (the balanced split of SkSplit);
// * after a tile's K slice, each CTA keeps the accumulator rows it owns (an
//   S-th of the tile's 128 weight rows; for SiLU*mul the gate row i and up row
//   64 + i always share an owner) and stores every other row straight into its
//   owner's shared memory (st.async, completing bytes on the owner's
//   mbarrier);
// * each owner sums the S slices of its rows in rank (= K) order and writes
//   them to y with the epilogue.
//
// So a split tile costs one trip over the cluster's shared-memory network — no
// fp32 partials in global memory and no second kernel — and every output is
// summed in a fixed order, bit-identical across calls and graph replays.
//
// All waits are bounded (sm100.cuh).  A CTA leaves only after every peer's
// access to its shared memory is over: the rows sent to it are counted by its
// receive barrier, and after a cluster's last tile no CTA sends anything more
// (nor releases a buffer), so the receive wait of that tile is the last one.
#pragma once
#include "sm100.cuh"
#include "tc_gemm.cuh"

namespace simsd {

constexpr int TC_CL_MAX = 8;          // largest cluster (portable)
constexpr int TC_AG_MAX_WORLD = 8;    // ranks of a fused column-parallel all-gather
// A rank's signal block (ints): arrivals of every rank at the fused
// all-gather's sync points (each rank adds 1 per sync point, cumulative) and
// this rank's count of sync points.
constexpr int AG_SIG_ARRIVED = 0;
constexpr int AG_SIG_SYNCS = 2;
constexpr int TC_CL_RED_ROWS = 144;   // >= S * rows one owner holds, for every S <= 8

struct TcClusterArgs {
  CUtensorMap tmA0;          // weights (gate rows when silu): 2-D {K, N}
  CUtensorMap tmA1;          // up rows (silu), or the second weight of a concatenation
  CUtensorMap tmA2;          // the third weight of a concatenation
  // concatenated weights (plain epilogue): output tiles [0, cat_t1) read tmA0,
  // [cat_t1, cat_t2) tmA1 and [cat_t2, row_tiles) tmA2, each from its row 0,
  // into one y of the concatenated width; cat_t1 == 0: one weight
  int cat_t1, cat_t2;
  CUtensorMap tmB;           // activations: 2-D {K, M}
  void* out;                 // y, row stride ld_out elements
  const void* bias;          // [rows_out] or nullptr
  int* err;                  // device error word
  long long ld_out;
  int rows;                  // M (<= BMAX)
  int kb;                    // K blocks of 64 (>= cluster size)
  int rows_out;              // output columns (N, or N of the gate weight with silu)
  int row_tiles;             // output tiles (128 weight rows, or 64 gate + 64 up rows)
  int silu, is_bf16, pdl, prefetch;
  int l2_ahead;              // ring stages of weights requested into L2 ahead of the ring
  // argmax mode (amax_keys != nullptr, plain epilogue, world 1): y is not
  // written; amax_idx[t] = the first column of the largest output of row t
  // after rounding to the output type (torch.argmax over the rounded logits).
  // amax_keys [rows] and amax_count are zero before the launch and again after.
  unsigned long long* amax_keys;
  long long* amax_idx;
  int* amax_count;
  unsigned long long* trace; // optional: 8 %globaltimer stamps per CTA (diagnostics)
  // column-parallel all-gather (world > 1, the AG instantiation): every output
  // element is stored at column col_offset + col of each rank's y (peer_out[r],
  // NVLink mappings).  The launch signals nothing and nobody waits here: after
  // the launches whose outputs it needs, a reader runs ag_sync_kernel
  int world, rank, col_offset;
  void* peer_out[TC_AG_MAX_WORLD];
};

// F32: fp32 operands on the tensor cores.  A K block is then 32 elements (one
// 128-byte row, as 64 bf16 are), and each stage holds every atom twice: the
// raw fp32 words as loaded (turned in place into their tf32 "hi" parts) and the
// "lo" remainders, so the MMA can form hi*hi + hi*lo + lo*hi.
template <int BMAX, int KS, bool F32 = false>
struct TcClusterConfig {
  static constexpr int SPLIT = F32 ? 2 : 1;
  static constexpr int KW = F32 ? 32 : 64;   // K elements per block
  static constexpr int A_ATOM = TC_A_BYTES;
  static constexpr int B_ATOM = BMAX * 128;
  static constexpr int A_STAGE = SPLIT * KS * A_ATOM;
  static constexpr int B_STAGE = SPLIT * KS * B_ATOM;
  static constexpr int STAGE_BYTES = A_STAGE + B_STAGE;
  static constexpr int RED_BYTES = TC_CL_RED_ROWS * BMAX * 4;
  static constexpr int TAIL_BYTES = 2 * 10 * 8 + 8 * 8 + 64 + 64 * 16 * 4 + 64 * 8;
  static constexpr int STAGES_RAW = (227 * 1024 - 1024 - RED_BYTES - TAIL_BYTES) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 10 ? 10 : STAGES_RAW;
  // TMEM per accumulator buffer (two buffers).  F32: the tensor cores' fp32
  // accumulation loses a little with every MMA added into one accumulator, so
  // the hi*hi products of a CTA's K range go to NACC accumulators (consecutive
  // runs of K blocks) and the small hi*lo + lo*hi terms to one more; the
  // epilogue adds them with IEEE fp32 adds in a fixed order.
  static constexpr int NACC = F32 ? (BMAX >= 64 ? 3 : 7) : 1;
  static constexpr int ACC_STRIDE = F32 ? (NACC + 1) * BMAX : BMAX;
  static constexpr int TMEM_RAW = 2 * ACC_STRIDE;
  static constexpr int TMEM_COLS = TMEM_RAW <= 32 ? 32 : TMEM_RAW <= 64 ? 64 : TMEM_RAW <= 128 ? 128
                                   : TMEM_RAW <= 256 ? 256 : 512;
  static_assert(TMEM_RAW <= 512, "TMEM columns");
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + RED_BYTES + TAIL_BYTES;
  static_assert(STAGES >= 2, "ring needs two stages");
  static_assert(SMEM_BYTES <= 227 * 1024, "shared memory budget");
  static_assert(BMAX <= 64, "cluster reduction holds at most 64 activation rows");
};

// Owner (cluster rank) of accumulator row r and the row's index in the owner's
// receive slot, for cluster size S.  Plain tiles: rows cut into S runs of
// ceil(128 / S).  SiLU*mul tiles: the pair (i, 64 + i) cut into S runs of
// ceil(64 / S) pairs; an owner holds its gate rows first, then its up rows.
struct RowOwner {
  int S, silu, per;  // per = rows (plain) or pairs (silu) per owner
  __host__ __device__ __forceinline__ RowOwner(int S_, int silu_)
      : S(S_), silu(silu_), per(silu_ ? (64 + S_ - 1) / S_ : (128 + S_ - 1) / S_) {}
  __host__ __device__ __forceinline__ int owner(int r) const { return silu ? (r & 63) / per : r / per; }
  __host__ __device__ __forceinline__ int local(int r) const {
    return silu ? (r & 63) - owner(r) * per + (r >= 64 ? per : 0) : r - owner(r) * per;
  }
  // rows of one sender's slot in an owner's receive buffer
  __host__ __device__ __forceinline__ int slot_rows() const { return silu ? 2 * per : per; }
  // rows owner o holds
  __host__ __device__ __forceinline__ int rows_of(int o) const {
    const int total = silu ? 64 : 128;
    const int n = total - o * per;
    const int k = n < per ? (n > 0 ? n : 0) : per;
    return silu ? 2 * k : k;
  }
};

// Tensor map and first weight row of plain output tile `rtile` (one weight, or
// the part of a concatenation the tile falls in).
__device__ __forceinline__ const CUtensorMap* weight_map(const TcClusterArgs& p, int rtile, int& row0) {
  if (p.cat_t1 > 0 && rtile >= p.cat_t1) {
    if (rtile >= p.cat_t2) {
      row0 = (rtile - p.cat_t2) * 128;
      return &p.tmA2;
    }
    row0 = (rtile - p.cat_t1) * 128;
    return &p.tmA1;
  }
  row0 = rtile * 128;
  return &p.tmA0;
}

// Argmax key of output column `col` with value v: the value rounded to the
// output type, in an order-preserving unsigned form (NaN above everything, the
// two zeros equal), then 0xffffffff - col so that equal values keep the lowest
// column under a max.
__device__ __forceinline__ unsigned long long amax_key(float v, int col, int odt) {
  float r = odt == 0 ? __bfloat162float(__float2bfloat16_rn(v))
                     : (odt == 1 ? __half2float(__float2half_rn(v)) : v);
  if (r == 0.0f) r = 0.0f;
  const uint32_t b = __float_as_uint(r);
  const uint32_t k = (r != r) ? 0xffffffffu : ((b & 0x80000000u) ? ~b : (b | 0x80000000u));
  return ((unsigned long long)k << 32) | (unsigned long long)(0xffffffffu - (uint32_t)col);
}

template <int BMAX, int KS, bool F32 = false, bool AG = false>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_cluster_kernel(const __grid_constant__ TcClusterArgs p) {
  using Cfg = TcClusterConfig<BMAX, KS, F32>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int KW = Cfg::KW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_STAGE;
  float* red = reinterpret_cast<float*>(sB + STAGES * Cfg::B_STAGE);   // [S][slot rows][BMAX]
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + Cfg::RED_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* accf_bar = empty_bar + STAGES;  // [2]
  uint64_t* acce_bar = accf_bar + 2;        // [2]
  uint64_t* drain_bar = acce_bar + 2;       // [1]
  uint64_t* red_full = drain_bar + 1;       // [1] peers' rows for this CTA have landed
  uint64_t* red_free = red_full + 1;        // [1] every owner has consumed this CTA's rows
  int* misc = reinterpret_cast<int*>(red_free + 1);  // 16 ints
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort_flag = misc + 1;
  float* xbuf = reinterpret_cast<float*>(misc + 16);  // [16][64]
  unsigned long long* amax_best = reinterpret_cast<unsigned long long*>(xbuf + 16 * 64);  // [64]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = (int)cluster_nctarank();
  const int q = (int)cluster_ctarank();
  const int cid = (int)cluster_id_x();
  const int C = (int)cluster_count_x();
  if (p.trace && tid == 0) p.trace[blockIdx.x * 8 + 0] = globaltimer_ns();

  // ---- set-up
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
    mbar_init(smem_u32(red_full), 1);
    mbar_init(smem_u32(red_free), S > 1 ? S - 1 : 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&p.tmA0);
    if (p.silu || p.cat_t1 > 0) prefetch_tmap(&p.tmA1);
    if (p.cat_t1 > 0) prefetch_tmap(&p.tmA2);
    prefetch_tmap(&p.tmB);
  }
  if (warp == 5) {
    tmem_alloc(smem_u32(tmem_slot), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  if (tid == 0) griddep_launch_dependents();
  tc_fence_before();
  // Barrier initialisation is released to the cluster here and acquired by the
  // epilogue right before its first remote access (and by every other thread at
  // its end), so no CTA waits for its peers on the start-up path.
  cluster_arrive_release();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (p.trace && tid == 0) p.trace[blockIdx.x * 8 + 1] = globaltimer_ns();

  const int kb = p.kb;
  const int tiles = ((p.rows + BMAX - 1) / BMAX) * p.row_tiles;
  const SkSplit ksplit(kb, S);
  const int k_lo = ksplit.start(q), k_hi = ksplit.start(q + 1);
  const int n_tiles = cid < tiles ? (tiles - 1 - cid) / C + 1 : 0;
  auto tile_of = [&](int i) { return cid + i * C; };
  const int nrows_all = p.rows < BMAX ? p.rows : BMAX;   // rows <= BMAX: one row block
  // F32: K blocks of this CTA and the hi*hi accumulator runs they are cut into
  const int f32_nblk = k_hi - k_lo;
  const int f32_nch = f32_nblk < Cfg::NACC ? f32_nblk : Cfg::NACC;
  const int nb = (nrows_all + TC_BOX_ROWS - 1) / TC_BOX_ROWS;

  if (warp == 4) {
    // ================= TMA producer
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued_mask = 0;
      uint32_t last_parity = 0;
      bool ok = true;
      // Programmatic dependent launch: the first `prefetch` stages of weights
      // are requested before griddep_wait(); their activation boxes follow it.
      bool dep_ready = !p.pdl;
      int npend = 0;
      bool traced_first = false;
      uint32_t pend_dst[STAGES], pend_bar[STAGES];
      int pend_k0[STAGES], pend_na[STAGES];
      auto flush_pending = [&]() {
        griddep_wait();
        dep_ready = true;
        for (int s2 = 0; s2 < npend; ++s2)
          for (int at = 0; at < pend_na[s2]; ++at)
            tma_load_2d(pend_dst[s2] + at * Cfg::B_ATOM, &p.tmB, pend_bar[s2], pend_k0[s2] + at * KW, 0, pol_x);
        npend = 0;
      };
      // L2 prefetch cursor over the (tile, stage) sequence: DRAM requests for the
      // weights run l2_ahead stages ahead of the shared-memory ring
      const int nsteps = (k_hi - k_lo + KS - 1) / KS;
      const int total_steps = n_tiles * nsteps;
      int pf = 0, step = 0;
      for (int i = 0; ok && i < n_tiles; ++i) {
        const int rtile = tile_of(i);   // one row block: tile index == output tile
        for (int k = k_lo; k < k_hi; k += KS, ++step) {
          const int na = min(KS, k_hi - k);
          if (pf <= step) pf = step + 1;
          for (; pf < total_steps && pf <= step + p.l2_ahead; ++pf) {
            const int pi = pf / nsteps;
            const int pk = k_lo + (pf - pi * nsteps) * KS;
            const int prt = tile_of(pi);
            for (int at = 0; at < KS && pk + at < k_hi; ++at) {
              if (p.silu) {
                tma_prefetch_l2_2d(&p.tmA0, (pk + at) * KW, prt * 64, pol_w);
                tma_prefetch_l2_2d(&p.tmA1, (pk + at) * KW, prt * 64, pol_w);
              } else {
                int pr0;
                const CUtensorMap* pm = weight_map(p, prt, pr0);
                tma_prefetch_l2_2d(pm, (pk + at) * KW, pr0, pol_w);
              }
            }
          }
          if (!dep_ready && npend >= min(STAGES, p.prefetch)) flush_pending();
          if (!mbar_wait(smem_u32(&empty_bar[stage]), phase ^ 1, abort_flag, p.err)) { ok = false; break; }
          const uint32_t fb = smem_u32(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, na * (TC_A_BYTES + Cfg::B_ATOM));
          issued_mask |= 1u << stage;
          last_parity = (last_parity & ~(1u << stage)) | (phase << stage);
          const uint32_t b_dst = smem_u32(sB + stage * Cfg::B_STAGE);
          for (int at = 0; at < na; ++at) {
            const uint32_t a_dst = smem_u32(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM);
            const int k0 = (k + at) * KW;
            if (p.silu) {
              tma_load_2d(a_dst, &p.tmA0, fb, k0, rtile * 64, pol_w);
              tma_load_2d(a_dst + 8192, &p.tmA1, fb, k0, rtile * 64, pol_w);
            } else {
              int r0;
              const CUtensorMap* wm = weight_map(p, rtile, r0);
              tma_load_2d(a_dst, wm, fb, k0, r0, pol_w);
            }
            if (dep_ready) tma_load_2d(b_dst + at * Cfg::B_ATOM, &p.tmB, fb, k0, 0, pol_x);
          }
          if (p.trace && !traced_first) { p.trace[blockIdx.x * 8 + 2] = globaltimer_ns(); traced_first = true; }
          if (!dep_ready) {
            pend_dst[npend] = b_dst;
            pend_bar[npend] = fb;
            pend_k0[npend] = k * KW;
            pend_na[npend] = na;
            ++npend;
          }
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      if (!dep_ready) flush_pending();
      if (p.trace) p.trace[blockIdx.x * 8 + 4] = globaltimer_ns();
      if (!ok) {
        for (int s2 = 0; s2 < STAGES; ++s2)
          if (issued_mask & (1u << s2))
            mbar_wait_drain(smem_u32(&full_bar[s2]), (last_parity >> s2) & 1u, 100000000ull);
      }
    }
    __syncwarp();
    cluster_wait_acquire();   // pairs this warp's set-up arrive
  } else if (warp == 5) {
    // ================= MMA issuer
    if constexpr (F32) {
      // fp32 operands: the whole warp turns each landed stage into tf32 parts
      // (hi in place, lo beside it), then lane 0 issues hi*hi + hi*lo + lo*hi
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      const uint32_t idesc = make_idesc_tf32(128, nb * TC_BOX_ROWS);
      const int b_vec = nb * TC_BOX_ROWS * 8;   // float4s of the activation rows the MMA reads
      for (int i = 0; ok && i < n_tiles; ++i) {
        const int a = i & 1;
        const uint32_t aphase = (i >> 1) & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&acce_bar[a]), aphase ^ 1, abort_flag, p.err))) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_base = tmem_base + a * Cfg::ACC_STRIDE;
        const uint32_t d_small = d_base + Cfg::NACC * BMAX;
        for (int k = k_lo; k < k_hi; k += KS) {
          const int na = min(KS, k_hi - k);
          // KS == 1: one K block per stage; its run j of the NACC hi*hi accumulators
          const int jrun = (k - k_lo) * f32_nch / f32_nblk;
          const bool run_start = k == k_lo || (k - 1 - k_lo) * f32_nch / f32_nblk != jrun;
          if (!__all_sync(0xffffffffu, mbar_wait(smem_u32(&full_bar[stage]), phase, abort_flag, p.err))) {
            ok = false;
            break;
          }
          uint8_t* const a_st = sA + stage * Cfg::A_STAGE;
          uint8_t* const b_st = sB + stage * Cfg::B_STAGE;
          for (int at = 0; at < na; ++at) {
            float4* ah = reinterpret_cast<float4*>(a_st + at * Cfg::A_ATOM);
            float4* al = reinterpret_cast<float4*>(a_st + (KS + at) * Cfg::A_ATOM);
#pragma unroll 4
            for (int v = lane; v < Cfg::A_ATOM / 16; v += 32) split_tf32(ah, al, v);
            float4* bh = reinterpret_cast<float4*>(b_st + at * Cfg::B_ATOM);
            float4* bl = reinterpret_cast<float4*>(b_st + (KS + at) * Cfg::B_ATOM);
            for (int v = lane; v < b_vec; v += 32) split_tf32(bh, bl, v);
          }
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            tc_fence_after();
            if (p.trace && !issued_any) p.trace[blockIdx.x * 8 + 3] = globaltimer_ns();
            for (int at = 0; at < na; ++at) {
              const uint64_t ahd = make_sw128_desc(smem_u32(a_st + at * Cfg::A_ATOM));
              const uint64_t ald = make_sw128_desc(smem_u32(a_st + (KS + at) * Cfg::A_ATOM));
              const uint64_t bhd = make_sw128_desc(smem_u32(b_st + at * Cfg::B_ATOM));
              const uint64_t bld = make_sw128_desc(smem_u32(b_st + (KS + at) * Cfg::B_ATOM));
#pragma unroll
              for (int kk = 0; kk < 4; ++kk) {
                const uint32_t acc_main = (run_start && at == 0 && kk == 0) ? 0u : 1u;
                const uint32_t acc_small = (k > k_lo || at > 0 || kk > 0) ? 1u : 0u;
                tc_mma_tf32(d_base + jrun * BMAX, ahd + 2 * kk, bhd + 2 * kk, idesc, acc_main);
                tc_mma_tf32(d_small, ahd + 2 * kk, bld + 2 * kk, idesc, acc_small);
                tc_mma_tf32(d_small, ald + 2 * kk, bhd + 2 * kk, idesc, 1u);
              }
            }
            tc_commit(smem_u32(&empty_bar[stage]));
          }
          __syncwarp();
          issued_any = true;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        if (lane == 0) tc_commit(smem_u32(&accf_bar[a]));
        __syncwarp();
      }
      if (lane == 0) {
        if (p.trace) p.trace[blockIdx.x * 8 + 5] = globaltimer_ns();
        if (!ok && issued_any) {
          tc_commit(smem_u32(drain_bar));
          mbar_wait_drain(smem_u32(drain_bar), 0, 100000000ull);
        }
      }
    } else if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      bool issued_any = false;
      const uint32_t idesc = make_idesc_f16(p.is_bf16, 128, nb * TC_BOX_ROWS);
      for (int i = 0; ok && i < n_tiles; ++i) {
        const int a = i & 1;
        const uint32_t aphase = (i >> 1) & 1;
        if (!mbar_wait(smem_u32(&acce_bar[a]), aphase ^ 1, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BMAX;
        for (int k = k_lo; k < k_hi; k += KS) {
          const int na = min(KS, k_hi - k);
          if (!mbar_wait(smem_u32(&full_bar[stage]), phase, abort_flag, p.err)) { ok = false; break; }
          tc_fence_after();
          if (p.trace && !issued_any) p.trace[blockIdx.x * 8 + 3] = globaltimer_ns();
          for (int at = 0; at < na; ++at) {
            const uint64_t adesc = make_sw128_desc(smem_u32(sA + stage * Cfg::A_STAGE + at * Cfg::A_ATOM));
            const uint64_t bdesc = make_sw128_desc(smem_u32(sB + stage * Cfg::B_STAGE + at * Cfg::B_ATOM));
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              tc_mma_f16(d_tmem, adesc + 2 * kk, bdesc + 2 * kk, idesc, (k > k_lo || at > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          tc_commit(smem_u32(&empty_bar[stage]));
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
        if (!ok) break;
        tc_commit(smem_u32(&accf_bar[a]));
      }
      if (p.trace) p.trace[blockIdx.x * 8 + 5] = globaltimer_ns();
      if (!ok && issued_any) {
        tc_commit(smem_u32(drain_bar));
        mbar_wait_drain(smem_u32(drain_bar), 0, 100000000ull);
      }
    }
    __syncwarp();
    cluster_wait_acquire();   // pairs this warp's set-up arrive
  } else {
    // ================= epilogue warps 0-3: TMEM lanes 32*warp .. 32*warp+31
    const int row = tid;   // 0..127 == TMEM lane == accumulator (weight) row
    const RowOwner ro(S, p.silu);
    const int own = ro.owner(row);
    const int lr = ro.local(row);
    const int slot_rows = ro.slot_rows();
    const int odt = F32 ? 2 : (p.is_bf16 ? 0 : 1);
    char* outp = reinterpret_cast<char*>(p.out);
    const uint32_t red_u32 = smem_u32(red);
    const uint32_t red_full_u32 = smem_u32(red_full);
    const uint32_t red_free_u32 = smem_u32(red_free);
    auto swz = [](int lr, int j) { return BMAX >= 32 ? (j ^ (lr & 7)) : (j ^ ((lr >> 1) & 3)); };
    bool cluster_acquired = false;
    // y[t, col] on this GPU, or on every rank's GPU for the fused all-gather,
    // or (argmax mode) the CTA's running maximum of row t
    if (p.amax_keys != nullptr && row < BMAX) amax_best[row] = 0ull;   // before the first tile's barrier
    auto put = [&](long long t, int col, float v) {
      if (p.amax_keys != nullptr) {
        atomicMax(&amax_best[t], amax_key(v, col, odt));
      } else if (p.world <= 1) {
        store_f(outp, t * p.ld_out + col, v, odt);
      } else {
        for (int r = 0; r < p.world; ++r) store_f(p.peer_out[r], t * p.ld_out + p.col_offset + col, v, odt);
      }
    };
    // Owner sums (step 5).  The CTA's owned outputs are a grid of units (rows,
    // or gate/up pairs: output columns) x groups of 4 activation rows.  A work
    // item is a block of EP_CW consecutive units (BMAX / 16 of them: 1, 2 or 4)
    // and one group; items are numbered so that a quarter-warp's 8 lanes take
    // 8 / EP_CW column blocks x EP_CW groups: their slot reads (16-byte group
    // swz(l, g) of row l) fall on 8 different bank groups, and a lane's EP_CW
    // results of one activation row are adjacent in y, so they leave as one
    // 2-, 4- or 8-byte store.  Thread `row` takes items row, row + 128, ...;
    // its first item is fixed for the launch.
    constexpr int EP_CW = BMAX >= 64 ? 4 : (BMAX >= 32 ? 2 : 1);
    const int ep_units = S > 1 ? (p.silu ? ro.rows_of(q) / 2 : ro.rows_of(q)) : 0;
    const int ep_ncb = (ep_units + EP_CW - 1) / EP_CW;                  // column blocks
    const int ep_groups = (nrows_all + 3) >> 2;
    const int ep_gsup = (ep_groups + EP_CW - 1) / EP_CW;                 // groups / EP_CW, rounded up
    const int ep_items = ep_ncb * ep_gsup * EP_CW;
    auto ep_item = [&](int it, int& cb, int& g) {
      const int lo = it % EP_CW, rest = it / EP_CW;
      cb = rest % ep_ncb;
      g = (rest / ep_ncb) * EP_CW + lo;
    };
    int ep_cb0 = 0, ep_g0 = 0;
    if (ep_ncb > 0) ep_item(row, ep_cb0, ep_g0);
    // plain stores into y (AG: into every rank's y); 8- and 4-byte stores need
    // every target base aligned to them
    const bool ep_fast = p.amax_keys == nullptr && (AG || p.world <= 1);
    int ep_base_al = 8;
    {
      const int nt = AG ? p.world : 1;
      for (int r = 0; r < nt; ++r) {
        const uintptr_t b = reinterpret_cast<uintptr_t>(AG ? p.peer_out[r] : p.out);
        ep_base_al = min(ep_base_al, (b & 7) == 0 ? 8 : ((b & 3) == 0 ? 4 : 2));
      }
    }
    const long long ep_ld = p.ld_out;
    const int ep_silu = p.silu;
    const int ep_rows_out = p.rows_out;
    // 16 accumulator columns (activation rows ch*16 ..) of this thread's row;
    // F32: the hi*hi runs in order, then the small terms, with IEEE fp32 adds
    auto acc_ld16 = [&](uint32_t tb, int ch, float (&v)[16]) {
      tmem_ld16(tb + ch * 16, v);
      if constexpr (F32) {
        tmem_wait_ld();
#pragma unroll 1
        for (int j = 1; j <= f32_nch; ++j) {
          float w[16];
          tmem_ld16(tb + (j < f32_nch ? j : Cfg::NACC) * BMAX + ch * 16, w);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; ++e) v[e] = __fadd_rn(v[e], w[e]);
        }
      }
    };
    int done = 0;
    for (int i = 0; i < n_tiles; ++i) {
      const int rtile = tile_of(i);
      const int a = i & 1;
      const uint32_t aphase = (i >> 1) & 1;
      if (!named_bar_and(1, 128, mbar_wait(smem_u32(&accf_bar[a]), aphase, abort_flag, p.err))) break;
      tc_fence_after();
      const uint32_t t_base = tmem_base + ((uint32_t)(warp * 32) << 16) + a * Cfg::ACC_STRIDE;
      const int out_col0 = p.silu ? rtile * 64 : rtile * 128;

      if (S == 1) {
        // whole K range here: straight to y (as tc_gemm_kernel's whole tiles)
        for (int ch = 0; ch < nb; ++ch) {
          float v[16];
          acc_ld16(t_base, ch, v);
          tmem_wait_ld();
          if (ch == nb - 1) {
            tc_fence_before();
            mbar_arrive(smem_u32(&acce_bar[a]));
          }
          if (!p.silu) {
            const int col = out_col0 + row;
            if (col < p.rows_out) {
              const float bv = p.bias ? load_f(p.bias, col, odt) : 0.0f;
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int t = ch * 16 + j;
                if (t < nrows_all) put(t, col, __fadd_rn(v[j], bv));
              }
            }
          } else {
            if (row >= 64) {
#pragma unroll
              for (int j = 0; j < 16; ++j) xbuf[j * 64 + (row - 64)] = v[j];
            }
            named_bar_sync(1, 128);
            if (row < 64) {
              const int col = out_col0 + row;
              if (col < p.rows_out) {
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                  const int t = ch * 16 + j;
                  if (t < nrows_all)
                    put(t, col, silu_mul(v[j], xbuf[j * 64 + row]));
                }
              }
            }
            named_bar_sync(1, 128);
          }
        }
        ++done;
        continue;
      }

      if (!cluster_acquired) {
        cluster_wait_acquire();   // the peers' barriers are initialised
        cluster_acquired = true;
      }
      // -- 1. the owners have consumed this CTA's rows of the previous tile
      if (i > 0 && !named_bar_and(1, 128, mbar_wait_cluster(red_free_u32, (i - 1) & 1, abort_flag, p.err))) break;
      // -- 2. bytes this CTA receives for the tile: its rows from every peer
      if (row == 0) mbar_arrive_expect_tx(red_full_u32, (uint32_t)((S - 1) * ro.rows_of(q) * nb * 64));
      // -- 3. drain the accumulator: keep own rows, send the others to their owners
      // this CTA's own rows go straight into its own slot of the receive
      // buffer (slot q: no peer writes it, and every thread finished reading
      // it for the previous tile before the barrier that ended that tile)
      float4* const own_dst = reinterpret_cast<float4*>(red + ((q * slot_rows) + lr) * BMAX);
      const uint32_t dst_row = mapa_shared(red_u32 + (uint32_t)(((q * slot_rows) + lr) * BMAX * 4), (uint32_t)own);
      // 16-byte column group j of a received row sits at group swz(j): the XOR
      // spreads the rows that one quarter-warp touches over all 32 banks
      const uint32_t dst_bar = mapa_shared(red_full_u32, (uint32_t)own);
#pragma unroll
      for (int ch = 0; ch < BMAX / 16; ++ch) {
        if (ch < nb) {
          float v[16];
          acc_ld16(t_base, ch, v);
          tmem_wait_ld();
          if (own == q) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              own_dst[swz(lr, ch * 4 + u)] = make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          } else {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              st_async_v4(dst_row + (uint32_t)(swz(lr, ch * 4 + u) * 16), v[4 * u], v[4 * u + 1], v[4 * u + 2],
                          v[4 * u + 3], dst_bar);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&acce_bar[a]));
      // first output column this CTA owns; the bias of the first item's
      // columns, fetched before the wait
      const int ep_c0 = out_col0 + q * ro.per;
      float ep_bias[EP_CW];
#pragma unroll
      for (int u = 0; u < EP_CW; ++u) {
        const int c = ep_cb0 * EP_CW + u;
        ep_bias[u] = (row < ep_items && !ep_silu && p.bias && c < ep_units && ep_c0 + c < ep_rows_out)
                         ? load_f(p.bias, ep_c0 + c, odt) : 0.0f;
      }
      // -- 4. every peer's rows for this CTA have landed
      if (!named_bar_and(1, 128, mbar_wait_cluster(red_full_u32, i & 1, abort_flag, p.err))) break;
      // -- 5. all 128 threads share the owned outputs: each item's sums run
      // over the S slots in rank (= K) order (the barrier of step 4 ordered
      // every thread's own-slot writes); slot rows are clamped so every load
      // is in range and none waits on a branch; only the stores are predicated
      {
        auto slot4 = [&](int r, int l, int g) -> float4 {
          return reinterpret_cast<const float4*>(red + ((r * slot_rows) + l) * BMAX)[swz(l, g)];
        };
#pragma unroll 1
        for (int it = row; it < ep_items; it += 128) {
          int cb = ep_cb0, g = ep_g0;
          if (it != row) ep_item(it, cb, g);
          const int u0 = cb * EP_CW;
          const int ncol = min(min(EP_CW, ep_units - u0), ep_rows_out - (ep_c0 + u0));
          if (g >= ep_groups || ncol <= 0) continue;
          float4 a[EP_CW], b[EP_CW];
#pragma unroll
          for (int u = 0; u < EP_CW; ++u) a[u] = b[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
          for (int r = 0; r < TC_CL_MAX; ++r) {
            if (r >= S) break;
#pragma unroll
            for (int u = 0; u < EP_CW; ++u) {
              const int l = u0 + min(u, ncol - 1);
              const float4 f = slot4(r, l, g);
              a[u].x = __fadd_rn(a[u].x, f.x);
              a[u].y = __fadd_rn(a[u].y, f.y);
              a[u].z = __fadd_rn(a[u].z, f.z);
              a[u].w = __fadd_rn(a[u].w, f.w);
              if (ep_silu) {
                const float4 h = slot4(r, ro.per + l, g);
                b[u].x = __fadd_rn(b[u].x, h.x);
                b[u].y = __fadd_rn(b[u].y, h.y);
                b[u].z = __fadd_rn(b[u].z, h.z);
                b[u].w = __fadd_rn(b[u].w, h.w);
              }
            }
          }
          float bias[EP_CW];
#pragma unroll
          for (int u = 0; u < EP_CW; ++u)
            bias[u] = it == row ? ep_bias[u]
                                : ((!ep_silu && p.bias && u < ncol) ? load_f(p.bias, ep_c0 + u0 + u, odt) : 0.0f);
          const int col = ep_c0 + u0;
#pragma unroll
          for (int k4 = 0; k4 < 4; ++k4) {
            const int t = 4 * g + k4;
            if (t >= nrows_all) break;
            float v[EP_CW];
#pragma unroll
            for (int u = 0; u < EP_CW; ++u) {
              const float x = k4 == 0 ? a[u].x : k4 == 1 ? a[u].y : k4 == 2 ? a[u].z : a[u].w;
              const float y = k4 == 0 ? b[u].x : k4 == 1 ? b[u].y : k4 == 2 ? b[u].z : b[u].w;
              v[u] = ep_silu ? silu_mul(x, y) : __fadd_rn(x, bias[u]);
            }
            if (!ep_fast) {
#pragma unroll
              for (int u = 0; u < EP_CW; ++u)
                if (u < ncol) put(t, col + u, v[u]);
            } else if constexpr (F32) {
              float* dst = reinterpret_cast<float*>(outp) + (long long)t * ep_ld + col;
#pragma unroll
              for (int u = 0; u < EP_CW; ++u)
                if (u < ncol) dst[u] = v[u];
            } else {
              // 16-bit outputs, packed two to a word where the columns allow
              uint32_t pk[(EP_CW + 1) / 2] = {};
#pragma unroll
              for (int u = 0; u + 1 < EP_CW; u += 2)
                pk[u / 2] = (uint32_t)f32_to_16bit(v[u], odt) | ((uint32_t)f32_to_16bit(v[u + 1], odt) << 16);
              const long long e = (long long)t * ep_ld + (AG ? (long long)p.col_offset : 0ll) + col;
              const int nt = AG ? p.world : 1;
              for (int r = 0; r < nt; ++r) {
                uint16_t* dst = reinterpret_cast<uint16_t*>(AG ? p.peer_out[r] : outp) + e;
                bool done_st = false;
                if constexpr (EP_CW == 4) {
                  if (ncol == 4 && ep_base_al >= 8 && (e & 3) == 0) {
                    *reinterpret_cast<uint2*>(dst) = make_uint2(pk[0], pk[1]);
                    done_st = true;
                  }
                }
                if constexpr (EP_CW >= 2) {
                  if (!done_st && ep_base_al >= 4 && (e & 1) == 0) {
#pragma unroll
                    for (int u = 0; u < EP_CW; u += 2) {
                      if (u + 1 < ncol) *reinterpret_cast<uint32_t*>(dst + u) = pk[u / 2];
                      else if (u < ncol) dst[u] = f32_to_16bit(v[u], odt);
                    }
                    done_st = true;
                  }
                }
                if (!done_st) {
#pragma unroll
                  for (int u = 0; u < EP_CW; ++u)
                    if (u < ncol) dst[u] = f32_to_16bit(v[u], odt);
                }
              }
            }
          }
        }
      }
      // -- 6. this CTA's receive buffer is free again: tell every sender.  Not
      // after the last tile: nothing is sent after it, so once its rows have
      // landed here (step 4) no peer touches this CTA's shared memory again and
      // every CTA may leave as soon as its own rows are written.
      if (i + 1 < n_tiles) {
        named_bar_sync(1, 128);
        if (row == 0)
          for (int r = 0; r < S; ++r)
            if (r != q) mbar_arrive_remote(mapa_shared(red_free_u32, (uint32_t)r));
      }
      ++done;
    }
    if (p.amax_keys != nullptr) {
      // every CTA adds its maxima to the launch's keys and counts itself; the
      // last one turns the keys into column indices and zeroes them again
      volatile int* sh_amax_last = misc + 5;
      named_bar_sync(1, 128);
      if (row < nrows_all && amax_best[row] != 0ull) atomicMax(&p.amax_keys[row], amax_best[row]);
      __threadfence();
      named_bar_sync(1, 128);
      if (row == 0) *sh_amax_last = atomicAdd(p.amax_count, 1) == (int)gridDim.x - 1 ? 1 : 0;
      named_bar_sync(1, 128);
      if (*sh_amax_last) {
        __threadfence();
        if (row < nrows_all) {
          const unsigned long long k = atomicExch(&p.amax_keys[row], 0ull);
          p.amax_idx[row] = (long long)(0xffffffffu - (uint32_t)(k & 0xffffffffull));
        }
        if (row == 0) atomicExch(p.amax_count, 0);
      }
    }
    if (!cluster_acquired) cluster_wait_acquire();
    if (S > 1 && done < n_tiles && row == 0) {
      // aborting: give peers that may still be sending to this CTA time to land
      mbar_wait_cluster_drain(red_full_u32, done & 1, 100000000ull);
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

// The fused all-gather's sync point, run by every rank on the stream of its
// launches, before the kernels that read their outputs.  One thread:
//  1. griddep_wait(): every earlier kernel on the stream has completed, so
//     this rank's peer stores of every fused launch issued so far are
//     performed (kernel completion flushes them, as it does stores to host
//     memory);
//  2. a system-scope fence, then adds 1 with release to the arrival counter
//     of every rank (this rank's own included) and advances this rank's sync
//     count;
//  3. waits (bounded) until its own arrival counter reaches world x its sync
//     count: every rank has passed step 2 of this sync point, so all their
//     columns are in this rank's outputs.
// Counters are cumulative and compared modulo 2^32.  The launches themselves
// carry no signal, so a fused launch costs what a local one does, and ranks
// meet once per sync point instead of once per launch.
struct AgSyncArgs {
  int* sig[TC_AG_MAX_WORLD];   // every rank's signal block (NVLink mappings; own at [rank])
  int world, rank;
  int* err;
};

__global__ void ag_sync_kernel(const __grid_constant__ AgSyncArgs a) {
  if (threadIdx.x != 0) return;
  griddep_launch_dependents();   // the reader may launch and set up; its own wait covers this kernel
  griddep_wait();
  __threadfence_system();
  int* mine = a.sig[a.rank];
  volatile int* syncs = mine + AG_SIG_SYNCS;
  const unsigned count = (unsigned)*syncs + 1u;
  *syncs = (int)count;
  for (int r = 0; r < a.world; ++r) red_add_release_sys(a.sig[r] + AG_SIG_ARRIVED, 1);
  const unsigned target = count * (unsigned)a.world;
  const uint64_t t0 = globaltimer_ns();
  while ((int)((unsigned)ld_acquire_sys(mine + AG_SIG_ARRIVED) - target) < 0) {
    if (globaltimer_ns() - t0 > SIMSD_WAIT_LIMIT_NS) {
      atomicOr(a.err, SIMSD_DEV_ERR_TIMEOUT);
      break;
    }
  }
  __threadfence_system();
}

}  // namespace simsd
