// Verify attention on the 5th-generation tensor cores, split over keys inside a
// thread-block cluster:
//   o[t, h, :] = softmax_j(scale * q[h, t] . k[g, j] | mask[t, j]) v[g, j],
//   g = h / G (G = Hq / Hk query heads per KV head), keys j < Lk.
// One cluster of S CTAs per KV head g; CTA rank r takes the key tiles (128 keys
// each) [r nt / S, (r + 1) nt / S) of the cache, at most ATC_NT_MAX of them.  The
// G query heads x L rows of the head group form one 128-row tile (row =
// head_in_group * L + t), so every K/V tile is read once for all of them
// (native GQA: no expanded K/V).
//
// Per key tile i (warp 8 loads with TMA, warp 9 issues tcgen05.mma, warps 0-7
// hold the query rows, one TMEM lane each, two threads a row: warp w takes the
// rows of TMEM lane quarter w % 4 and the 64 keys / dims of half w / 4):
//   S = Q K_i^T         bf16 x bf16 -> fp32 in TMEM columns [0, 128)
//   softmax of the row over the tile's 128 keys (fp32, exp2 of log2-scaled
//   scores, masked keys -inf), P_i = bf16(p) written to shared memory in the
//   128-byte-swizzled K-major layout the MMA reads
//   O_i = P_i V_i       V read in place as an MN-major operand, fp32 in TMEM
//                       columns [128 (i + 1), 128 (i + 2))
// with the tile's row max m_i and sum l_i (of the unrounded p) kept in
// registers.  Then each CTA merges its tiles, O = sum_i 2^(m_i - M) O_i, and the
// S CTAs of the cluster merge theirs the same way over distributed shared
// memory: each CTA owns a 1/S slice of the rows, the others send it their
// (O, M, L) rows with st.async, and the owner writes o = O / L in bf16 into the
// [L, Hq, 128] layout the output projection reads.  No fp32 partials in global
// memory and no second kernel.
//
// Numerics as flash attention: P rounded to bf16 for the second product, fp32
// everywhere else; a row with every key masked comes out as zeros.  All waits
// are bounded (sm100.cuh); every CTA passes the two cluster barriers
// unconditionally, so an aborting CTA never strands its peers.
#pragma once
#include "sm100.cuh"

namespace simsd {

constexpr int ATC_THREADS = 320;   // warps 0-7 softmax / merge (two per TMEM lane quarter), 8 loads, 9 MMA
constexpr int ATC_SM_THREADS = 256;
constexpr int ATC_TILE = 128;      // keys per tile
constexpr int ATC_NT_MAX = 3;      // key tiles per CTA (TMEM: S + 3 O accumulators = 512 columns)
constexpr int ATC_CL_MAX = 8;      // CTAs per cluster (portable)
constexpr int ATC_CL_MAX_NP = 16;  // non-portable cluster size, where the device runs it
constexpr int ATC_REC = 132;       // floats per merged row record: O[128], M, L, 2 pad
constexpr int ATC_G4 = ATC_REC / 4;  // its 16-byte groups
constexpr int ATC_Q_BYTES = 32768;            // 128 rows x 128 dims bf16, two 64-dim atoms
constexpr int ATC_STAGE_BYTES = 65536;        // K tile + V tile
constexpr int ATC_P_BYTES = 32768;            // 128 rows x 128 keys bf16, two 64-key atoms
constexpr int ATC_XCH_BYTES = 4096;          // row max / sum halves exchanged between the two warps of a row
constexpr int ATC_SMEM = 1024 + ATC_Q_BYTES + 2 * ATC_STAGE_BYTES + ATC_P_BYTES + 256 + ATC_XCH_BYTES;
static_assert(ATC_CL_MAX_NP * ((128 + ATC_CL_MAX_NP - 1) / ATC_CL_MAX_NP) * ATC_REC * 4 <= 2 * ATC_STAGE_BYTES,
              "the merge records fit in the K/V stages");

struct AttnTcArgs {
  CUtensorMap tmQ;        // q [Hq * L, 128] bf16, box {64, 128}
  CUtensorMap tmK;        // k_cache [Hk * cap, 128] bf16, box {64, 128}
  CUtensorMap tmV;        // v_cache, same
  const uint8_t* mask;    // [L, ldm], nonzero = attend
  void* o;                // [L, Hq, 128] bf16
  int* err;               // device error word
  long long cap, ldm;
  int Hq, Hk, L, Lk, ntiles, mask_vec;
  float scale_log2;       // softmax scale * log2(e)
  // optional diagnostics: 8 %globaltimer stamps per CTA (entry, set-up done,
  // first S MMA issued, tile 0's P written, last P V committed, all P V done,
  // merge records sent, exit)
  unsigned long long* trace;
};

// Shared-memory descriptor of an MN-major operand in the 128-byte-swizzle
// layout: atoms of 8 K-rows x 128 bytes (64 bf16 along MN); `lbo` = bytes from
// one 64-wide MN block to the next, `sbo` = bytes from one 8-row K group to the
// next.
__device__ __forceinline__ uint64_t make_sw128_desc_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// 2^x with the hardware approximation (the probabilities are rounded to bf16
// right after, so its ~2^-22 relative error is invisible)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// two floats -> packed bf16x2 (round to nearest even), low half = lo
__device__ __forceinline__ uint32_t pack2_bf16(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__global__ void __launch_bounds__(ATC_THREADS, 1) attn_tc_kernel(const __grid_constant__ AttnTcArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Qs = smem;
  uint8_t* Stg = Qs + ATC_Q_BYTES;                       // 2 stages: [K atom0, K atom1, V atom0, V atom1]
  uint8_t* Ps = Stg + 2 * ATC_STAGE_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(Ps + ATC_P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]  K tile landed / free again (its S issued and done)
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* p_free = bars + 8;
  uint64_t* o_done = bars + 9;
  uint64_t* recv_full = bars + 10;
  uint64_t* v_full = bars + 11;  // [2]  V tile landed / free again (its P V done)
  uint64_t* v_empty = bars + 13; // [2]
  int* misc = reinterpret_cast<int*>(bars + 16);
  float* xch = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(bars) + 256);   // [2][128] max, [3][2][128] sum
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc);
  volatile int* abort_flag = misc + 1;
  float* recv = reinterpret_cast<float*>(Stg);            // merge records, after every MMA is done

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int S = (int)cluster_nctarank();
  const int q = (int)cluster_ctarank();
  const int g = (int)cluster_id_x();
  const int G = p.Hq / p.Hk;
  const int R = G * p.L;
  const int t_lo = (q * p.ntiles) / S, t_hi = ((q + 1) * p.ntiles) / S;
  const int nt = t_hi - t_lo;
  const int RP = (R + S - 1) / S;            // rows each CTA merges and writes
  unsigned long long* const tr = p.trace ? p.trace + (long long)blockIdx.x * 8 : nullptr;
  if (tr && tid == 0) tr[0] = globaltimer_ns();

  if (tid == 0) {
    mbar_init(smem_u32(q_full), 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    mbar_init(smem_u32(s_full), 1);
    mbar_init(smem_u32(s_free), ATC_SM_THREADS);
    mbar_init(smem_u32(p_full), ATC_SM_THREADS);
    mbar_init(smem_u32(p_free), 1);
    mbar_init(smem_u32(o_done), 1);
    mbar_init(smem_u32(recv_full), 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    prefetch_tmap(&p.tmQ);
    prefetch_tmap(&p.tmK);
    prefetch_tmap(&p.tmV);
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  if (tid == 0) griddep_launch_dependents();
  tc_fence_before();
  cluster_arrive_release();     // barrier initialisation, acquired before the first remote access
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tr && tid == 0) tr[1] = globaltimer_ns();
  // set-up above overlaps the previous kernel; everything below reads what it
  // wrote (q, the cache rows) or writes what it may still read
  griddep_wait();

  if (warp == 8) {
    // ================= loads
    if (lane == 0) {
      const uint64_t pol_kv = policy_evict_first();
      const uint64_t pol_q = policy_evict_last();
      bool ok = true;
      uint32_t issued = 0, parity_of = 0;   // bit s: stage s's K (bit s) / V (bit 2 + s) loads in flight, and their parity
      mbar_arrive_expect_tx(smem_u32(q_full), ATC_Q_BYTES);
      tma_load_2d(smem_u32(Qs), &p.tmQ, smem_u32(q_full), 0, g * R, pol_q);
      tma_load_2d(smem_u32(Qs + 16384), &p.tmQ, smem_u32(q_full), 64, g * R, pol_q);
      // K of tile i can load once S of tile i - 2 has run; V once its P V has
      for (int i = 0; i < nt; ++i) {
        const int st = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        const int row0 = (int)((long long)g * p.cap) + (t_lo + i) * ATC_TILE;
        uint8_t* kv = Stg + st * ATC_STAGE_BYTES;
        if (!mbar_wait(smem_u32(&k_empty[st]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        const uint32_t kb = smem_u32(&k_full[st]);
        mbar_arrive_expect_tx(kb, ATC_STAGE_BYTES / 2);
        issued |= 1u << st;
        parity_of = (parity_of & ~(1u << st)) | (ph << st);
        tma_load_2d(smem_u32(kv), &p.tmK, kb, 0, row0, pol_kv);
        tma_load_2d(smem_u32(kv + 16384), &p.tmK, kb, 64, row0, pol_kv);
        if (!mbar_wait(smem_u32(&v_empty[st]), ph ^ 1u, abort_flag, p.err)) { ok = false; break; }
        const uint32_t vb = smem_u32(&v_full[st]);
        mbar_arrive_expect_tx(vb, ATC_STAGE_BYTES / 2);
        issued |= 4u << st;
        parity_of = (parity_of & ~(4u << st)) | (ph << (2 + st));
        tma_load_2d(smem_u32(kv + 32768), &p.tmV, vb, 0, row0, pol_kv);
        tma_load_2d(smem_u32(kv + 49152), &p.tmV, vb, 64, row0, pol_kv);
      }
      if (!ok) {
        mbar_wait_drain(smem_u32(q_full), 0, 100000000ull);
        for (int s2 = 0; s2 < 2; ++s2) {
          if (issued & (1u << s2)) mbar_wait_drain(smem_u32(&k_full[s2]), (parity_of >> s2) & 1u, 100000000ull);
          if (issued & (4u << s2)) mbar_wait_drain(smem_u32(&v_full[s2]), (parity_of >> (2 + s2)) & 1u, 100000000ull);
        }
      }
    }
    __syncwarp();
  } else if (warp == 9) {
    // ================= MMA issue
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_f16(1, 128, 128);
      const uint32_t idesc_o = idesc_s | (1u << 16);   // B (V) MN-major
      bool ok = mbar_wait(smem_u32(q_full), 0, abort_flag, p.err);
      bool issued_any = false;
      for (int i = 0; ok && i < nt; ++i) {
        const int st = i & 1;
        const uint32_t ph = (uint32_t)(i >> 1) & 1u;
        if (!mbar_wait(smem_u32(&k_full[st]), ph, abort_flag, p.err)) { ok = false; break; }
        if (i > 0 && !mbar_wait(smem_u32(s_free), (uint32_t)(i - 1) & 1u, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint8_t* kv = Stg + st * ATC_STAGE_BYTES;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = make_sw128_desc(smem_u32(Qs + (kk >> 2) * 16384)) + 2 * (kk & 3);
          const uint64_t bd = make_sw128_desc(smem_u32(kv + (kk >> 2) * 16384)) + 2 * (kk & 3);
          tc_mma_f16(tmem_base, ad, bd, idesc_s, kk > 0 ? 1u : 0u);
        }
        if (tr && !issued_any) tr[2] = globaltimer_ns();
        issued_any = true;
        tc_commit(smem_u32(s_full));
        tc_commit(smem_u32(&k_empty[st]));    // K of this stage free once S has run
        if (!mbar_wait(smem_u32(p_full), (uint32_t)i & 1u, abort_flag, p.err)) { ok = false; break; }
        if (!mbar_wait(smem_u32(&v_full[st]), ph, abort_flag, p.err)) { ok = false; break; }
        tc_fence_after();
        const uint32_t d_o = tmem_base + (uint32_t)(ATC_TILE * (i + 1));
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint64_t ad = make_sw128_desc(smem_u32(Ps + (kk >> 2) * 16384)) + 2 * (kk & 3);
          const uint64_t bd = make_sw128_desc_mn(smem_u32(kv + 32768 + kk * 2048), 16384, 1024);
          tc_mma_f16(d_o, ad, bd, idesc_o, kk > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&v_empty[st]));
        tc_commit(smem_u32(p_free));
      }
      if (tr) tr[4] = globaltimer_ns();
      if (ok) {
        tc_commit(smem_u32(o_done));
      } else if (issued_any) {
        tc_commit(smem_u32(o_done));
        mbar_wait_drain(smem_u32(o_done), 0, 100000000ull);
      }
    }
    __syncwarp();
  } else {
    // ================= softmax and merge: TMEM lane quarter w % 4, half w / 4
    const int lq = warp & 3, hc = warp >> 2;
    const int row = lq * 32 + lane;            // query row = TMEM lane
    const int st_id = tid;                     // 0..255
    const bool live = row < R;
    const int t = live ? row % p.L : 0;
    const uint8_t* mrow = p.mask + (long long)t * p.ldm;
    const float NEG = -__int_as_float(0x7f800000);
    float mi[ATC_NT_MAX], lh[ATC_NT_MAX];
    const uint32_t t_lane = tmem_base + ((uint32_t)(lq * 32) << 16);
    float* xmax = xch;                         // [2][128]
    float* xsum = xch + 256;                   // [ATC_NT_MAX][2][128]
    bool ok = true;
    // this thread's 64 keys of every tile of the CTA as mask bits (bit j of word
    // w: key (t_lo + i) * 128 + 64 hc + 32 w + j; keys past Lk are masked), all
    // loads issued before the first use
    uint32_t mbits[ATC_NT_MAX][2];
#pragma unroll
    for (int i = 0; i < ATC_NT_MAX; ++i) {
      const int k0 = (t_lo + i) * ATC_TILE + 64 * hc;
      if (p.mask_vec && i < nt && k0 + 64 <= p.Lk) {
        uint4 u[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) u[c] = *reinterpret_cast<const uint4*>(mrow + k0 + 16 * c);
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          uint32_t bits = 0;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const uint4 v = u[2 * w + h];
            const uint32_t wd[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int e = 0; e < 16; ++e)
              bits |= (((wd[e >> 2] >> (8 * (e & 3))) & 0xffu) != 0 ? 1u : 0u) << (16 * h + e);
          }
          mbits[i][w] = bits;
        }
      } else {
#pragma unroll
        for (int w = 0; w < 2; ++w) {
          uint32_t bits = 0;
          if (i < nt) {
            for (int e = 0; e < 32; ++e) {
              const int k = k0 + 32 * w + e;
              if (k < p.Lk && mrow[k] != 0) bits |= 1u << e;
            }
          }
          mbits[i][w] = bits;
        }
      }
      if (!live) mbits[i][0] = mbits[i][1] = 0u;
    }
    for (int i = 0; i < nt; ++i) {
      mi[i] = NEG;
      lh[i] = 0.0f;
    }
    for (int i = 0; ok && i < nt; ++i) {
      if (!named_bar_and(1, ATC_SM_THREADS, mbar_wait(smem_u32(s_full), (uint32_t)i & 1u, abort_flag, p.err))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int k0 = (t_lo + i) * ATC_TILE;
      const uint32_t mb0 = i == 0 ? mbits[0][0] : (i == 1 ? mbits[1][0] : mbits[2][0]);
      const uint32_t mb1 = i == 0 ? mbits[0][1] : (i == 1 ? mbits[1][1] : mbits[2][1]);
      const bool all_on = (mb0 & mb1) == 0xffffffffu;
      // this half's 64 raw scores; the maximum over the unmasked ones (the scale
      // is positive, so it commutes with the maximum)
      float v[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld16(t_lane + (uint32_t)(64 * hc + 16 * c), v[c]);
      tmem_wait_ld();
      float m4[4] = {NEG, NEG, NEG, NEG};
      if (all_on) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < 16; ++j) m4[j & 3] = fmaxf(m4[j & 3], v[c][j]);
      } else {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int key = 16 * c + j;
            if (((key < 32 ? mb0 : mb1) >> (key & 31)) & 1u) m4[j & 3] = fmaxf(m4[j & 3], v[c][j]);
          }
      }
      float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      // the row maximum over both halves
      xmax[hc * 128 + row] = mx;
      // the P buffer is free once the previous tile's P V has run (and the
      // other half's maximum is in shared memory)
      const bool pf = i == 0 || mbar_wait(smem_u32(p_free), (uint32_t)(i - 1) & 1u, abort_flag, p.err);
      if (!named_bar_and(1, ATC_SM_THREADS, pf)) {
        ok = false;
        break;
      }
      mx = fmaxf(mx, xmax[(hc ^ 1) * 128 + row]);
      // p = 2^(scale_log2 s - scale_log2 max): one FMA and one ex2 per score
      const float nbase = mx == NEG ? 0.0f : -__fmul_rn(mx, p.scale_log2);
      float l = 0.0f;
      uint8_t* atom = Ps + hc * 16384 + row * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float pv[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int key = 16 * c + j;
          const bool on = all_on || ((((key < 32 ? mb0 : mb1) >> (key & 31)) & 1u) != 0);
          pv[j] = on ? ex2_approx(__fmaf_rn(v[c][j], p.scale_log2, nbase)) : 0.0f;
          l += pv[j];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int chunk = 2 * c + h;
          uint4 u;
          u.x = pack2_bf16(pv[8 * h + 0], pv[8 * h + 1]);
          u.y = pack2_bf16(pv[8 * h + 2], pv[8 * h + 3]);
          u.z = pack2_bf16(pv[8 * h + 4], pv[8 * h + 5]);
          u.w = pack2_bf16(pv[8 * h + 6], pv[8 * h + 7]);
          *reinterpret_cast<uint4*>(atom + ((chunk ^ (row & 7)) << 4)) = u;
        }
      }
      if (k0 + ATC_TILE > p.Lk) {
        // V rows past Lk (p = 0 there) may hold anything the cache holds: zero
        // this half's atom of them, once the V tile has landed, so 0 * V stays 0
        const uint32_t vph = (uint32_t)(i >> 1) & 1u;
        if (!named_bar_and(1, ATC_SM_THREADS, mbar_wait(smem_u32(&v_full[i & 1]), vph, abort_flag, p.err))) {
          ok = false;
          break;
        }
        if (k0 + row >= p.Lk) {
          uint8_t* vrow = Stg + (i & 1) * ATC_STAGE_BYTES + 32768 + hc * 16384 + row * 128;
#pragma unroll
          for (int c16 = 0; c16 < 8; ++c16) *reinterpret_cast<uint4*>(vrow + c16 * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      // log2-scaled row maximum of the tile (the merges work in log2 units)
      mx = mx == NEG ? NEG : __fmul_rn(mx, p.scale_log2);
      tc_fence_before();
      mbar_arrive(smem_u32(s_free));          // S read: the next tile's S may overwrite it
      fence_proxy_async_smem();
      mbar_arrive(smem_u32(p_full));          // P (and any zeroed V rows) written
      mi[i] = mx;
      lh[i] = l;
      if (tr && i == 0 && st_id == 0) tr[3] = globaltimer_ns();
    }
    if (ok && !named_bar_and(1, ATC_SM_THREADS, mbar_wait(smem_u32(o_done), 0, abort_flag, p.err))) ok = false;
    tc_fence_after();
    if (tr && st_id == 0) tr[5] = globaltimer_ns();
    // the row sums over both halves
    for (int i = 0; i < nt; ++i) xsum[(i * 2 + hc) * 128 + row] = lh[i];
    named_bar_sync(1, ATC_SM_THREADS);
    // this CTA's tiles merged: O = sum_i 2^(m_i - M) O_i, L = sum_i 2^(m_i - M) l_i
    float M = NEG;
    for (int i = 0; i < nt; ++i) M = fmaxf(M, mi[i]);
    float wi[ATC_NT_MAX];
    float Lsum = 0.0f;
    for (int i = 0; i < nt; ++i) {
      wi[i] = (mi[i] == NEG || !ok) ? 0.0f : exp2f(mi[i] - M);
      const float li = __fadd_rn(xsum[(i * 2) * 128 + row], xsum[(i * 2 + 1) * 128 + row]);
      Lsum = __fadd_rn(Lsum, __fmul_rn(wi[i], li));
    }
    // ---- cluster merge: every CTA's MMAs are done (its stages are free for the
    // records) once all have passed this barrier
    cluster_wait_acquire();       // pairs the set-up arrive: peers' barriers are initialised
    cluster_arrive_release();
    cluster_wait_acquire();
    const int own = row / RP, lr = row - own * RP;
    const uint32_t recv_u32 = smem_u32(recv);
    const uint32_t bar_u32 = smem_u32(recv_full);
    const int own_rows = max(0, min(RP, R - q * RP));
    if (st_id == 0) mbar_arrive_expect_tx(bar_u32, (uint32_t)((S - 1) * own_rows * ATC_REC * 4));
    // records are stored group-major, [sender][16-byte group][row of the owner's
    // slice], so the 32 rows of a warp write contiguous runs
    auto g4_off = [&](int sender, int g4, int r) { return ((sender * ATC_G4 + g4) * RP + r) * 4; };
    {
      // every lane runs the TMEM loads (tcgen05.ld is warp-collective); only
      // live rows send or park their half of the record
      const int own_c = live ? own : q;
      const uint32_t dst = mapa_shared(recv_u32, (uint32_t)own_c);
      const uint32_t dbar = mapa_shared(bar_u32, (uint32_t)own_c);
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int col = 64 * hc + 16 * c;
        float acc[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) acc[j] = 0.0f;
        float ov[ATC_NT_MAX][16];
#pragma unroll
        for (int i = 0; i < ATC_NT_MAX; ++i)
          if (i < nt) tmem_ld16(t_lane + (uint32_t)(ATC_TILE * (i + 1) + col), ov[i]);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < ATC_NT_MAX; ++i)
          if (i < nt)
#pragma unroll
            for (int j = 0; j < 16; ++j) acc[j] = __fadd_rn(acc[j], __fmul_rn(wi[i], ov[i][j]));
        if (live) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int off = g4_off(q, (col >> 2) + u, lr);
            if (own == q)
              *reinterpret_cast<float4*>(recv + off) =
                  make_float4(acc[4 * u], acc[4 * u + 1], acc[4 * u + 2], acc[4 * u + 3]);
            else
              st_async_v4(dst + (uint32_t)(off * 4), acc[4 * u], acc[4 * u + 1], acc[4 * u + 2], acc[4 * u + 3],
                          dbar);
          }
        }
      }
      if (live && hc == 0) {
        const int off = g4_off(q, ATC_G4 - 1, lr);
        if (own == q)
          *reinterpret_cast<float4*>(recv + off) = make_float4(M, Lsum, 0.0f, 0.0f);
        else
          st_async_v4(dst + (uint32_t)(off * 4), M, Lsum, 0.0f, 0.0f, dbar);
      }
    }
    if (tr && st_id == 0) tr[6] = globaltimer_ns();
    // every peer's records for this CTA's rows have landed (and its own, after the CTA barrier)
    const bool got = named_bar_and(1, ATC_SM_THREADS, mbar_wait_cluster(bar_u32, 0, abort_flag, p.err));
    if (got && ok) {
      // 256 threads over own_rows x 32 groups of 4 dims: o = sum_s 2^(M_s - Mt) O_s / sum_s 2^(M_s - Mt) L_s
      for (int item = st_id; item < own_rows * 32; item += ATC_SM_THREADS) {
        const int r = item >> 5, d4 = item & 31;
        float Mt = NEG;
        for (int s2 = 0; s2 < S; ++s2) Mt = fmaxf(Mt, recv[g4_off(s2, ATC_G4 - 1, r)]);
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        float den = 0.0f;
        if (Mt != NEG) {
          for (int s2 = 0; s2 < S; ++s2) {
            const float2 ml = *reinterpret_cast<const float2*>(recv + g4_off(s2, ATC_G4 - 1, r));
            if (ml.x == NEG) continue;
            const float w = exp2f(ml.x - Mt);
            den = __fadd_rn(den, __fmul_rn(w, ml.y));
            const float4 ov = *reinterpret_cast<const float4*>(recv + g4_off(s2, d4, r));
            acc.x = __fadd_rn(acc.x, __fmul_rn(w, ov.x));
            acc.y = __fadd_rn(acc.y, __fmul_rn(w, ov.y));
            acc.z = __fadd_rn(acc.z, __fmul_rn(w, ov.z));
            acc.w = __fadd_rn(acc.w, __fmul_rn(w, ov.w));
          }
        }
        const float inv = den > 0.0f ? 1.0f / den : 0.0f;
        const int grow = q * RP + r;
        const int h = g * G + grow / p.L, tt = grow % p.L;
        uint8_t* dsto = reinterpret_cast<uint8_t*>(p.o) + (((long long)tt * p.Hq + h) * 128 + d4 * 4) * 2;
        uint2 pk;
        pk.x = pack_bf16(acc.x * inv, acc.y * inv);
        pk.y = pack_bf16(acc.z * inv, acc.w * inv);
        *reinterpret_cast<uint2*>(dsto) = pk;
      }
    }
    if (!got && st_id == 0 && S > 1) {
      // aborting: give peers' records in flight time to land before this CTA exits
      mbar_wait_drain(bar_u32, 0, 100000000ull);
    }
  }
  if (warp >= 8) {
    cluster_wait_acquire();
    cluster_arrive_release();
    cluster_wait_acquire();
  }
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
  if (tr && tid == 0) tr[7] = globaltimer_ns();
}

}  // namespace simsd
