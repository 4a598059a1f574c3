// sm_100a building blocks: mbarriers, TMA tensor loads, tcgen05 (MMA, TMEM
// alloc/load, commit, fences) and bounded waits.
//
// Every wait in this library is bounded: it polls an mbarrier until it
// completes, a CTA-wide abort flag is raised, or a wall-clock limit
// (SIMSD_WAIT_LIMIT_NS, read from %globaltimer) runs out.  A timed-out wait
// raises the abort flag so that every later wait in the CTA returns at once,
// records SIMSD_DEV_ERR_TIMEOUT in the caller's device error word and lets the
// kernel drain its own async copies and free its TMEM before it returns.  No
// kernel here traps or spins without a limit.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#ifndef SIMSD_WAIT_LIMIT_NS
#define SIMSD_WAIT_LIMIT_NS 2000000000ull   // 2 s: a pipeline stage needs microseconds
#endif

// device error word bits (OR-ed into the caller's error word)
#define SIMSD_DEV_ERR_TIMEOUT   1
#define SIMSD_DEV_ERR_BAD_INDEX 2
#define SIMSD_DEV_ERR_CAPACITY  4   // expert-parallel bucket overflow

namespace simsd {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase of `bar` with parity `parity`.  Returns false when
// the CTA is aborting (flag already raised, or this wait ran out of time).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* err_word) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > SIMSD_WAIT_LIMIT_NS) {
      *abort_flag = 1;
      if (err_word) atomicOr(err_word, SIMSD_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}
// Bounded wait that ignores the abort flag: used only while draining, to make
// sure no async copy is still writing shared memory when the CTA exits.
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// 2-D tiled load: box at (c0 = innermost element index, c1 = row) into smem.
// c0 * element size must be a multiple of 16 bytes (callers only pass multiples
// of 64 elements).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const void* tmap, uint32_t bar, int c0,
                                            int c1, int c2, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "l"(policy)
      : "memory");
}

// Fetch a 2-D box of a tensor into L2 only (no shared memory, no barrier): lets
// a weight stream keep more DRAM requests in flight than its shared-memory ring
// holds.  Same coordinate rules as tma_load_2d.
__device__ __forceinline__ void tma_prefetch_l2_2d(const void* tmap, int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.prefetch.tensor.2d.L2.global.tile.L2::cache_hint [%0, {%1, %2}], %3;" ::"l"(
          reinterpret_cast<uint64_t>(tmap)),
      "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/fp16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (+)= A B^T with A, B tf32 operands read as 32-bit words from shared memory
// (K = 8 per instruction); the fp32 tensor-core path splits every operand so
// that each word it hands in is exactly representable in tf32.
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Split the four fp32 words hi[v] into tf32 parts: hi[v] keeps the sign,
// exponent and top 10 mantissa bits of each word (exact in tf32), lo[v] gets
// the rest, x - hi (exact in fp32), cut to tf32 the same way.  hi + lo matches
// x to 2^-21 of |x|, so hi*hi' + hi*lo' + lo*hi' matches x*x' to about
// 3 * 2^-21 relative.  Infinities and NaNs keep hi = x and lo = 0.
__device__ __forceinline__ float tf32_hi(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }
__device__ __forceinline__ float tf32_lo(float x, float h) {
  return (__float_as_uint(x) & 0x7f800000u) == 0x7f800000u ? 0.0f : tf32_hi(__fsub_rn(x, h));
}
__device__ __forceinline__ void split_tf32(float4* hi, float4* lo, int v) {
  const float4 x = hi[v];
  const float4 h = make_float4(tf32_hi(x.x), tf32_hi(x.y), tf32_hi(x.z), tf32_hi(x.w));
  lo[v] = make_float4(tf32_lo(x.x, h.x), tf32_lo(x.y, h.y), tf32_lo(x.z, h.z), tf32_lo(x.w, h.w));
  hi[v] = h;
}
// Shared-memory writes of this thread (generic proxy) become visible to the
// tensor cores and TMA (async proxy) that are ordered after this fence.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Arrive (once) on `bar` when every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}
// 32 TMEM lanes x 16 columns of 32-bit: thread i of the warp gets lane (base+i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major, 128-byte-swizzled operand tile
// whose rows are 128 bytes (64 bf16) and whose 8-row swizzle atoms are 1024
// bytes apart.  The tile base must be 1024-byte aligned; stepping along K inside
// the 128-byte row is done by adding (bytes >> 4) to the start-address field.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);        // start address        [0,14)
  d |= (uint64_t)(16 >> 4) << 16;                     // leading byte offset  [16,30) (unused)
  d |= (uint64_t)(1024 >> 4) << 32;                   // stride byte offset   [32,46)
  d |= (uint64_t)1 << 46;                             // descriptor version   [46,48)
  d |= (uint64_t)2 << 61;                             // SWIZZLE_128B         [61,64)
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulate, A and B of the same
// 16-bit type (bf16 when is_bf16 else fp16), both K-major, shape M x N.
__host__ __device__ __forceinline__ uint32_t make_idesc_f16(int is_bf16, int M, int N) {
  uint32_t d = 0;
  d |= 1u << 4;                                 // D format: f32
  d |= (uint32_t)(is_bf16 ? 1 : 0) << 7;        // A format
  d |= (uint32_t)(is_bf16 ? 1 : 0) << 10;       // B format
  d |= (uint32_t)(N >> 3) << 17;                // N / 8
  d |= (uint32_t)(M >> 4) << 24;                // M / 16
  return d;
}

// Instruction descriptor, kind::tf32: fp32 accumulate, A and B tf32 (format 2),
// both K-major, shape M x N.
__host__ __device__ __forceinline__ uint32_t make_idesc_tf32(int M, int N) {
  uint32_t d = 0;
  d |= 1u << 4;                                 // D format: f32
  d |= 2u << 7;                                 // A format: tf32
  d |= 2u << 10;                                // B format: tf32
  d |= (uint32_t)(N >> 3) << 17;                // N / 8
  d |= (uint32_t)(M >> 4) << 24;                // M / 16
  return d;
}

// ---------------------------------------------------------------- clusters / DSMEM
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_nctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// Every thread of every CTA in the cluster: makes barrier initialisation (and
// other shared-memory writes before it) visible cluster-wide.  Used once, right
// after set-up, when no CTA can be held up by another's work.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split form: every thread arrives (releasing its shared-memory writes, e.g.
// barrier initialisation) and later waits (acquiring the other CTAs'), so the
// wait can sit right before the first remote access instead of on the start-up
// path.  Each thread must wait once after it arrived, before the CTA exits.
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address in CTA `rank`'s shared memory of the variable at local address `a`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(rank));
  return d;
}
// 16-byte store into another CTA's shared memory that completes `bytes` of the
// transaction count of the mbarrier at `remote_bar` (same CTA as the data).
__device__ __forceinline__ void st_async_v4(uint32_t remote_addr, float a, float b, float c, float d,
                                            uint32_t remote_bar) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.b32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
          remote_addr),
      "r"(__float_as_uint(a)), "r"(__float_as_uint(b)), "r"(__float_as_uint(c)), "r"(__float_as_uint(d)),
      "r"(remote_bar)
      : "memory");
}
// Arrive on an mbarrier in another CTA of the cluster, releasing this thread's
// prior memory accesses (and, through a preceding CTA barrier, its CTA's) at
// cluster scope.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (as mbar_wait) for a phase completed by other CTAs of the
// cluster, acquiring their writes at cluster scope.
__device__ __forceinline__ bool mbar_wait_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                  int* err_word) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > SIMSD_WAIT_LIMIT_NS) {
      *abort_flag = 1;
      if (err_word) atomicOr(err_word, SIMSD_DEV_ERR_TIMEOUT);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait_cluster_drain(uint32_t bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (!mbar_try_wait_cluster(bar, parity)) {
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
  return true;
}

// ---------------------------------------------------------------- cross-GPU signals
// Add to an int in another GPU's memory (an NVLink peer mapping) with release
// semantics at system scope: every write this thread made before it (and,
// through a preceding CTA barrier, its CTA's) is visible to a reader that
// acquires the new value.
__device__ __forceinline__ void red_add_release_sys(int* addr, int v) {
  asm volatile("red.release.sys.global.add.s32 [%0], %1;" ::"l"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel_sys(int* addr, int v) {
  int old;
  asm volatile("atom.acq_rel.sys.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(addr), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ int ld_acquire_sys(const int* addr) {
  int v;
  asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with programmatic stream
// serialization may start before the previous kernel on its stream finishes;
// griddep_wait() blocks until that kernel has completed and its writes are
// visible (a no-op when the launch had no such dependency), and
// griddep_launch_dependents() lets the next kernel begin launching early.
// Every kernel here triggers first and waits second: the next kernel's own
// griddep_wait() still orders it after this one (completion is transitive),
// so the early trigger only lets its set-up and weight prefetch overlap.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------- misc
__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
// Named barrier over `nthreads` threads that also ANDs a predicate across them.
__device__ __forceinline__ bool named_bar_and(int id, int nthreads, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ float load_f(const void* p, int64_t i, int dtype) {
  if (dtype == 0) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == 1) return __half2float(reinterpret_cast<const __half*>(p)[i]);
  return reinterpret_cast<const float*>(p)[i];
}
__device__ __forceinline__ void store_f(void* p, int64_t i, float v, int dtype) {
  if (dtype == 0)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else if (dtype == 1)
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}
// fp32 -> the bits of a bf16 (dtype 0) or fp16 (dtype 1), round to nearest even
__device__ __forceinline__ uint16_t f32_to_16bit(float v, int dtype) {
  if (dtype == 0) return __bfloat16_as_ushort(__float2bfloat16_rn(v));
  return __half_as_ushort(__float2half_rn(v));
}
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

}  // namespace simsd
