// extern "C" entry points of libsimsd_b200.so (declared in include/simsd_b200.h).
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <initializer_list>
#include <type_traits>
#include <utility>
#include <cstdio>
#include <cmath>
#include <cstdlib>
#include <mutex>

#include "moe.cuh"
#include "norm.cuh"
#include "attn.cuh"
#include "attn_tc.cuh"
#include "simsd_b200.h"
#include "simt_gemm.cuh"
#include "tc_cluster.cuh"
#include "tc_gemm.cuh"

using namespace simsd;

namespace {

constexpr int kMaxDev = 64;
std::mutex g_mu;
int g_sm_count[kMaxDev];
bool g_smem_attr[kMaxDev][40];
unsigned long long* g_trace = nullptr;
size_t g_trace_bytes = 0;
size_t g_trace_used = 0;   // bytes of the trace buffer taken by earlier launches

// The trace record of the next GEMM launch of `ctas` CTAs: the next free
// 64 * ctas bytes of the buffer, or nullptr once it is full (or unset).
unsigned long long* trace_slot(long long ctas) {
  std::lock_guard<std::mutex> lk(g_mu);
  const size_t need = (size_t)ctas * 64;
  if (g_trace == nullptr || g_trace_used + need > g_trace_bytes) return nullptr;
  unsigned long long* t = g_trace + g_trace_used / 8;
  g_trace_used += need;
  return t;
}
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

std::atomic<int> g_launch_flags{0};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

inline bool pdl_on() { return (g_launch_flags.load(std::memory_order_relaxed) & SIMSD_LAUNCH_PDL) != 0; }

// Launch `kern` on `s`, as a programmatic dependent of the previous kernel on
// the stream when SIMSD_LAUNCH_PDL is set (every kernel here starts with
// griddepcontrol.wait before it reads anything another kernel produced).
template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  if (pdl_on()) {
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  if (cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? SIMSD_OK : SIMSD_ERR_LAUNCH;
}
inline int esize(int dtype) { return dtype == SIMSD_F32 ? 4 : 2; }
inline long long cdiv(long long a, long long b) { return (a + b - 1) / b; }

int current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDev) return -1;
  return dev;
}

int sm_count_of(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 0;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

int ensure_encode() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_encode) return SIMSD_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) !=
          cudaSuccess ||
      q != cudaDriverEntryPointSuccess || fn == nullptr)
    return SIMSD_ERR_DEVICE;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return SIMSD_OK;
}

// 128-byte-swizzled tiled map: box = {one 128-byte row (64 16-bit or 32 fp32 elements), box_rows[, 1]}.
int encode_map(CUtensorMap* m, const void* base, int dtype, int rank, const uint64_t* dims,
               const uint64_t* stride_bytes, uint32_t box_rows) {
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return SIMSD_ERR_ALIGN;
  for (int i = 0; i + 1 < rank; ++i)
    if ((stride_bytes[i] & 15) != 0 || stride_bytes[i] == 0) return SIMSD_ERR_ALIGN;
  cuuint64_t gdim[3];
  cuuint64_t gstride[2];
  cuuint32_t box[3] = {dtype == SIMSD_F32 ? 32u : 64u, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) gdim[i] = dims[i];
  for (int i = 0; i + 1 < rank; ++i) gstride[i] = stride_bytes[i];
  const CUtensorMapDataType dt = dtype == SIMSD_BF16  ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : dtype == SIMSD_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  const CUresult r = g_encode(m, dt, rank, const_cast<void*>(base), gdim, gstride, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? SIMSD_OK : SIMSD_ERR_ALIGN;
}

int pick_bmax_rows(long long rows) {
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 64) return 64;
  if (rows <= 128) return 128;
  return 256;
}

// K atoms per ring stage: SIMSD_TC_KS (1, 2 or 4) overrides the default; stages
// must still fit twice in shared memory, so wide activation tiles cap it.
// Ring budget: SIMSD_TC_RING (196 or 96, KB) overrides the default.
int env_choice(const char* name, std::initializer_list<int> allowed, int dflt) {
  const char* e = getenv(name);
  if (!e) return dflt;
  const int v = atoi(e);
  for (int a : allowed)
    if (a == v) return v;
  return dflt;
}

int ring_kb() {
  static const int v = env_choice("SIMSD_TC_RING", {196, 96}, 196);
  return v;
}

// Weight stages a programmatic dependent launch fetches before waiting for the
// previous kernel: SIMSD_TC_PREFETCH overrides the default.  The activation
// boxes of those stages queue behind them, so a deep prefetch delays the first
// MMA once the previous kernel is done.
int prefetch_stages() {
  static const int v = env_choice("SIMSD_TC_PREFETCH", {1, 2, 3, 4, 6, 10}, 2);
  return v;
}

inline bool use_counters() {
  return (g_launch_flags.load(std::memory_order_relaxed) & SIMSD_LAUNCH_INKERNEL_REDUCE) != 0;
}
// grouped (MoE) GEMMs: in-kernel reduction unless SIMSD_LAUNCH_GROUPED_FIXUP
inline bool use_counters_grouped() {
  return (g_launch_flags.load(std::memory_order_relaxed) & SIMSD_LAUNCH_GROUPED_FIXUP) == 0;
}

// Weight stages the cluster GEMM requests into L2 ahead of its shared-memory
// ring: SIMSD_TC_L2_AHEAD overrides the default.
int l2_ahead_stages() {
  static const int v = env_choice("SIMSD_TC_L2_AHEAD", {0, 2, 4, 8, 12, 16, 24}, 0);
  return v;
}

int ks_for(int bmax) {
  static const int req = env_choice("SIMSD_TC_KS", {1, 2, 4}, 2);
  if (ring_kb() == 96) return std::min(req, bmax <= 32 ? 2 : 1);
  return std::min(req, bmax <= 64 ? 4 : 2);
}

template <int BMAX, int KS, int RING>
int launch_tc_b(const TcGemmArgs& a, int grid, cudaStream_t s, int dev) {
  constexpr int smem = TcConfig<BMAX, KS, RING>::SMEM_BYTES;
  constexpr int bi = BMAX == 16 ? 0 : BMAX == 32 ? 1 : BMAX == 64 ? 2 : BMAX == 128 ? 3 : 4;
  constexpr int idx = (RING == 196 ? 0 : 15) + bi * 3 + (KS == 1 ? 0 : KS == 2 ? 1 : 2);
  static_assert(RING == 196 || 2 * (TcConfig<BMAX, KS, RING>::SMEM_BYTES + 1024) <= 228 * 1024,
                "two CTAs of the small ring must share an SM");
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_smem_attr[dev][idx]) {
      if (cudaFuncSetAttribute(tc_gemm_kernel<BMAX, KS, RING>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
          cudaSuccess)
        return SIMSD_ERR_LAUNCH;
      g_smem_attr[dev][idx] = true;
    }
  }
  TcGemmArgs args = a;
  args.pdl = pdl_on() ? 1 : 0;
  args.prefetch = prefetch_stages();
  args.trace = trace_slot(grid);
  return launch(tc_gemm_kernel<BMAX, KS, RING>, dim3(grid), dim3(TC_THREADS), smem, s, args);
}

template <int BMAX>
int launch_tc_ks(const TcGemmArgs& a, int grid, cudaStream_t s, int dev) {
  const int ks = ks_for(BMAX);
  if (ring_kb() == 96) {
    if constexpr (BMAX <= 32) {
      if (ks == 2) return launch_tc_b<BMAX, 2, 96>(a, grid, s, dev);
    }
    if constexpr (BMAX <= 128) return launch_tc_b<BMAX, 1, 96>(a, grid, s, dev);
  }
  switch (ks) {
    case 1: return launch_tc_b<BMAX, 1, 196>(a, grid, s, dev);
    case 2: return launch_tc_b<BMAX, 2, 196>(a, grid, s, dev);
    default:
      if constexpr (BMAX <= 64) return launch_tc_b<BMAX, 4, 196>(a, grid, s, dev);
      else return launch_tc_b<BMAX, 2, 196>(a, grid, s, dev);
  }
}

int launch_tc(int bmax, const TcGemmArgs& a, int grid, cudaStream_t s, int dev) {
  switch (bmax) {
    case 16: return launch_tc_ks<16>(a, grid, s, dev);
    case 32: return launch_tc_ks<32>(a, grid, s, dev);
    case 64: return launch_tc_ks<64>(a, grid, s, dev);
    case 128: return launch_tc_ks<128>(a, grid, s, dev);
    case 256: return launch_tc_ks<256>(a, grid, s, dev);
  }
  return SIMSD_ERR_UNSUPPORTED;
}

// Fixup launch: one block per CTA boundary of the GEMM (grid - 1) and 16-row chunk.
// Small kernels that run between tensor-core GEMMs ask for the largest
// shared-memory carve-out: an SM changes its L1/shared split only when idle, so a
// block configured otherwise would keep the next GEMM's CTA (about 200 KB of
// shared memory) off its SM until the block exits.
template <typename F>
int prefer_shared(F* kern, int dev, int idx) {
  static bool done[kMaxDev][16];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!done[dev][idx]) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared) !=
        cudaSuccess)
      return SIMSD_ERR_LAUNCH;
    done[dev][idx] = true;
  }
  return SIMSD_OK;
}

template <int BMAX>
int launch_fixup_b(const TcFixupArgs& f, cudaStream_t s, int dev) {
  if (f.grid <= 1) return SIMSD_OK;
  constexpr int idx = BMAX == 16 ? 0 : BMAX == 32 ? 1 : BMAX == 64 ? 2 : BMAX == 128 ? 3 : 4;
  if (prefer_shared(tc_fixup_kernel<BMAX>, dev, idx) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  const size_t smem = f.group_counts ? (size_t)2 * (f.num_groups + 1) * sizeof(int) : 0;
  return launch(tc_fixup_kernel<BMAX>, dim3((unsigned)(f.grid - 1), BMAX / 16), dim3(128), smem, s, f);
}

int launch_fixup(int bmax, const TcFixupArgs& f, cudaStream_t s) {
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  switch (bmax) {
    case 16: return launch_fixup_b<16>(f, s, dev);
    case 32: return launch_fixup_b<32>(f, s, dev);
    case 64: return launch_fixup_b<64>(f, s, dev);
    case 128: return launch_fixup_b<128>(f, s, dev);
    case 256: return launch_fixup_b<256>(f, s, dev);
  }
  return SIMSD_ERR_UNSUPPORTED;
}

TcFixupArgs fixup_args(const TcGemmArgs& a, int grid) {
  TcFixupArgs f;
  f.partials = a.partials;
  f.out = a.out;
  f.bias = a.bias;
  f.group_counts = a.group_counts;
  f.tables = a.tables;
  f.ld_out = a.ld_out;
  f.single_rows = a.single_rows;
  f.num_groups = a.num_groups;
  f.kb = a.kb;
  f.rows_out = a.rows_out;
  f.row_tiles = a.row_tiles;
  f.silu = a.silu;
  f.is_bf16 = a.is_bf16;
  f.grid = grid;
  return f;
}

// Does the stream-K split of (tiles x kb) over `grid` CTAs cut any tile?
bool any_split_tile(long long tiles, long long kb, long long grid) {
  const int iters = (int)(tiles * kb);
  const SkSplit sk(iters, (int)std::min<long long>(grid, iters));
  for (int t = 0; t < (int)tiles; ++t)
    if (sk.owner(t * (int)kb) != sk.owner(t * (int)kb + (int)kb - 1)) return true;
  return false;
}

// ---------------------------------------------------------------- thin linear plan
constexpr long long TC_MIN_ATOMS_PER_CTA = 8;

struct ThinPlan {
  int bmax, row_tiles, kb, grid;
  long long tiles, iters;
  size_t ws_bytes;
};

ThinPlan plan_thin(int M, int N, int K, int epilogue, int split, int sms) {
  ThinPlan p{};
  p.bmax = pick_bmax_rows(M);
  p.row_tiles = (int)(epilogue == SIMSD_EPI_SILU_MUL ? cdiv(N, 64) : cdiv(N, 128));
  p.kb = (int)cdiv(K, 64);
  p.tiles = cdiv(M, p.bmax) * p.row_tiles;
  p.iters = p.tiles * p.kb;
  long long g;
  if (split > 0) {
    g = std::min<long long>(p.tiles * split, p.iters);
  } else {
    // at least TC_MIN_ATOMS_PER_CTA K atoms per CTA: a CTA's set-up and first
    // ring fill cost a few microseconds, and every split tile adds fp32
    // partials and a reduction, so a small GEMM uses fewer CTAs instead
    g = std::min<long long>(sms > 0 ? sms : 148, p.iters / TC_MIN_ATOMS_PER_CTA);
  }
  g = std::max<long long>(1, std::min<long long>(g, TC_MAX_GRID));
  p.grid = (int)g;
  p.ws_bytes = WS_COUNTER_BYTES + align256((size_t)2 * p.grid * p.bmax * 128 * sizeof(float));
  return p;
}

// ---------------------------------------------------------------- cluster path
// K atoms per ring stage of tc_cluster_kernel: two (per-stage barrier and
// issue overheads halve; at 64 activation rows that leaves three stages, 96 KB
// of weights in flight, and still measured 12-14 % faster than seven
// single-atom stages).  fp32 operands (F32) hold every atom twice (tf32 hi and
// lo parts): one atom a stage.
constexpr int cluster_ks(int bmax, bool f32 = false) { return f32 ? 1 : (bmax <= 64 ? 2 : 1); }

template <int BMAX, bool F32 = false, bool AG = false>
int cluster_prepare(int dev) {
  constexpr int KS = cluster_ks(BMAX, F32);
  constexpr int smem = TcClusterConfig<BMAX, KS, F32>::SMEM_BYTES;
  static bool done[kMaxDev];
  std::lock_guard<std::mutex> lk(g_mu);
  if (!done[dev]) {
    if (cudaFuncSetAttribute(tc_cluster_kernel<BMAX, KS, F32, AG>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return SIMSD_ERR_LAUNCH;
    done[dev] = true;
  }
  return SIMSD_OK;
}

// Clusters of S CTAs of tc_cluster_kernel<BMAX> that fit on the device at once
// (the occupancy calculator knows how clusters pack into GPCs); 0 if none.
template <int BMAX, bool F32 = false>
int max_clusters_b(int S, int dev) {
  constexpr int KS = cluster_ks(BMAX, F32);
  static int cache[kMaxDev][TC_CL_MAX + 1];
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cache[dev][S] != 0) return cache[dev][S] > 0 ? cache[dev][S] : 0;
  }
  if (cluster_prepare<BMAX, F32>(dev) != SIMSD_OK) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S);
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TcClusterConfig<BMAX, KS, F32>::SMEM_BYTES;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_cluster_kernel<BMAX, KS, F32>, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  cache[dev][S] = n > 0 ? n : -1;
  return n > 0 ? n : 0;
}

int max_clusters(int bmax, int S, int dev, bool f32 = false) {
  switch (bmax) {
    case 16: return f32 ? max_clusters_b<16, true>(S, dev) : max_clusters_b<16>(S, dev);
    case 32: return f32 ? max_clusters_b<32, true>(S, dev) : max_clusters_b<32>(S, dev);
    case 64: return f32 ? max_clusters_b<64, true>(S, dev) : max_clusters_b<64>(S, dev);
  }
  return 0;
}

template <int BMAX, bool F32 = false, bool AG = false>
int launch_cluster_b(const TcClusterArgs& a, int S, int C, cudaStream_t s, int dev) {
  constexpr int KS = cluster_ks(BMAX, F32);
  if (cluster_prepare<BMAX, F32, AG>(dev) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  TcClusterArgs args = a;
  args.pdl = pdl_on() ? 1 : 0;
  args.prefetch = prefetch_stages();
  args.l2_ahead = l2_ahead_stages();
  args.trace = trace_slot((long long)C * S);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(C * S));
  cfg.blockDim = dim3(TC_THREADS);
  cfg.dynamicSmemBytes = TcClusterConfig<BMAX, KS, F32>::SMEM_BYTES;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  int n = 0;
  attr[n].id = cudaLaunchAttributeClusterDimension;
  attr[n].val.clusterDim.x = (unsigned)S;
  attr[n].val.clusterDim.y = 1;
  attr[n].val.clusterDim.z = 1;
  ++n;
  if (pdl_on()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  if (cudaLaunchKernelEx(&cfg, tc_cluster_kernel<BMAX, KS, F32, AG>, args) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  return cudaGetLastError() == cudaSuccess ? SIMSD_OK : SIMSD_ERR_LAUNCH;
}

int launch_cluster(int bmax, const TcClusterArgs& a, int S, int C, cudaStream_t s, int dev, bool f32 = false) {
  if (a.world > 1) {
    // fused all-gather: the instantiation with the peer-store epilogue (16-bit only)
    if (f32) return SIMSD_ERR_UNSUPPORTED;
    switch (bmax) {
      case 16: return launch_cluster_b<16, false, true>(a, S, C, s, dev);
      case 32: return launch_cluster_b<32, false, true>(a, S, C, s, dev);
      case 64: return launch_cluster_b<64, false, true>(a, S, C, s, dev);
    }
    return SIMSD_ERR_UNSUPPORTED;
  }
  switch (bmax) {
    case 16: return f32 ? launch_cluster_b<16, true>(a, S, C, s, dev) : launch_cluster_b<16>(a, S, C, s, dev);
    case 32: return f32 ? launch_cluster_b<32, true>(a, S, C, s, dev) : launch_cluster_b<32>(a, S, C, s, dev);
    case 64: return f32 ? launch_cluster_b<64, true>(a, S, C, s, dev) : launch_cluster_b<64>(a, S, C, s, dev);
  }
  return SIMSD_ERR_UNSUPPORTED;
}

// Cluster size S and cluster count C for `tiles` output tiles of kb K blocks:
// the fewest K blocks on any CTA (tiles per cluster x K blocks per rank), then
// more CTAs, then the smaller cluster.  S = 0: no cluster plan (use stream-K).
struct ClusterPlan {
  int S = 0, C = 0;
};
// SIMSD_TC_MAX_CTAS caps the CTAs of a cluster launch (measurement knob;
// default: no cap beyond what fits)
int cluster_cta_cap() {
  static const int v = [] {
    const char* e = getenv("SIMSD_TC_MAX_CTAS");
    const int n = e ? atoi(e) : 0;
    return n > 0 ? n : 1 << 30;
  }();
  return v;
}

// Cluster plan: tile c, c + C, ... to cluster c, the K blocks of each split
// over the S ranks; the S with the fewest K blocks per CTA (then the most
// CTAs).  Whole tiles per cluster leave the SMs that no cluster fills free for
// the next launch's CTAs, which fetch their first weight stages there while
// this launch drains (programmatic dependent launch).
ClusterPlan plan_cluster(int bmax, long long tiles, int kb, int dev, bool f32 = false) {
  ClusterPlan best;
  long long best_cost = -1, best_ctas = 0;
  for (int S = 1; S <= TC_CL_MAX && S <= kb; ++S) {
    const long long cmax = std::min<long long>(max_clusters(bmax, S, dev, f32), cluster_cta_cap() / S);
    if (cmax <= 0) continue;
    const long long c0 = std::min(cmax, tiles);
    const long long w = cdiv(tiles, c0);
    const long long C = cdiv(tiles, w);
    const long long cost = w * cdiv(kb, S);
    const long long ctas = C * S;
    if (best_cost < 0 || cost < best_cost || (cost == best_cost && ctas > best_ctas)) {
      best_cost = cost;
      best_ctas = ctas;
      best.S = S;
      best.C = (int)C;
    }
  }
  return best;
}

// The plan for `tiles` output tiles with the cluster size pinned to `S` (the
// K split of each tile fixed): as many clusters as fit, tiles dealt evenly.
ClusterPlan plan_cluster_with_s(int bmax, long long tiles, int S, int dev, bool f32 = false) {
  ClusterPlan cp;
  const long long cmax = std::min<long long>(max_clusters(bmax, S, dev, f32), cluster_cta_cap() / S);
  if (cmax <= 0 || tiles <= 0) return cp;
  const long long c0 = std::min(cmax, tiles);
  const long long w = cdiv(tiles, c0);
  cp.S = S;
  cp.C = (int)cdiv(tiles, w);
  return cp;
}

// Clusters of S CTAs of attn_tc_kernel that fit on the device at once (0: S does
// not run here).  Sets the kernel's shared-memory and cluster-size attributes.
int attn_max_clusters(int S, int dev) {
  static int cache[kMaxDev][ATC_CL_MAX_NP + 1];
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (cache[dev][S] != 0) return cache[dev][S] > 0 ? cache[dev][S] : 0;
  }
  if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATC_SMEM) != cudaSuccess ||
      cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
    (void)cudaGetLastError();
    return 0;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)S);
  cfg.blockDim = dim3(ATC_THREADS);
  cfg.dynamicSmemBytes = ATC_SMEM;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = (unsigned)S;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, attn_tc_kernel, &cfg) != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  cache[dev][S] = n > 0 ? n : -1;
  return n > 0 ? n : 0;
}

// SIMSD_ATTN_TC=0 keeps verify attention on the mma.sync split kernel + combine.
bool attn_tc_enabled() {
  static const bool v = env_choice("SIMSD_ATTN_TC", {0, 1}, 1) == 1;
  return v;
}

bool cluster_enabled() {
  static const bool v = env_choice("SIMSD_TC_CLUSTER", {0, 1}, 1) == 1;
  return v;
}

// One tc_cluster_kernel launch for a thin linear with M <= 64 (layouts already
// checked by thin_tc_possible).  world > 1: the fused all-gather variant, with
// peer outputs / signal blocks and this rank's column offset.  Returns
// SIMSD_ERR_UNSUPPORTED when no cluster plan fits.
// Up to three weights whose outputs are concatenated along N (plain epilogue):
// w[i] [n[i], K] with row stride ldw[i]; every part but the last a multiple of 128 rows.
struct CatSpec {
  int parts = 0;
  const void* w[3] = {nullptr, nullptr, nullptr};
  long long ldw[3] = {0, 0, 0};
  int n[3] = {0, 0, 0};
};

int thin_cluster(const void* x, long long ldx_m, const void* w, long long ldw_n, const void* w_up, const void* bias,
                 void* y, long long ldy, int M, int N, int K, int dtype, bool silu, int* err, void* const* peer_y,
                 int col_offset, int world, int rank, cudaStream_t s, int dev,
                 unsigned long long* amax_keys = nullptr, long long* amax_idx = nullptr, int* amax_count = nullptr,
                 const CatSpec* cat = nullptr, int plan_n = 0) {
  const bool f32 = dtype == SIMSD_F32;   // fp32 operands: 32-element K blocks, tf32 split on chip
  const long long esz = f32 ? 4 : 2;
  const int bmax = pick_bmax_rows(M);
  const long long row_tiles = silu ? cdiv(N, 64) : cdiv(N, 128);
  const int kb = (int)cdiv(K, f32 ? 32 : 64);
  ClusterPlan cp = plan_cluster(bmax, row_tiles, kb, dev, f32);
  if (plan_n > 0) {
    // the K split a single-GPU call with plan_n output columns would use, so
    // every output element is summed exactly as it would be there
    const ClusterPlan full = plan_cluster(bmax, silu ? cdiv(plan_n, 64) : cdiv(plan_n, 128), kb, dev, f32);
    if (full.S <= 0) return SIMSD_ERR_UNSUPPORTED;
    cp = plan_cluster_with_s(bmax, row_tiles, full.S, dev, f32);
  }
  if (cp.S <= 0) return SIMSD_ERR_UNSUPPORTED;
  if (ensure_encode() != SIMSD_OK) return SIMSD_ERR_DEVICE;
  TcClusterArgs a;
  memset(&a, 0, sizeof(a));
  // a one-row operand's stride is never used; give the map any legal one
  const long long pad_ld = ((K * esz + 15) / 16) * 16 / esz;
  const long long lx = (M > 1) ? ldx_m : pad_ld;
  const long long lw = (N > 1) ? ldw_n : pad_ld;
  const uint64_t xd[2] = {(uint64_t)K, (uint64_t)M}, xs[1] = {(uint64_t)(lx * esz)};
  const uint64_t wd[2] = {(uint64_t)K, (uint64_t)N}, wsb[1] = {(uint64_t)(lw * esz)};
  int rc = encode_map(&a.tmB, x, dtype, 2, xd, xs, (uint32_t)bmax);
  if (cat != nullptr && cat->parts > 1) {
    CUtensorMap* maps[3] = {&a.tmA0, &a.tmA1, &a.tmA2};
    for (int i = 0; i < cat->parts && rc == SIMSD_OK; ++i) {
      const long long li = cat->n[i] > 1 ? cat->ldw[i] : pad_ld;
      const uint64_t di[2] = {(uint64_t)K, (uint64_t)cat->n[i]}, si[1] = {(uint64_t)(li * esz)};
      rc = encode_map(maps[i], cat->w[i], dtype, 2, di, si, 128);
    }
    a.cat_t1 = cat->n[0] / 128;
    a.cat_t2 = cat->parts > 2 ? (cat->n[0] + cat->n[1]) / 128 : 1 << 30;
  } else {
    if (rc == SIMSD_OK) rc = encode_map(&a.tmA0, w, dtype, 2, wd, wsb, silu ? 64 : 128);
    if (rc == SIMSD_OK && silu) rc = encode_map(&a.tmA1, w_up, dtype, 2, wd, wsb, 64);
  }
  if (rc != SIMSD_OK) return rc;
  a.out = y;
  a.bias = bias;
  a.err = err;
  a.ld_out = ldy;
  a.rows = M;
  a.kb = kb;
  a.rows_out = N;
  a.row_tiles = (int)row_tiles;
  a.silu = silu ? 1 : 0;
  a.is_bf16 = dtype == SIMSD_BF16 ? 1 : 0;
  a.amax_keys = amax_keys;
  a.amax_idx = amax_idx;
  a.amax_count = amax_count;
  a.world = world;
  a.rank = rank;
  a.col_offset = col_offset;
  for (int r = 0; r < world && world > 1; ++r) a.peer_out[r] = peer_y[r];
  return launch_cluster(bmax, a, cp.S, cp.C, s, dev, f32);
}

// fp32 thin linear on the cluster kernel (tf32 hi/lo split, M <= 64): layouts
// TMA can read with 32-element (128-byte) K blocks.
int f32_tc_possible(const void* x, long long ldx_m, long long ldx_k, const void* w, long long ldw_n,
                    long long ldw_k, const void* w_up, int M, int N, int K) {
  if (M > 64 || K < 32 || ldx_k != 1 || ldw_k != 1) return 0;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(x) || !al(w) || (w_up && !al(w_up))) return 0;
  if (M > 1 && (ldx_m < K || ((ldx_m * 4) & 15) != 0)) return 0;
  if (N > 1 && (ldw_n < K || ((ldw_n * 4) & 15) != 0)) return 0;
  return 1;
}

int thin_tc_possible(const void* x, long long ldx_m, long long ldx_k, const void* w, long long ldw_n,
                     long long ldw_k, const void* w_up, int M, int N, int K, int dtype) {
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return 0;
  if (ldx_k != 1 || ldw_k != 1) return 0;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!al(x) || !al(w) || (w_up && !al(w_up))) return 0;
  if (M > 1 && (ldx_m < K || ((ldx_m * 2) & 15) != 0)) return 0;
  if (N > 1 && (ldw_n < K || ((ldw_n * 2) & 15) != 0)) return 0;
  // the tensor-core kernel indexes (tile, k-block) iterations with 32-bit ints
  if (cdiv(M, pick_bmax_rows(M)) * cdiv(N, 64) * cdiv(K, 64) >= (1LL << 31)) return 0;
  return 1;
}

// ---------------------------------------------------------------- static scratch
// Scratch of simsd_thin_linear_noalloc: a fixed device array that exists on every
// GPU that loads this library, from module load until the process exits, so that
// entry point never allocates.  Its first 64 KiB hold the error word (offset 0)
// and the per-tile arrival counters (from offset 256; zero from module load, and
// every launch leaves them zero); the rest holds the split-K partial slots.  Its name is only a host-side handle: the device
// address comes from cudaGetSymbolAddress, once per device.
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;   // 8 MiB
constexpr size_t kNoAllocHeader = size_t(64) << 10;
constexpr size_t kNoAllocCounterOffset = 256;
constexpr long long kNoAllocCounters = (long long)((kNoAllocHeader - kNoAllocCounterOffset) / 4);
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];
void* g_noalloc_ptr[kMaxDev];

// Device address of g_noalloc_scratch on the current device `dev` (resolved on
// the first call there, with `dev` current; nullptr if the runtime refuses).
void* noalloc_scratch(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return nullptr;
    g_noalloc_ptr[dev] = ptr;
  }
  return g_noalloc_ptr[dev];
}

}  // namespace

// ======================================================================== API
extern "C" {

const char* simsd_version(void) { return "simsd_b200 0.1 (sm_100a)"; }

const char* simsd_status_string(int s) {
  switch (s) {
    case SIMSD_OK: return "ok";
    case SIMSD_ERR_SHAPE: return "bad shape";
    case SIMSD_ERR_DTYPE: return "bad dtype";
    case SIMSD_ERR_WORKSPACE: return "workspace missing or too small";
    case SIMSD_ERR_LAUNCH: return "CUDA launch failed";
    case SIMSD_ERR_ALIGN: return "pointer or stride not usable by this path";
    case SIMSD_ERR_DEVICE: return "no usable CUDA device";
    case SIMSD_ERR_UNSUPPORTED: return "outside this build's limits";
    case SIMSD_ERR_SCRATCH_LIMIT:
      return "request needs more scratch than simsd_thin_linear_noalloc's fixed static buffer";
  }
  return "unknown status";
}

int simsd_set_launch_flags(int flags) {
  return g_launch_flags.exchange(flags & (SIMSD_LAUNCH_PDL | SIMSD_LAUNCH_INKERNEL_REDUCE | SIMSD_LAUNCH_GROUPED_FIXUP |
                                         SIMSD_LAUNCH_MOE_SIZE_CLASSES));
}

int simsd_get_launch_flags(void) { return g_launch_flags.load(); }

int simsd_debug_set_trace(void* buf, size_t bytes) {
  std::lock_guard<std::mutex> lk(g_mu);
  g_trace = reinterpret_cast<unsigned long long*>(buf);
  g_trace_bytes = buf ? bytes : 0;
  g_trace_used = 0;
  return SIMSD_OK;
}

int simsd_debug_cluster_plan(int M, int N, int K, int silu, int* S, int* C, int* max_clusters_by_s) {
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  if (M < 1 || M > 64 || N < 1 || K < 1 || !S || !C) return SIMSD_ERR_SHAPE;
  const int bmax = pick_bmax_rows(M);
  const ClusterPlan cp = plan_cluster(bmax, silu ? cdiv(N, 64) : cdiv(N, 128), (int)cdiv(K, 64), dev);
  *S = cp.S;
  *C = cp.C;
  if (max_clusters_by_s)
    for (int s2 = 1; s2 <= TC_CL_MAX; ++s2) max_clusters_by_s[s2 - 1] = max_clusters(bmax, s2, dev);
  return SIMSD_OK;
}

int simsd_device_sm_count(void) {
  const int dev = current_device();
  return dev < 0 ? 0 : sm_count_of(dev);
}

size_t simsd_workspace_header_bytes(void) { return WS_COUNTER_BYTES; }

int simsd_workspace_init(void* ws, size_t bytes, void* stream) {
  if (ws == nullptr || bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  return cudaMemsetAsync(ws, 0, WS_COUNTER_BYTES, (cudaStream_t)stream) == cudaSuccess ? SIMSD_OK
                                                                                      : SIMSD_ERR_LAUNCH;
}

int simsd_workspace_error(const void* ws, void* stream, int* out) {
  if (ws == nullptr || out == nullptr) return SIMSD_ERR_WORKSPACE;
  int v = 0;
  if (cudaMemcpyAsync(&v, reinterpret_cast<const char*>(ws) + WS_ERR_OFFSET, sizeof(int), cudaMemcpyDeviceToHost,
                      (cudaStream_t)stream) != cudaSuccess)
    return SIMSD_ERR_LAUNCH;
  if (cudaStreamSynchronize((cudaStream_t)stream) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  *out = v;
  return SIMSD_OK;
}

size_t simsd_thin_linear_workspace_size(int M, int N, int K, int dtype, int epilogue, int split) {
  if (M < 1 || N < 1 || K < 1) return WS_COUNTER_BYTES;
  (void)dtype;
  const int dev = current_device();
  const int sms = dev < 0 ? 148 : sm_count_of(dev);
  return plan_thin(M, N, K, epilogue, split, sms).ws_bytes;
}

int simsd_thin_linear(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n, int64_t ldw_k,
                      const void* w_up, const void* bias, void* y, int64_t ldy_m, int M, int N, int K, int dtype,
                      int epilogue, int split, int path, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 1 || N < 1 || K < 1 || split < 0) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (epilogue != SIMSD_EPI_NONE && epilogue != SIMSD_EPI_SILU_MUL) return SIMSD_ERR_UNSUPPORTED;
  const bool silu = epilogue == SIMSD_EPI_SILU_MUL;
  if (silu && (w_up == nullptr || bias != nullptr)) return SIMSD_ERR_UNSUPPORTED;
  if (x == nullptr || w == nullptr || y == nullptr) return SIMSD_ERR_SHAPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  int* err = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + WS_ERR_OFFSET);

  if (dtype == SIMSD_F32 && path != SIMSD_PATH_SIMT && split == 0 && cluster_enabled() &&
      f32_tc_possible(x, ldx_m, ldx_k, w, ldw_n, ldw_k, w_up, M, N, K)) {
    // fp32, M <= 64: the same cluster kernel on tf32 hi/lo parts (three
    // products per K step, fp32 accumulate)
    const int rc = thin_cluster(x, ldx_m, w, ldw_n, w_up, bias, y, ldy_m, M, N, K, dtype, silu, err, nullptr, 0, 1,
                                0, s, dev);
    if (rc != SIMSD_ERR_UNSUPPORTED) return rc;
  }
  const bool tc_ok = thin_tc_possible(x, ldx_m, ldx_k, w, ldw_n, ldw_k, w_up, M, N, K, dtype) != 0;
  bool use_tc;
  if (path == SIMSD_PATH_TC) {
    if (!tc_ok) return SIMSD_ERR_ALIGN;
    use_tc = true;
  } else if (path == SIMSD_PATH_SIMT) {
    use_tc = false;
  } else {
    use_tc = tc_ok && K >= 64;
  }

  if (use_tc && M <= 64 && split == 0 && cluster_enabled()) {
    // M <= 64: split-K tiles reduced inside thread-block clusters
    const int rc = thin_cluster(x, ldx_m, w, ldw_n, w_up, bias, y, ldy_m, M, N, K, dtype, silu, err, nullptr, 0, 1,
                                0, s, dev);
    if (rc != SIMSD_ERR_UNSUPPORTED) return rc;
  }

  if (use_tc) {
    if (ensure_encode() != SIMSD_OK) return SIMSD_ERR_DEVICE;
    const ThinPlan pl = plan_thin(M, N, K, epilogue, split, sm_count_of(dev));
    if (workspace_bytes < pl.ws_bytes) return SIMSD_ERR_WORKSPACE;
    TcGemmArgs a;
    memset(&a, 0, sizeof(a));
    const long long lx = (M > 1) ? ldx_m : ((K * 2 + 15) / 16) * 8;
    const long long lw = (N > 1) ? ldw_n : ((K * 2 + 15) / 16) * 8;
    const uint64_t xd[2] = {(uint64_t)K, (uint64_t)M}, xs[1] = {(uint64_t)lx * 2};
    const uint64_t wd[2] = {(uint64_t)K, (uint64_t)N}, wsb[1] = {(uint64_t)lw * 2};
    int rc = encode_map(&a.tmB, x, dtype, 2, xd, xs, (uint32_t)pl.bmax);
    if (rc == SIMSD_OK) rc = encode_map(&a.tmA0, w, dtype, 2, wd, wsb, silu ? 64 : 128);
    if (rc == SIMSD_OK && silu) rc = encode_map(&a.tmA1, w_up, dtype, 2, wd, wsb, 64);
    if (rc != SIMSD_OK) return rc;
    a.out = y;
    a.ld_out = ldy_m;
    a.bias = bias;
    a.partials = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + WS_COUNTER_BYTES);
    a.tables = nullptr;
    a.counters = use_counters() && pl.tiles <= WS_MAX_COUNTERS ? reinterpret_cast<int*>(workspace) : nullptr;
    a.err = err;
    a.group_counts = nullptr;
    a.num_groups = 1;
    a.single_rows = M;
    a.kb = pl.kb;
    a.rows_out = N;
    a.row_tiles = pl.row_tiles;
    a.silu = silu ? 1 : 0;
    a.three_d = 0;
    a.is_bf16 = dtype == SIMSD_BF16 ? 1 : 0;
    int rc2 = launch_tc(pl.bmax, a, pl.grid, s, dev);
    if (rc2 != SIMSD_OK || a.counters != nullptr || !any_split_tile(pl.tiles, pl.kb, pl.grid)) return rc2;
    return launch_fixup(pl.bmax, fixup_args(a, pl.grid), s);
  }

  SimtGemmArgs a;
  memset(&a, 0, sizeof(a));
  a.a = x;
  a.w = w;
  a.w_up = w_up;
  a.bias = bias;
  a.out = y;
  a.group_counts = nullptr;
  a.err = err;
  a.lda_m = ldx_m;
  a.lda_k = ldx_k;
  a.ldw_n = ldw_n;
  a.ldw_k = ldw_k;
  a.ldw_g = 0;
  a.ld_out = ldy_m;
  a.rows = M;
  a.num_groups = 1;
  a.N = N;
  a.K = K;
  a.dtype = dtype;
  a.silu = silu ? 1 : 0;
  const long long gy = cdiv(M, SIMT_ROWS);
  if (gy > 65535) return SIMSD_ERR_UNSUPPORTED;
  dim3 grid((unsigned)cdiv(N, SIMT_WARPS), (unsigned)gy);
  return launch(simt_gemm_kernel, grid, dim3(SIMT_WARPS * 32), 0, s, a);
}

int simsd_thin_linear_noalloc(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n,
                              int64_t ldw_k, const void* w_up, const void* bias, void* y, int64_t ldy_m, int M,
                              int N, int K, int dtype, int epilogue, void* stream) {
  if (M < 1 || N < 1 || K < 1) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (epilogue != SIMSD_EPI_NONE && epilogue != SIMSD_EPI_SILU_MUL) return SIMSD_ERR_UNSUPPORTED;
  const bool silu = epilogue == SIMSD_EPI_SILU_MUL;
  if (silu && (w_up == nullptr || bias != nullptr)) return SIMSD_ERR_UNSUPPORTED;
  if (x == nullptr || w == nullptr || y == nullptr) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  char* scratch = reinterpret_cast<char*>(noalloc_scratch(dev));
  if (scratch == nullptr) return SIMSD_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  // the error word is zero from module load and after every
  // simsd_thin_linear_noalloc_error that finds it set; kernels only OR bits into
  // it, so it keeps any failure until the caller reads it
  int* err = reinterpret_cast<int*>(scratch);

  const bool tc_ok = thin_tc_possible(x, ldx_m, ldx_k, w, ldw_n, ldw_k, w_up, M, N, K, dtype) != 0;
  if (tc_ok && K >= 64) {
    if (ensure_encode() != SIMSD_OK) return SIMSD_ERR_DEVICE;
    const ThinPlan pl = plan_thin(M, N, K, epilogue, 0, sm_count_of(dev));
    const size_t part_bytes = (size_t)2 * pl.grid * pl.bmax * 128 * sizeof(float);
    if (part_bytes > kNoAllocScratchBytes - kNoAllocHeader) return SIMSD_ERR_SCRATCH_LIMIT;
    TcGemmArgs a;
    memset(&a, 0, sizeof(a));
    const long long lx = (M > 1) ? ldx_m : ((K * 2 + 15) / 16) * 8;
    const long long lw = (N > 1) ? ldw_n : ((K * 2 + 15) / 16) * 8;
    const uint64_t xd[2] = {(uint64_t)K, (uint64_t)M}, xs[1] = {(uint64_t)lx * 2};
    const uint64_t wd[2] = {(uint64_t)K, (uint64_t)N}, wsb[1] = {(uint64_t)lw * 2};
    int rc = encode_map(&a.tmB, x, dtype, 2, xd, xs, (uint32_t)pl.bmax);
    if (rc == SIMSD_OK) rc = encode_map(&a.tmA0, w, dtype, 2, wd, wsb, silu ? 64 : 128);
    if (rc == SIMSD_OK && silu) rc = encode_map(&a.tmA1, w_up, dtype, 2, wd, wsb, 64);
    if (rc != SIMSD_OK) return rc;
    a.out = y;
    a.ld_out = ldy_m;
    a.bias = bias;
    a.partials = reinterpret_cast<float*>(scratch + kNoAllocHeader);
    a.tables = nullptr;
    a.counters = use_counters() && pl.tiles <= kNoAllocCounters
                     ? reinterpret_cast<int*>(scratch + kNoAllocCounterOffset)
                     : nullptr;
    a.err = err;
    a.group_counts = nullptr;
    a.num_groups = 1;
    a.single_rows = M;
    a.kb = pl.kb;
    a.rows_out = N;
    a.row_tiles = pl.row_tiles;
    a.silu = silu ? 1 : 0;
    a.three_d = 0;
    a.is_bf16 = dtype == SIMSD_BF16 ? 1 : 0;
    rc = launch_tc(pl.bmax, a, pl.grid, s, dev);
    if (rc != SIMSD_OK || a.counters != nullptr || !any_split_tile(pl.tiles, pl.kb, pl.grid)) return rc;
    return launch_fixup(pl.bmax, fixup_args(a, pl.grid), s);
  }
  // layouts the tensor-core kernel cannot read need no scratch beyond the error word
  SimtGemmArgs a;
  memset(&a, 0, sizeof(a));
  a.a = x;
  a.w = w;
  a.w_up = w_up;
  a.bias = bias;
  a.out = y;
  a.err = err;
  a.lda_m = ldx_m;
  a.lda_k = ldx_k;
  a.ldw_n = ldw_n;
  a.ldw_k = ldw_k;
  a.ld_out = ldy_m;
  a.rows = M;
  a.num_groups = 1;
  a.N = N;
  a.K = K;
  a.dtype = dtype;
  a.silu = silu ? 1 : 0;
  const long long gy = cdiv(M, SIMT_ROWS);
  if (gy > 65535) return SIMSD_ERR_UNSUPPORTED;
  return launch(simt_gemm_kernel, dim3((unsigned)cdiv(N, SIMT_WARPS), (unsigned)gy), dim3(SIMT_WARPS * 32), 0, s, a);
}

int simsd_thin_linear_noalloc_error(void* stream, int* out) {
  if (out == nullptr) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  char* scratch = reinterpret_cast<char*>(noalloc_scratch(dev));
  if (scratch == nullptr) return SIMSD_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  int v = 0;
  if (cudaMemcpyAsync(&v, scratch, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  if (v != 0) {
    // a launch that gave up part-way may have left per-tile arrival counters
    // raised; zero the whole header (error word and counters) so the next call
    // starts from the state every completed launch leaves behind
    if (cudaMemsetAsync(scratch, 0, kNoAllocHeader, s) != cudaSuccess) return SIMSD_ERR_LAUNCH;
    if (cudaStreamSynchronize(s) != cudaSuccess) return SIMSD_ERR_LAUNCH;
  }
  *out = v;
  return SIMSD_OK;
}

// ---------------------------------------------------------------- MoE
int simsd_moe_route(const void* x, int64_t ldx, int x_dtype, const void* wr, int64_t ldw, int w_dtype,
                    const float* bias, int T, int H, int E, int k, int renorm, float scale, int64_t* topk_ids,
                    float* topk_weight, float* logits, void* stream) {
  return simsd_moe_route_ex(x, ldx, x_dtype, wr, ldw, w_dtype, bias, T, H, E, k, renorm, scale, topk_ids, topk_weight,
                            k, -1, logits, stream);
}

int simsd_moe_route_ex(const void* x, int64_t ldx, int x_dtype, const void* wr, int64_t ldw, int w_dtype,
                       const float* bias, int T, int H, int E, int k, int renorm, float scale, int64_t* topk_ids,
                       float* topk_weight, int64_t ld_topk, int extra_id, float* logits, void* stream) {
  if (T < 0 || H < 1 || E < 1 || E > 1024 || k < 1 || k > 32 || k > E) return SIMSD_ERR_SHAPE;
  if (ld_topk < k + (extra_id >= 0 ? 1 : 0) || ld_topk > (1 << 20) || extra_id > 1024) return SIMSD_ERR_SHAPE;
  if (x_dtype < 0 || x_dtype > 2 || w_dtype < 0 || w_dtype > 2) return SIMSD_ERR_DTYPE;
  if (T == 0) return SIMSD_OK;
  if (!x || !wr || !topk_ids || !topk_weight) return SIMSD_ERR_SHAPE;
  RouteArgs a;
  a.x = x;
  a.w = wr;
  a.bias = bias;
  a.topk_ids = reinterpret_cast<long long*>(topk_ids);
  a.topk_weight = topk_weight;
  a.logits = logits;
  a.ldx = ldx;
  a.ldw = ldw;
  a.T = T;
  a.H = H;
  a.E = E;
  a.k = k;
  a.x_dtype = x_dtype;
  a.w_dtype = w_dtype;
  a.renorm = renorm;
  a.scale = scale;
  a.ldo = (int)ld_topk;
  a.extra_id = extra_id;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool fast = (x_dtype == SIMSD_BF16 || x_dtype == SIMSD_F16) && H % 8 == 0 && ldx % 8 == 0 && al16(x) &&
                    al16(wr) && ((w_dtype != SIMSD_F32 && ldw % 8 == 0) || (w_dtype == SIMSD_F32 && ldw % 4 == 0));
  if (fast) {
    const int sms = sm_count_of(dev) > 0 ? sm_count_of(dev) : 148;
    // tokens per block: 16 from 16 per SM, else 8 (measured on the MoE layer
    // of H = 2048, E = 256: 4-token blocks were 3-4 us slower at T = 16..256
    // even with the experts split over blocks; 16-token blocks slower at
    // T = 1024).  SIMSD_ROUTE_TT (4, 8 or 16) pins it.
    static const int tt_pin = env_choice("SIMSD_ROUTE_TT", {0, 4, 8, 16}, 0);
    int tt = tt_pin > 0 ? tt_pin : (T >= 16 * sms ? 16 : 8);
    auto smem_for = [&](int t) { return (size_t)t * H * 4 + (size_t)2 * t * E * sizeof(float); };
    while (tt > 4 && smem_for(tt) > 200 * 1024) tt >>= 1;
    if (smem_for(tt) <= 200 * 1024) {
      size_t smem = smem_for(tt);
      // few token blocks: split the experts over blocks as well (logits to
      // `logits`, then route_topk_kernel) so the router uses more SMs
      const long long bx = cdiv(T, tt);
      int ny = 1;
      if (logits != nullptr && bx * 2 <= sms) ny = (int)std::min<long long>(16, sms / bx);
      // with the experts split, a block's router rows are staged in shared
      // memory when they fit (4-token blocks only)
      const int ee = 32 / tt;
      const long long per = ((E + ny - 1) / ny + ee - 1) / ee * ee;
      const size_t wbytes = (size_t)per * H * (w_dtype == SIMSD_F32 ? 4 : 2);
      const bool wsm = ny > 1 && tt == 4 && smem + wbytes <= 200 * 1024;
      if (wsm) smem += wbytes;
      const dim3 grid((unsigned)bx, (unsigned)ny), block(ROUTE_FAST_WARPS * 32);
      cudaStream_t st = (cudaStream_t)stream;
      auto go = [&](auto kern) -> int {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
          return SIMSD_ERR_LAUNCH;
        int rc = launch(kern, grid, block, smem, st, a);
        if (rc != SIMSD_OK || ny == 1) return rc;
        const size_t tsmem = (size_t)2 * ROUTE_WARPS * E * sizeof(float);
        if (cudaFuncSetAttribute(route_topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tsmem) !=
            cudaSuccess)
          return SIMSD_ERR_LAUNCH;
        return launch(route_topk_kernel, dim3((unsigned)cdiv(T, ROUTE_WARPS)), dim3(ROUTE_WARPS * 32), tsmem, st, a);
      };
      auto by_w = [&](auto xdt) -> int {
        constexpr int X = decltype(xdt)::value;
        if (w_dtype == SIMSD_F32) {
          if (tt == 16) return go(route_fast_kernel<16, X, 2, false>);
          if (tt == 8) return go(route_fast_kernel<8, X, 2, false>);
          return wsm ? go(route_fast_kernel<4, X, 2, true>) : go(route_fast_kernel<4, X, 2, false>);
        }
        if (w_dtype == SIMSD_F16) {
          if (tt == 16) return go(route_fast_kernel<16, X, 1, false>);
          if (tt == 8) return go(route_fast_kernel<8, X, 1, false>);
          return wsm ? go(route_fast_kernel<4, X, 1, true>) : go(route_fast_kernel<4, X, 1, false>);
        }
        if (tt == 16) return go(route_fast_kernel<16, X, 0, false>);
        if (tt == 8) return go(route_fast_kernel<8, X, 0, false>);
        return wsm ? go(route_fast_kernel<4, X, 0, true>) : go(route_fast_kernel<4, X, 0, false>);
      };
      if (x_dtype == SIMSD_F16) return by_w(std::integral_constant<int, 1>{});
      return by_w(std::integral_constant<int, 0>{});
    }
  }
  const int smem = 2 * ROUTE_TOK * E * (int)sizeof(float);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_smem_attr[dev][38]) {
      if (cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * ROUTE_TOK * 1024 * 4) !=
          cudaSuccess)
        return SIMSD_ERR_LAUNCH;
      g_smem_attr[dev][38] = true;
    }
  }
  return launch(route_kernel, dim3((unsigned)cdiv(T, ROUTE_TOK)), dim3(ROUTE_WARPS * 32), smem,
                (cudaStream_t)stream, a);
}

static int launch_align(const int64_t* ids, int S, int E, int32_t* counts, int32_t* offsets, int32_t* sorted,
                        int32_t* s2r, int block_m, int num_tiles, int32_t* slots_padded, int32_t* tile_expert,
                        int* err, cudaStream_t s, int dev) {
  AlignArgs a;
  a.ids = reinterpret_cast<const long long*>(ids);
  a.counts = counts;
  a.offsets = offsets;
  a.sorted_slots = sorted;
  a.slot_to_row = s2r;
  a.slots_padded = slots_padded;
  a.tile_expert = tile_expert;
  a.err = err;
  a.S = S;
  a.E = E;
  a.block_m = block_m;
  a.num_tiles = num_tiles;
  int smem = (32 * E + 2 * (E + 1)) * (int)sizeof(int);
  a.ids_in_smem = (smem + (size_t)S * sizeof(int) <= 200 * 1024) ? 1 : 0;
  if (a.ids_in_smem) smem += S * (int)sizeof(int);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_smem_attr[dev][39]) {
      if (cudaFuncSetAttribute(align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) !=
          cudaSuccess)
        return SIMSD_ERR_LAUNCH;
      g_smem_attr[dev][39] = true;
    }
  }
  return launch(align_kernel, dim3(1), dim3(ALIGN_THREADS), smem, s, a);
}

int simsd_moe_align(const int64_t* topk_ids, int S, int E, int32_t* counts, int32_t* offsets, int32_t* sorted_slots,
                    int32_t* slot_to_row, int block_m, int num_tiles, int32_t* slots_padded, int32_t* tile_expert,
                    int* err_word, void* stream) {
  if (S < 0 || E < 1 || E > 1024) return SIMSD_ERR_SHAPE;
  if ((slots_padded == nullptr) != (tile_expert == nullptr)) return SIMSD_ERR_SHAPE;
  if (slots_padded && (block_m < 1 || num_tiles < 0)) return SIMSD_ERR_SHAPE;
  if (!counts || !offsets || (S > 0 && (!topk_ids || !sorted_slots || !slot_to_row))) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  if (err_word == nullptr) return SIMSD_ERR_WORKSPACE;
  return launch_align(topk_ids, S, E, counts, offsets, sorted_slots, slot_to_row, block_m, num_tiles, slots_padded,
                      tile_expert, err_word, (cudaStream_t)stream, dev);
}

namespace {
struct MoePlan {
  bool tc;
  int bmax, bmax_big, grid;
  size_t off_counts, off_offsets, off_sorted, off_s2r, off_xs, off_h, off_ys, off_tables, off_part, total;
  long long max_chunks;
};

MoePlan plan_moe(int T, int k, int E, int H, int I, int dtype, int sms, bool tc) {
  MoePlan p{};
  const long long S = (long long)T * k;
  const int es = esize(dtype);
  p.tc = tc;
  // Activation rows per tile: enough for a busy expert (mean + 4 sd of a
  // Poisson count, plus slack) so it is rarely split into chunks that would each
  // re-read its weights.
  const double avg = E > 0 ? (double)S / E : (double)S;
  const double want = avg + 4.0 * std::sqrt(avg) + 8.0;
  p.bmax = want <= 16 ? 16 : want <= 32 ? 32 : want <= 64 ? 64 : want <= 128 ? 128 : 256;
  // SIMSD_MOE_BMAX (16, 32, 64, 128, 256) overrides the choice (measurement knob)
  p.bmax = env_choice("SIMSD_MOE_BMAX", {16, 32, 64, 128, 256}, p.bmax);
  // Skewed routing (SIMSD_LAUNCH_MOE_SIZE_CLASSES): groups with more rows than
  // bmax go to a second launch of each grouped GEMM with 256-row tiles, the
  // device choosing the class of every group from its count.  Off by default:
  // with near-uniform routing the second class holds little work and its
  // launches and 256-row split-K partials cost more than the chunks they save.
  const bool two_class = (g_launch_flags.load(std::memory_order_relaxed) & SIMSD_LAUNCH_MOE_SIZE_CLASSES) != 0;
  p.bmax_big = (tc && two_class && p.bmax < 256 && T > p.bmax) ? 256 : 0;
  p.grid = std::max(1, std::min(sms > 0 ? sms : 148, TC_MAX_GRID));
  size_t o = WS_COUNTER_BYTES;
  p.off_counts = o; o = align256(o + (size_t)E * 4);
  p.off_offsets = o; o = align256(o + (size_t)(E + 1) * 4);
  p.off_sorted = o; o = align256(o + (size_t)S * 4);
  p.off_s2r = o; o = align256(o + (size_t)S * 4);
  p.off_xs = o; o = align256(o + (size_t)S * H * es);
  p.off_h = o; o = align256(o + (size_t)S * I * es);
  p.off_ys = o; o = align256(o + (size_t)S * H * es);
  p.off_tables = o; o = align256(o + (size_t)TC_TABLE_INTS * 4);
  p.off_part = o;
  if (tc) o = align256(o + (size_t)2 * p.grid * std::max(p.bmax, p.bmax_big) * 128 * sizeof(float));
  p.total = o;
  p.max_chunks = std::min<long long>(E, S) + S / p.bmax + 1;
  return p;
}
}  // namespace

size_t simsd_moe_workspace_size(int T, int k, int E, int H, int I, int dtype) {
  if (T < 0 || k < 1 || E < 1 || H < 1 || I < 1) return WS_COUNTER_BYTES;
  const int dev = current_device();
  const int sms = dev < 0 ? 148 : sm_count_of(dev);
  return plan_moe(T, k, E, H, I, dtype, sms, dtype != SIMSD_F32).total;
}

static int moe_dispatch_impl(const void* x, int64_t ldx, const int64_t* topk_ids, const float* topk_weight,
                             const void* w_gate, const void* w_up, int64_t ldg_e, int64_t ldg_i, const void* w_down,
                             int64_t ldd_e, int64_t ldd_h, void* out, int64_t ld_out, const void* add,
                             int64_t ld_add, int T, int k, int E, int H, int I, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream, int shared_last);

int simsd_moe_dispatch(const void* x, int64_t ldx, const int64_t* topk_ids, const float* topk_weight,
                       const void* w_gate, const void* w_up, int64_t ldg_e, int64_t ldg_i, const void* w_down,
                       int64_t ldd_e, int64_t ldd_h, void* out, int64_t ld_out, const void* add, int64_t ld_add,
                       int T, int k, int E, int H, int I, int dtype, void* workspace, size_t workspace_bytes,
                       void* stream) {
  return moe_dispatch_impl(x, ldx, topk_ids, topk_weight, w_gate, w_up, ldg_e, ldg_i, w_down, ldd_e, ldd_h, out,
                           ld_out, add, ld_add, T, k, E, H, I, dtype, workspace, workspace_bytes, stream, 0);
}

int simsd_moe_dispatch_shared_last(const void* x, int64_t ldx, const int64_t* topk_ids, const float* topk_weight,
                                   const void* w_gate, const void* w_up, int64_t ldg_e, int64_t ldg_i,
                                   const void* w_down, int64_t ldd_e, int64_t ldd_h, void* out, int64_t ld_out,
                                   int T, int k, int E, int H, int I, int dtype, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  if (k < 2) return SIMSD_ERR_SHAPE;
  return moe_dispatch_impl(x, ldx, topk_ids, topk_weight, w_gate, w_up, ldg_e, ldg_i, w_down, ldd_e, ldd_h, out,
                           ld_out, nullptr, 0, T, k, E, H, I, dtype, workspace, workspace_bytes, stream, 1);
}

// The dispatch; shared_last: column k-1 of every row is an always-on (shared)
// expert whose output is added unweighted after the routed sum is rounded.
static int moe_dispatch_impl(const void* x, int64_t ldx, const int64_t* topk_ids, const float* topk_weight,
                             const void* w_gate, const void* w_up, int64_t ldg_e, int64_t ldg_i, const void* w_down,
                             int64_t ldd_e, int64_t ldd_h, void* out, int64_t ld_out, const void* add,
                             int64_t ld_add, int T, int k, int E, int H, int I, int dtype, void* workspace,
                             size_t workspace_bytes, void* stream, int shared_last) {
  if (T < 0 || k < 1 || E < 1 || E > 1024 || H < 1 || I < 1) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  if (T == 0) return SIMSD_OK;
  if (!x || !topk_ids || !topk_weight || !w_gate || !w_up || !w_down || !out) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  const int es = esize(dtype);
  const long long S = (long long)T * k;
  if (S > (1LL << 30)) return SIMSD_ERR_UNSUPPORTED;

  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  bool tc = dtype != SIMSD_F32 && H >= 64 && I >= 64 && (H % 8) == 0 && (I % 8) == 0 && al(w_gate) && al(w_up) &&
            al(w_down) && (ldg_e % 8) == 0 && (ldg_i % 8) == 0 && (ldd_e % 8) == 0 && (ldd_h % 8) == 0 &&
            ldg_i >= H && ldd_h >= I;
  {
    // the grouped GEMMs index (tile, k-block) iterations with 32-bit ints
    const long long chunks = std::min<long long>(E, S) + S / 16 + 1;
    if (chunks * std::max(cdiv(I, 64) * cdiv(H, 64), cdiv(H, 128) * cdiv(I, 64)) >= (1LL << 31)) tc = false;
  }
  const MoePlan plan = plan_moe(T, k, E, H, I, dtype, sm_count_of(dev), tc);
  if (workspace_bytes < plan.total) return SIMSD_ERR_WORKSPACE;

  char* ws = reinterpret_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws + WS_ERR_OFFSET);
  int32_t* counts = reinterpret_cast<int32_t*>(ws + plan.off_counts);
  int32_t* offsets = reinterpret_cast<int32_t*>(ws + plan.off_offsets);
  int32_t* sorted = reinterpret_cast<int32_t*>(ws + plan.off_sorted);
  int32_t* s2r = reinterpret_cast<int32_t*>(ws + plan.off_s2r);
  void* xs = ws + plan.off_xs;
  void* hbuf = ws + plan.off_h;
  void* ys = ws + plan.off_ys;

  int rc = launch_align(topk_ids, (int)S, E, counts, offsets, sorted, s2r, 16, 0, nullptr, nullptr, err, s, dev);
  if (rc != SIMSD_OK) return rc;
  if (prefer_shared(gather_rows_kernel, dev, 5) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  rc = launch(gather_rows_kernel, dim3((unsigned)S), dim3(256), 0, s, x, (long long)ldx, (const int*)sorted, xs,
              (long long)H, (int)S, k, H, es);
  if (rc != SIMSD_OK) return rc;

  if (plan.tc) {
    if (ensure_encode() != SIMSD_OK) return SIMSD_ERR_DEVICE;
    // One grouped GEMM over the groups of class (lo, hi] rows with bm-row tiles:
    // gate/up (out[row, i] = silu(xs[row] . w_gate[e, i]) * (xs[row] . w_up[e, i]))
    // or down (ys[row, h] = hbuf[row] . w_down[e, h]).
    auto grouped = [&](bool up, int bm, int lo, int hi) -> int {
      TcGemmArgs a;
      memset(&a, 0, sizeof(a));
      int r;
      if (up) {
        const uint64_t gd[3] = {(uint64_t)H, (uint64_t)I, (uint64_t)E};
        const uint64_t gs[2] = {(uint64_t)ldg_i * es, (uint64_t)ldg_e * es};
        const uint64_t bd[2] = {(uint64_t)H, (uint64_t)S};
        const uint64_t bs[1] = {(uint64_t)H * es};
        r = encode_map(&a.tmA0, w_gate, dtype, 3, gd, gs, 64);
        if (r == SIMSD_OK) r = encode_map(&a.tmA1, w_up, dtype, 3, gd, gs, 64);
        if (r == SIMSD_OK) r = encode_map(&a.tmB, xs, dtype, 2, bd, bs, (uint32_t)bm);
        a.out = hbuf;
        a.ld_out = I;
        a.kb = (int)cdiv(H, 64);
        a.rows_out = I;
        a.row_tiles = (int)cdiv(I, 64);
        a.silu = 1;
      } else {
        const uint64_t dd[3] = {(uint64_t)I, (uint64_t)H, (uint64_t)E};
        const uint64_t ds[2] = {(uint64_t)ldd_h * es, (uint64_t)ldd_e * es};
        const uint64_t bd[2] = {(uint64_t)I, (uint64_t)S};
        const uint64_t bs[1] = {(uint64_t)I * es};
        r = encode_map(&a.tmA0, w_down, dtype, 3, dd, ds, 128);
        if (r == SIMSD_OK) r = encode_map(&a.tmB, hbuf, dtype, 2, bd, bs, (uint32_t)bm);
        a.out = ys;
        a.ld_out = H;
        a.kb = (int)cdiv(I, 64);
        a.rows_out = H;
        a.row_tiles = (int)cdiv(H, 128);
        a.silu = 0;
      }
      if (r != SIMSD_OK) return r;
      a.partials = reinterpret_cast<float*>(ws + plan.off_part);
      a.tables = reinterpret_cast<int*>(ws + plan.off_tables);
      const long long max_chunks = std::min<long long>(E, S) + S / bm + 1;
      a.counters = use_counters_grouped() && max_chunks * a.row_tiles <= WS_MAX_COUNTERS ? reinterpret_cast<int*>(ws)
                                                                                         : nullptr;
      a.err = err;
      a.group_counts = counts;
      a.num_groups = E;
      a.cls_lo = lo;
      a.cls_hi = hi;
      a.three_d = 1;
      a.is_bf16 = dtype == SIMSD_BF16 ? 1 : 0;
      // a grouped GEMM with at least two tiles per CTA splits no tile
      // (tc_whole_tiles); with the class filter the chunk count is only known
      // on the device, so the fixup kernel runs unless the in-kernel reduction does
      const long long min_chunks = hi == 0 && lo == 0 ? std::max<long long>(1, cdiv(S, bm)) : 0;
      r = launch_tc(bm, a, plan.grid, s, dev);
      if (r == SIMSD_OK && a.counters == nullptr &&
          !tc_whole_tiles(true, (int)std::min<long long>(min_chunks * a.row_tiles, 1 << 30), plan.grid))
        r = launch_fixup(bm, fixup_args(a, plan.grid), s);
      return r;
    };
    const int bs_hi = plan.bmax_big > 0 ? plan.bmax : 0;   // small tiles take groups of <= bmax rows
    rc = grouped(true, plan.bmax, 0, bs_hi);
    if (rc == SIMSD_OK && plan.bmax_big > 0) rc = grouped(true, plan.bmax_big, plan.bmax, 0);
    if (rc == SIMSD_OK) rc = grouped(false, plan.bmax, 0, bs_hi);
    if (rc == SIMSD_OK && plan.bmax_big > 0) rc = grouped(false, plan.bmax_big, plan.bmax, 0);
    if (rc != SIMSD_OK) return rc;
  } else {
    const long long max_chunks = std::min<long long>(E, S) + S / SIMT_ROWS + 1;
    if (max_chunks > 65535) return SIMSD_ERR_UNSUPPORTED;
    SimtGemmArgs a;
    memset(&a, 0, sizeof(a));
    a.a = xs;
    a.w = w_gate;
    a.w_up = w_up;
    a.out = hbuf;
    a.group_counts = counts;
    a.err = err;
    a.lda_m = H;
    a.lda_k = 1;
    a.ldw_n = ldg_i;
    a.ldw_k = 1;
    a.ldw_g = ldg_e;
    a.ld_out = I;
    a.num_groups = E;
    a.N = I;
    a.K = H;
    a.dtype = dtype;
    a.silu = 1;
    rc = launch(simt_gemm_kernel, dim3((unsigned)cdiv(I, SIMT_WARPS), (unsigned)max_chunks), dim3(SIMT_WARPS * 32),
                0, s, a);
    if (rc != SIMSD_OK) return rc;
    SimtGemmArgs d = a;
    d.a = hbuf;
    d.w = w_down;
    d.w_up = nullptr;
    d.out = ys;
    d.lda_m = I;
    d.ldw_n = ldd_h;
    d.ldw_g = ldd_e;
    d.ld_out = H;
    d.N = H;
    d.K = I;
    d.silu = 0;
    rc = launch(simt_gemm_kernel, dim3((unsigned)cdiv(H, SIMT_WARPS), (unsigned)max_chunks), dim3(SIMT_WARPS * 32),
                0, s, d);
    if (rc != SIMSD_OK) return rc;
  }
  const bool vec = dtype != SIMSD_F32 && H % 8 == 0 && ld_out % 8 == 0 && al(out) && (add == nullptr || (al(add) && ld_add % 8 == 0)) && k <= 32;
  if (vec) {
    if (prefer_shared(combine_vec_kernel, dev, 6) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
    return launch(combine_vec_kernel, dim3((unsigned)T), dim3(128), 0, s, (const void*)ys, (long long)H, (const int*)s2r,
                  topk_weight, out, (long long)ld_out, add, (long long)ld_add, T, k, H, dtype, shared_last);
  }
  if (prefer_shared(combine_kernel, dev, 7) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  return launch(combine_kernel, dim3((unsigned)T), dim3(256), 0, s, (const void*)ys, (long long)H, (const int*)s2r,
                topk_weight, out, (long long)ld_out, add, (long long)ld_add, T, k, H, dtype, shared_last);
}

int simsd_moe_ep_plan(const int64_t* topk_ids, int S, int E, int world, int capacity, int32_t* send_slot,
                      int32_t* send_expert, int32_t* slot_pos, int32_t* counts, int* err_word, void* stream) {
  if (S < 0 || E < 1 || world < 1 || world > EP_MAX_WORLD || E % world != 0 || capacity < 0) return SIMSD_ERR_SHAPE;
  if (S > 0 && (topk_ids == nullptr || slot_pos == nullptr)) return SIMSD_ERR_SHAPE;
  if (capacity > 0 && (send_slot == nullptr || send_expert == nullptr)) return SIMSD_ERR_SHAPE;
  if (counts == nullptr || err_word == nullptr) return SIMSD_ERR_SHAPE;
  if ((long long)world * capacity >= (1LL << 31)) return SIMSD_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  if (prefer_shared(ep_plan_kernel, dev, 8) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  EpPlanArgs a;
  a.ids = reinterpret_cast<const long long*>(topk_ids);
  a.send_slot = send_slot;
  a.send_expert = send_expert;
  a.slot_pos = slot_pos;
  a.counts = counts;
  a.err = err_word;
  a.S = S;
  a.E = E;
  a.world = world;
  a.cap = capacity;
  return launch(ep_plan_kernel, dim3(1), dim3(EP_THREADS), 0, (cudaStream_t)stream, a);
}

int simsd_moe_gather_rows(const void* x, int64_t ldx, const int32_t* slots, int R, int k, int H, int dtype,
                          void* out, int64_t ld_out, void* stream) {
  if (R < 0 || k < 1 || H < 1 || ldx < H || ld_out < H) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (R == 0) return SIMSD_OK;
  if (x == nullptr || slots == nullptr || out == nullptr) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  if (prefer_shared(gather_rows_kernel, dev, 5) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  return launch(gather_rows_kernel, dim3((unsigned)R), dim3(256), 0, (cudaStream_t)stream, x, (long long)ldx,
                (const int*)slots, out, (long long)ld_out, R, k, H, esize(dtype));
}

namespace {
int ep_exchange(const void* src, int64_t ld_src, const int32_t* sel, const int32_t* expert, int k, int H,
                int capacity, int rank, int world, void* const* rows, void* const* ids, int dtype, int mode,
                void* stream) {
  if (H < 1 || capacity < 1 || ld_src < H || world < 1 || world > EP_XCH_MAX_WORLD || rank < 0 || rank >= world ||
      (mode == 0 && k < 1))
    return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (src == nullptr || sel == nullptr || rows == nullptr || (mode == 0 && (expert == nullptr || ids == nullptr)))
    return SIMSD_ERR_SHAPE;
  const long long entries = (long long)world * capacity;
  if (entries >= (1LL << 31)) return SIMSD_ERR_SHAPE;
  const long long rb = (long long)H * esize(dtype);
  auto al = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!al(src) || (rb & 15) != 0 || ((ld_src * esize(dtype)) & 15) != 0 || rb >= (1LL << 31)) return SIMSD_ERR_ALIGN;
  EpExchangeArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    if (rows[r] == nullptr || (mode == 0 && ids[r] == nullptr)) return SIMSD_ERR_SHAPE;
    if (!al(rows[r])) return SIMSD_ERR_ALIGN;
    a.rows[r] = rows[r];
    if (mode == 0) a.ids[r] = static_cast<int*>(ids[r]);
  }
  if (current_device() < 0) return SIMSD_ERR_DEVICE;
  a.src = src;
  a.src_row_bytes = ld_src * esize(dtype);
  a.sel = sel;
  a.expert = expert;
  a.entries = (int)entries;
  a.cap = capacity;
  a.k = k;
  a.rank = rank;
  a.mode = mode;
  a.row_bytes = (int)rb;
  return launch(ep_exchange_kernel, dim3((unsigned)((entries + 7) / 8)), dim3(256), 0, (cudaStream_t)stream, a);
}
}  // namespace

int simsd_moe_ep_send(const void* x, int64_t ldx, const int32_t* send_slot, const int32_t* send_expert, int k, int H,
                      int capacity, int rank, int world, void* const* peer_rows, void* const* peer_ids, int dtype,
                      void* stream) {
  return ep_exchange(x, ldx, send_slot, send_expert, k, H, capacity, rank, world, peer_rows, peer_ids, dtype, 0,
                     stream);
}

int simsd_moe_ep_return(const void* y, int64_t ldy, const int32_t* recv_expert, int H, int capacity, int rank,
                        int world, void* const* peer_back, int dtype, void* stream) {
  return ep_exchange(y, ldy, recv_expert, nullptr, 1, H, capacity, rank, world, peer_back, nullptr, dtype, 1,
                     stream);
}

int simsd_moe_combine(const void* ys, int64_t ldys, const int32_t* slot_row, const float* topk_weight, void* out,
                      int64_t ld_out, const void* add, int64_t ld_add, int T, int k, int H, int dtype, void* stream) {
  if (T < 0 || k < 1 || H < 1 || ldys < H || ld_out < H || (add && ld_add < H)) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16 && dtype != SIMSD_F32) return SIMSD_ERR_DTYPE;
  if (T == 0) return SIMSD_OK;
  if (ys == nullptr || slot_row == nullptr || topk_weight == nullptr || out == nullptr) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  cudaStream_t s = (cudaStream_t)stream;
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const bool vec = dtype != SIMSD_F32 && H % 8 == 0 && ld_out % 8 == 0 && ldys % 8 == 0 && al(out) && al(ys) &&
                   (add == nullptr || (al(add) && ld_add % 8 == 0)) && k <= 32;
  if (vec) {
    if (prefer_shared(combine_vec_kernel, dev, 6) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
    return launch(combine_vec_kernel, dim3((unsigned)T), dim3(128), 0, s, ys, (long long)ldys, (const int*)slot_row,
                  topk_weight, out, (long long)ld_out, add, (long long)ld_add, T, k, H, dtype, 0);
  }
  if (prefer_shared(combine_kernel, dev, 7) != SIMSD_OK) return SIMSD_ERR_LAUNCH;
  return launch(combine_kernel, dim3((unsigned)T), dim3(256), 0, s, ys, (long long)ldys, (const int*)slot_row,
                topk_weight, out, (long long)ld_out, add, (long long)ld_add, T, k, H, dtype, 0);
}

int simsd_ipc_alloc(size_t bytes, void** dev_ptr) {
  if (dev_ptr == nullptr || bytes == 0) return SIMSD_ERR_SHAPE;
  void* p = nullptr;
  if (cudaMalloc(&p, bytes) != cudaSuccess) return SIMSD_ERR_DEVICE;
  if (cudaMemset(p, 0, bytes) != cudaSuccess) {
    cudaFree(p);
    return SIMSD_ERR_DEVICE;
  }
  *dev_ptr = p;
  return SIMSD_OK;
}

int simsd_ipc_free(void* dev_ptr) { return cudaFree(dev_ptr) == cudaSuccess ? SIMSD_OK : SIMSD_ERR_DEVICE; }

int simsd_ipc_handle(const void* dev_ptr, void* handle) {
  static_assert(sizeof(cudaIpcMemHandle_t) <= SIMSD_IPC_HANDLE_BYTES, "handle size");
  if (dev_ptr == nullptr || handle == nullptr) return SIMSD_ERR_SHAPE;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)) != cudaSuccess) return SIMSD_ERR_DEVICE;
  memset(handle, 0, SIMSD_IPC_HANDLE_BYTES);
  memcpy(handle, &h, sizeof(h));
  return SIMSD_OK;
}

int simsd_ipc_open(const void* handle, void** dev_ptr) {
  if (handle == nullptr || dev_ptr == nullptr) return SIMSD_ERR_SHAPE;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return SIMSD_ERR_DEVICE;
  *dev_ptr = p;
  return SIMSD_OK;
}

int simsd_ipc_close(void* dev_ptr) {
  return cudaIpcCloseMemHandle(dev_ptr) == cudaSuccess ? SIMSD_OK : SIMSD_ERR_DEVICE;
}

int simsd_thin_linear_allgather(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n,
                                int64_t ldw_k, const void* w_up, const void* bias, void* const* peer_y, int64_t ldy,
                                int col_offset, int M, int N, int K, int dtype, int epilogue, int rank, int world,
                                int plan_n, void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 1 || N < 1 || K < 1 || col_offset < 0 || plan_n < 0) return SIMSD_ERR_SHAPE;
  if (world < 2 || world > TC_AG_MAX_WORLD || rank < 0 || rank >= world) return SIMSD_ERR_UNSUPPORTED;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return SIMSD_ERR_UNSUPPORTED;
  if (epilogue != SIMSD_EPI_NONE && epilogue != SIMSD_EPI_SILU_MUL) return SIMSD_ERR_UNSUPPORTED;
  const bool silu = epilogue == SIMSD_EPI_SILU_MUL;
  if (silu && (w_up == nullptr || bias != nullptr)) return SIMSD_ERR_UNSUPPORTED;
  if (x == nullptr || w == nullptr || peer_y == nullptr) return SIMSD_ERR_SHAPE;
  for (int r = 0; r < world; ++r)
    if (peer_y[r] == nullptr) return SIMSD_ERR_SHAPE;
  if (ldy < (long long)col_offset + N) return SIMSD_ERR_SHAPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  if (M > 64 || K < 64 || !cluster_enabled() ||
      !thin_tc_possible(x, ldx_m, ldx_k, w, ldw_n, ldw_k, w_up, M, N, K, dtype))
    return SIMSD_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  int* err = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + WS_ERR_OFFSET);
  return thin_cluster(x, ldx_m, w, ldw_n, w_up, bias, peer_y[rank], ldy, M, N, K, dtype, silu, err, peer_y,
                      col_offset, world, rank, (cudaStream_t)stream, dev, nullptr, nullptr, nullptr, nullptr, plan_n);
}

int simsd_allgather_wait(void* const* peer_signal, int rank, int world, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (peer_signal == nullptr || world < 2 || world > TC_AG_MAX_WORLD || rank < 0 || rank >= world)
    return SIMSD_ERR_SHAPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  if (current_device() < 0) return SIMSD_ERR_DEVICE;
  AgSyncArgs a;
  memset(&a, 0, sizeof(a));
  for (int r = 0; r < world; ++r) {
    if (peer_signal[r] == nullptr) return SIMSD_ERR_SHAPE;
    a.sig[r] = static_cast<int*>(peer_signal[r]);
  }
  a.world = world;
  a.rank = rank;
  a.err = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + WS_ERR_OFFSET);
  return launch(ag_sync_kernel, dim3(1), dim3(32), 0, (cudaStream_t)stream, a);
}

int simsd_thin_linear_argmax(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n,
                             int64_t ldw_k, const void* bias, int64_t* idx, int M, int N, int K, int dtype,
                             void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 1 || N < 1 || K < 1) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return SIMSD_ERR_UNSUPPORTED;
  if (x == nullptr || w == nullptr || idx == nullptr) return SIMSD_ERR_SHAPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  if (M > 64 || K < 64 || !cluster_enabled() ||
      !thin_tc_possible(x, ldx_m, ldx_k, w, ldw_n, ldw_k, nullptr, M, N, K, dtype))
    return SIMSD_ERR_UNSUPPORTED;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  char* ws = reinterpret_cast<char*>(workspace);
  int* err = reinterpret_cast<int*>(ws + WS_ERR_OFFSET);
  auto* keys = reinterpret_cast<unsigned long long*>(ws + WS_ARGMAX_OFFSET);
  int* count = reinterpret_cast<int*>(ws + WS_ARGMAX_OFFSET + 64 * 8);
  return thin_cluster(x, ldx_m, w, ldw_n, nullptr, bias, nullptr, 0, M, N, K, dtype, false, err, nullptr, 0, 1, 0,
                      (cudaStream_t)stream, dev, keys, reinterpret_cast<long long*>(idx), count);
}

int simsd_thin_linear_cat(const void* x, int64_t ldx_m, int64_t ldx_k, int parts, const void* const* w,
                          const int64_t* ldw_n, const int* n, void* y, int64_t ldy, int M, int K, int dtype,
                          void* workspace, size_t workspace_bytes, void* stream) {
  if (M < 1 || K < 1 || parts < 1 || parts > 3 || w == nullptr || ldw_n == nullptr || n == nullptr)
    return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return SIMSD_ERR_UNSUPPORTED;
  if (x == nullptr || y == nullptr) return SIMSD_ERR_SHAPE;
  if (workspace == nullptr || workspace_bytes < (size_t)WS_COUNTER_BYTES) return SIMSD_ERR_WORKSPACE;
  if (M > 64 || K < 64 || !cluster_enabled()) return SIMSD_ERR_UNSUPPORTED;
  CatSpec cs;
  cs.parts = parts;
  long long N = 0;
  for (int i = 0; i < parts; ++i) {
    if (w[i] == nullptr || n[i] < 1) return SIMSD_ERR_SHAPE;
    if (i + 1 < parts && n[i] % 128 != 0) return SIMSD_ERR_UNSUPPORTED;
    if (!thin_tc_possible(x, ldx_m, ldx_k, w[i], ldw_n[i], 1, nullptr, M, n[i], K, dtype)) return SIMSD_ERR_UNSUPPORTED;
    cs.w[i] = w[i];
    cs.ldw[i] = ldw_n[i];
    cs.n[i] = n[i];
    N += n[i];
  }
  if (N >= (1LL << 31) || ldy < N) return SIMSD_ERR_SHAPE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  int* err = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + WS_ERR_OFFSET);
  return thin_cluster(x, ldx_m, w[0], ldw_n[0], nullptr, nullptr, y, ldy, M, (int)N, K, dtype, false, err, nullptr,
                      0, 1, 0, (cudaStream_t)stream, dev, nullptr, nullptr, nullptr, &cs);
}

int simsd_rmsnorm(const void* x, int64_t ldx, const void* res, int64_t ldres, void* h_out, int64_t ldh,
                  const void* w, void* y, int64_t ldy, int rows, int n, float eps, int dtype, void* stream) {
  if (rows < 0 || n < 1 || n > 16384) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return SIMSD_ERR_DTYPE;
  if (rows == 0) return SIMSD_OK;
  if (!x || !w || !y || ldx < n || ldy < n || (res && ldres < n) || (h_out && ldh < n)) return SIMSD_ERR_SHAPE;
  RmsNormArgs a;
  a.x = x;
  a.res = res;
  a.h_out = h_out;
  a.w = w;
  a.y = y;
  a.ldx = ldx;
  a.ldres = ldres;
  a.ldh = ldh;
  a.ldy = ldy;
  a.rows = rows;
  a.n = n;
  a.dtype = dtype;
  a.eps = eps;
  auto al16 = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  const bool vec = (n & 7) == 0 && (ldx & 7) == 0 && (ldy & 7) == 0 && (!res || (ldres & 7) == 0) &&
                   (!h_out || (ldh & 7) == 0) && al16(x) && al16(w) && al16(y) && (!res || al16(res)) &&
                   (!h_out || al16(h_out));
  if (vec) {
    // 16-byte vectors, the row in registers (<= 8 vectors a thread)
    const int vpt = (int)cdiv(n / 8, NORM_THREADS);
    const dim3 g((unsigned)rows), b(NORM_THREADS);
    if (vpt <= 1) return launch(rmsnorm_vec_kernel<1>, g, b, 0, (cudaStream_t)stream, a);
    if (vpt <= 2) return launch(rmsnorm_vec_kernel<2>, g, b, 0, (cudaStream_t)stream, a);
    if (vpt <= 4) return launch(rmsnorm_vec_kernel<4>, g, b, 0, (cudaStream_t)stream, a);
    return launch(rmsnorm_vec_kernel<8>, g, b, 0, (cudaStream_t)stream, a);
  }
  const int smem = (n + NORM_THREADS / 32) * (int)sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(rmsnorm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return SIMSD_ERR_LAUNCH;
  return launch(rmsnorm_kernel, dim3((unsigned)rows), dim3(NORM_THREADS), smem, (cudaStream_t)stream, a);
}

int simsd_qk_norm_rope(const void* qkv, int64_t ldqkv, int L, int Hq, int Hk, int head_dim, const void* q_weight,
                       const void* k_weight, const void* cos, const void* sin, float eps, void* q_out, void* k_cache,
                       void* v_cache, int64_t cache_cap, int pos, int dtype, void* stream) {
  if (L < 0 || Hq < 1 || Hk < 1 || head_dim != 128 || pos < 0) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16 && dtype != SIMSD_F16) return SIMSD_ERR_DTYPE;
  if (L == 0) return SIMSD_OK;
  if (!qkv || !q_weight || !k_weight || !cos || !sin || !q_out || !k_cache || !v_cache) return SIMSD_ERR_SHAPE;
  if (ldqkv < (int64_t)(Hq + 2 * Hk) * head_dim || cache_cap < (int64_t)pos + L) return SIMSD_ERR_SHAPE;
  QkRopeArgs a;
  a.qkv = qkv;
  a.qw = q_weight;
  a.kw = k_weight;
  a.cos = cos;
  a.sin = sin;
  a.q_out = q_out;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.ldqkv = ldqkv;
  a.cache_cap = cache_cap;
  a.L = L;
  a.Hq = Hq;
  a.Hk = Hk;
  a.pos = pos;
  a.dtype = dtype;
  a.eps = eps;
  const long long units = (long long)L * (Hq + 2 * Hk);
  return launch(qk_norm_rope_kernel, dim3((unsigned)cdiv(units, QKR_WARPS)), dim3(QKR_WARPS * 32), 0,
                (cudaStream_t)stream, a);
}

size_t simsd_verify_attention_workspace_size(int Hq, int Hk, int L, int Lk) {
  if (Hq < 1 || Hk < 1 || L < 1 || Lk < 1) return WS_COUNTER_BYTES;
  const long long nch = cdiv(Lk, ATT_KC);
  return WS_COUNTER_BYTES + align256((size_t)Hk * nch * ATT_R * (ATT_D + 2) * sizeof(float));
}

int simsd_verify_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_cap, int Hq,
                           int Hk, int L, int Lk, const uint8_t* mask, int64_t ldmask, float scale, void* o,
                           int dtype, void* workspace, size_t workspace_bytes, void* stream) {
  if (Hq < 1 || Hk < 1 || L < 1 || Lk < 1 || Hq % Hk != 0) return SIMSD_ERR_SHAPE;
  if (dtype != SIMSD_BF16) return SIMSD_ERR_UNSUPPORTED;
  if ((Hq / Hk) * L > ATT_R) return SIMSD_ERR_UNSUPPORTED;
  if (!q || !k_cache || !v_cache || !mask || !o || cache_cap < Lk || ldmask < Lk) return SIMSD_ERR_SHAPE;
  auto al16 = [](const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
  if (!al16(q) || !al16(k_cache) || !al16(v_cache) || !al16(o)) return SIMSD_ERR_ALIGN;
  const int nch = (int)cdiv(Lk, ATT_KC);
  if (workspace == nullptr || workspace_bytes < simsd_verify_attention_workspace_size(Hq, Hk, L, Lk))
    return SIMSD_ERR_WORKSPACE;
  const int dev = current_device();
  if (dev < 0) return SIMSD_ERR_DEVICE;
  cudaStream_t st = (cudaStream_t)stream;
  // tensor cores (tcgen05), one cluster of up to 8 CTAs per KV head: needs at
  // most 3 key tiles per CTA and TMA-describable q / caches
  const int ntiles = (int)cdiv(Lk, ATC_TILE);
  if (attn_tc_enabled() && scale > 0.0f && ntiles <= ATC_CL_MAX * ATC_NT_MAX && (long long)Hk * cache_cap < (1LL << 31) &&
      (long long)Hq * L < (1LL << 31) && ensure_encode() == SIMSD_OK) {
    AttnTcArgs t;
    memset(&t, 0, sizeof(t));
    const uint64_t qd[2] = {128, (uint64_t)Hq * L}, kd[2] = {128, (uint64_t)(Hk * cache_cap)};
    const uint64_t rs[1] = {256};
    int rc = encode_map(&t.tmQ, q, SIMSD_BF16, 2, qd, rs, 128);
    if (rc == SIMSD_OK) rc = encode_map(&t.tmK, k_cache, SIMSD_BF16, 2, kd, rs, 128);
    if (rc == SIMSD_OK) rc = encode_map(&t.tmV, v_cache, SIMSD_BF16, 2, kd, rs, 128);
    if (rc == SIMSD_OK) {
      t.mask = mask;
      t.o = o;
      t.err = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + WS_ERR_OFFSET);
      t.cap = cache_cap;
      t.ldm = ldmask;
      t.Hq = Hq;
      t.Hk = Hk;
      t.L = L;
      t.Lk = Lk;
      t.ntiles = ntiles;
      t.mask_vec = ((ldmask & 15) == 0 && al16(mask)) ? 1 : 0;
      t.scale_log2 = scale * 1.4426950408889634f;
      // at most two key tiles per CTA where a cluster that large runs here
      // (every tile's loads then issue at once), else up to three in 8
      int S = std::min(ATC_CL_MAX, ntiles);
      const int S2 = (int)cdiv(ntiles, 2);
      if (S2 > ATC_CL_MAX && S2 <= ATC_CL_MAX_NP && attn_max_clusters(S2, dev) > 0) S = S2;
      t.trace = trace_slot((long long)Hk * S);
      {
        static bool done_tc[kMaxDev];
        std::lock_guard<std::mutex> lk(g_mu);
        if (!done_tc[dev]) {
          if (cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATC_SMEM) !=
              cudaSuccess)
            return SIMSD_ERR_LAUNCH;
          (void)cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
          (void)cudaGetLastError();
          done_tc[dev] = true;
        }
      }
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3((unsigned)(Hk * S));
      cfg.blockDim = dim3(ATC_THREADS);
      cfg.dynamicSmemBytes = ATC_SMEM;
      cfg.stream = st;
      cudaLaunchAttribute attr[2];
      int na = 0;
      attr[na].id = cudaLaunchAttributeClusterDimension;
      attr[na].val.clusterDim.x = (unsigned)S;
      attr[na].val.clusterDim.y = 1;
      attr[na].val.clusterDim.z = 1;
      ++na;
      if (pdl_on()) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
      }
      cfg.attrs = attr;
      cfg.numAttrs = na;
      if (cudaLaunchKernelEx(&cfg, attn_tc_kernel, t) != cudaSuccess) return SIMSD_ERR_LAUNCH;
      return cudaGetLastError() == cudaSuccess ? SIMSD_OK : SIMSD_ERR_LAUNCH;
    }
  }
  AttnArgs a;
  a.q = q;
  a.k = k_cache;
  a.v = v_cache;
  a.mask = mask;
  a.o = o;
  a.part_o = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) + WS_COUNTER_BYTES);
  a.part_ml = a.part_o + (size_t)Hk * nch * ATT_R * ATT_D;
  a.cap = cache_cap;
  a.ldm = ldmask;
  a.Hq = Hq;
  a.Hk = Hk;
  a.L = L;
  a.Lk = Lk;
  a.nchunks = nch;
  a.scale_log2 = scale * 1.4426950408889634f;
  constexpr int smem = 3 * 32768;
  {
    static bool done[kMaxDev];
    std::lock_guard<std::mutex> lk(g_mu);
    if (!done[dev]) {
      if (cudaFuncSetAttribute(attn_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
        return SIMSD_ERR_LAUNCH;
      done[dev] = true;
    }
  }
  int rc = launch(attn_split_kernel, dim3((unsigned)nch, (unsigned)Hk), dim3(ATT_THREADS), smem, st, a);
  if (rc != SIMSD_OK) return rc;
  const long long units = (long long)Hk * (Hq / Hk) * L;
  return launch(attn_combine_kernel, dim3((unsigned)cdiv(units, 8)), dim3(256), 0, st, a);
}

}  // extern "C"
