/*
 * simsd_b200.h - C ABI of the B200 (sm_100a) matmul hot path of SimSD.
 *
 * Plain pointers and sizes only: no torch or C++ types cross this boundary.
 * All device pointers must belong to the device that is current on the calling
 * thread; `stream` is a cudaStream_t (NULL = legacy default stream).  Every
 * call is asynchronous on `stream`, performs no host synchronisation and no
 * allocation, and is safe inside CUDA-graph capture.
 *
 * Workspaces are owned by the caller.  The first 256 KiB of every workspace
 * hold per-tile counters and a device error word: zero them once when the
 * workspace is created (simsd_workspace_init); the kernels leave them zero.
 * Calls that share a workspace must be ordered on one stream (overlapping calls
 * on different streams race on it), which is how the reference shares its
 * split-K staging buffer (kernels/thin_linear_fused.py:173-190).
 *
 * Return value: SIMSD_OK or a negative SIMSD_ERR_* code.  Device-side faults
 * that a kernel can detect (a bounded wait that ran out, an out-of-range expert
 * id) are OR-ed into the workspace's error word; read it with
 * simsd_workspace_error().
 */
#ifndef SIMSD_B200_H
#define SIMSD_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes */
#define SIMSD_OK 0
#define SIMSD_ERR_SHAPE -1        /* bad rank / size / K mismatch            -> ValueError */
#define SIMSD_ERR_DTYPE -2        /* unsupported or mismatched dtype         -> TypeError  */
#define SIMSD_ERR_WORKSPACE -3    /* workspace missing or too small                         */
#define SIMSD_ERR_LAUNCH -4       /* CUDA launch / attribute error                          */
#define SIMSD_ERR_ALIGN -5        /* pointer or stride unusable by the requested path       */
#define SIMSD_ERR_DEVICE -6       /* no usable CUDA device / driver entry point             */
#define SIMSD_ERR_UNSUPPORTED -7  /* valid request outside this build's limits              */
#define SIMSD_ERR_SCRATCH_LIMIT -8 /* simsd_thin_linear_noalloc: needs more than its static scratch */

/* ---- element types */
#define SIMSD_BF16 0
#define SIMSD_F16 1
#define SIMSD_F32 2

/* ---- thin linear epilogues */
#define SIMSD_EPI_NONE 0     /* y = x w^T (+ bias)                                   */
#define SIMSD_EPI_SILU_MUL 1 /* y = silu(x w_gate^T) * (x w_up^T), N = intermediate  */

/* ---- thin linear paths */
#define SIMSD_PATH_AUTO 0    /* tensor cores where the layout allows, else CUDA cores */
#define SIMSD_PATH_TC 1      /* force the tcgen05/TMA kernel (SIMSD_ERR_ALIGN if not possible) */
#define SIMSD_PATH_SIMT 2    /* force the CUDA-core kernel                            */

/* ---- device error bits (OR-ed into a device error word) */
#define SIMSD_DEV_ERR_TIMEOUT   1   /* a bounded wait ran out (the kernel gave up cleanly) */
#define SIMSD_DEV_ERR_BAD_INDEX 2   /* an expert id >= E */
#define SIMSD_DEV_ERR_CAPACITY  4   /* an expert-parallel bucket overflowed */

/* ---- launch flags (process-wide) */
#define SIMSD_LAUNCH_PDL 1   /* programmatic dependent launch, see simsd_set_launch_flags */
#define SIMSD_LAUNCH_INKERNEL_REDUCE 2  /* split-K tiles summed inside the GEMM, see below */
#define SIMSD_LAUNCH_GROUPED_FIXUP 4    /* MoE grouped GEMMs: split tiles summed by a second kernel */
#define SIMSD_LAUNCH_MOE_SIZE_CLASSES 8 /* MoE dispatch: large groups in a second, 256-row-tile launch */

/* Library version string. */
const char* simsd_version(void);

/* Human-readable name of a status code. */
const char* simsd_status_string(int status);

/*
 * Set the process-wide launch flags; returns the previous ones.  No counterpart
 * in the reference (its Triton launches have no such option).
 * SIMSD_LAUNCH_PDL: launch every kernel as a programmatic dependent of the
 * previous kernel on its stream, so its set-up and, for simsd_thin_linear, the
 * first ring of weight tiles overlap that kernel's tail; activations are read
 * and outputs written only after the previous kernel has completed.  Only set
 * it when the weights passed to simsd_thin_linear are not written by the kernel
 * launched just before it on the same stream (true for inference with fixed
 * weights).
 * SIMSD_LAUNCH_INKERNEL_REDUCE: a tile whose K range is split over several CTAs
 * is summed by the last of them to finish (counted per tile in the workspace
 * header) instead of by a separate reduction kernel launched after the GEMM.
 * Same summation order, so the two give identical bits.  The MoE dispatch's
 * grouped GEMMs always sum split tiles inside the GEMM (whether any tile is
 * split depends on the routing, which the host does not read, so a reduction
 * kernel would be launched for nothing at most token counts), unless
 * SIMSD_LAUNCH_GROUPED_FIXUP asks for the separate kernel (same bits).
 * SIMSD_LAUNCH_MOE_SIZE_CLASSES: simsd_moe_dispatch runs each grouped GEMM as
 * two launches, the experts with at most the planned tile height of rows in
 * one and the larger ones in another with 256-row tiles (each launch reads the
 * counts on the device and takes only its class).  For skewed routing (a
 * router bias that concentrates tokens on a few experts): about 20 % faster on
 * a 4096-wide layer with N(0, 0.5) bias at 256-1024 tokens, slower for
 * near-uniform routing.  Same results either way within rounding (the tiles'
 * K order is the same; only which launch computes a group changes).
 */
int simsd_set_launch_flags(int flags);

/* Current launch flags. */
int simsd_get_launch_flags(void);

/*
 * Diagnostics (no counterpart in the reference): while `buf` is set, the
 * tensor-core GEMM launches write 8 %globaltimer stamps (ns) per CTA into
 * successive records of 64 * grid bytes (the first launch at buf[cta*8 + i],
 * the next right after it, ...) while the buffer has room: entry, set-up done,
 * first TMA issued, first MMA stage ready, last TMA issued, last MMA
 * committed, SM id (not a time), exit.  Setting the buffer starts again at
 * its head.  NULL disables.  Not for concurrent use.
 */
int simsd_debug_set_trace(void* buf, size_t bytes);

/*
 * Diagnostics: the cluster plan simsd_thin_linear uses for an M <= 64 thin
 * linear (S CTAs per cluster, C clusters; S = 0 when no plan fits) and, when
 * `max_clusters_by_s` is not NULL, the clusters of size 1..8 that fit the
 * device at once (8 ints).
 */
int simsd_debug_cluster_plan(int M, int N, int K, int silu, int* S, int* C, int* max_clusters_by_s);

/* Number of SMs of the current device (0 if there is none). */
int simsd_device_sm_count(void);

/* Bytes every workspace reserves at its head for counters and the error word. */
size_t simsd_workspace_header_bytes(void);

/* Zero a workspace's header on `stream` (asynchronous; call once per new workspace). */
int simsd_workspace_init(void* workspace, size_t workspace_bytes, void* stream);

/* Copy the workspace's device error word to *out (synchronises `stream`; not for the hot path). */
int simsd_workspace_error(const void* workspace, void* stream, int* out);

/*
 * Workspace bytes simsd_thin_linear needs for this shape (header included).
 * `split` as in simsd_thin_linear.
 */
size_t simsd_thin_linear_workspace_size(int M, int N, int K, int dtype, int epilogue, int split);

/*
 * Thin-M linear:  y[m, n] = sum_k x[m, k] * w[n, k]  (+ bias[n]),  fp32 accumulate.
 * Replaces thin_linear(x, w, bias, config) - kernels/thin_linear_fused.py:265-345
 * (kernels _thin_gemv_kernel :67-136 and _thin_gemv_reduce :139-167).
 *
 *   x    [M, K]  element (m, k) at x + m*ldx_m + k*ldx_k   (strided views allowed)
 *   w    [N, K]  element (n, k) at w + n*ldw_n + k*ldw_k   (nn.Linear weight layout)
 *   w_up [N, K]  same strides as w; SIMSD_EPI_SILU_MUL only (w is then the gate weight)
 *   bias [N]     or NULL (same dtype as x; SIMSD_EPI_NONE only)
 *   y    [M, N]  element (m, n) at y + m*ldy_m + n
 *   dtype        SIMSD_BF16 | SIMSD_F16 | SIMSD_F32 (x, w, bias and y share it).
 *                fp32 with M <= 64 and split 0 runs on the tensor cores with each
 *                operand split on chip into two tf32 parts (hi*hi + hi*lo + lo*hi,
 *                about 2^-21 relative per product, fp32 accumulation - never a
 *                one-pass TF32 product); other fp32 calls, and SIMSD_PATH_SIMT,
 *                use IEEE fp32 FMA on the CUDA cores.
 *   split        0: balance the K reduction over all SMs (deterministic stream-K);
 *                s > 0: exactly s K-segments per output tile (the reference's
 *                config SPLIT_K); the sum order is fixed either way, so repeated
 *                calls are bit-identical.
 *   path         SIMSD_PATH_*.
 * M, N, K >= 1.  Any M is accepted; the tensor-core path reads w once per 256 rows of x.
 */
int simsd_thin_linear(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n,
                      int64_t ldw_k, const void* w_up, const void* bias, void* y, int64_t ldy_m, int M,
                      int N, int K, int dtype, int epilogue, int split, int path, void* workspace,
                      size_t workspace_bytes, void* stream);

/*
 * simsd_thin_linear without a workspace: the same computation (and the same
 * arguments minus split, path and workspace), for callers that cannot allocate
 * device memory or own a scratch buffer - a plugin host that hands out only the
 * tensors of the call and forbids allocation from plugins, code running inside
 * an allocator's own callback, or a foreign-language binding that has no CUDA
 * allocator to draw from.  No counterpart in the reference (its Triton kernel
 * allocates a staging buffer through torch).
 *
 * The split-K partials live in a fixed 8 MiB device array inside this library
 * (held by every GPU that loads it until the process exits); the call itself
 * allocates nothing and frees nothing.  A shape whose partials do not fit is
 * rejected with SIMSD_ERR_SCRATCH_LIMIT (on a 148-SM B200 this admits M <= 32
 * for every N and K; layouts that take the CUDA-core path need no partials).
 * The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) with that device current: make that first call before
 * any stream capture.  The address is kept for the life of the device's primary
 * context; do not call this entry point again after cudaDeviceReset.  All calls share the one array: calls that may overlap on
 * the GPU (different streams, or different host threads) race and must be
 * serialised by the caller.  A launch that gives up (a bounded wait ran out)
 * sets a bit in the array's error word, which keeps it across calls until
 * simsd_thin_linear_noalloc_error reads and clears it.
 */
int simsd_thin_linear_noalloc(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w,
                              int64_t ldw_n, int64_t ldw_k, const void* w_up, const void* bias,
                              void* y, int64_t ldy_m, int M, int N, int K, int dtype,
                              int epilogue, void* stream);

/*
 * The device error word of simsd_thin_linear_noalloc's static array on the
 * current device (SIMSD_DEV_ERR_* bits; 0 = every call since the last non-zero
 * read completed), read after the work queued on `stream` finishes (this call waits
 * for that stream).  A non-zero word means a launch gave up (a bounded wait ran
 * out) and its output is incomplete; this call then zeroes the array's whole
 * header - the error word and the per-tile arrival counters an aborted launch
 * may leave raised - so later calls start clean.  No counterpart in the
 * reference.  Same serialisation rule as simsd_thin_linear_noalloc.
 */
int simsd_thin_linear_noalloc_error(void* stream, int* out);

/*
 * MoE router: logits = x wr^T (fp32, fixed summation order), score = sigmoid(logits),
 * top-k by score + bias (ties to the lower expert id), weights = score of the chosen
 * experts, renormalised to sum 1 (+1e-20) when `renorm` and k > 1, then times `scale`.
 * Restates the synthetic router of kernels/workspace/moe_dispatch/build_oracle.py:71-90
 * with the selection bias of the LLaDA2 gate (remote code, absent from the reference).
 *
 *   x [T, H] (row stride ldx, x_dtype), wr [E, H] (row stride ldw, w_dtype),
 *   bias [E] fp32 or NULL -> topk_ids [T, k] int64, topk_weight [T, k] fp32,
 *   logits [T, E] fp32 or NULL (optional copy of the logits).
 * 1 <= k <= min(E, 32), E <= 1024.
 */
int simsd_moe_route(const void* x, int64_t ldx, int x_dtype, const void* wr, int64_t ldw,
                    int w_dtype, const float* bias, int T, int H, int E, int k, int renorm,
                    float scale, int64_t* topk_ids, float* topk_weight, float* logits,
                    void* stream);

/*
 * simsd_moe_route with the outputs at row stride ld_topk (>= k, or >= k + 1 with
 * extra_id) and, when extra_id >= 0, column k of every row set to (extra_id,
 * 1.0): the always-on shared expert stacked after the routed ones, for
 * simsd_moe_dispatch_shared_last.
 */
int simsd_moe_route_ex(const void* x, int64_t ldx, int x_dtype, const void* wr, int64_t ldw, int w_dtype,
                       const float* bias, int T, int H, int E, int k, int renorm, float scale, int64_t* topk_ids,
                       float* topk_weight, int64_t ld_topk, int extra_id, float* logits, void* stream);

/*
 * Expert align: per-expert counts, offsets and the stable slot permutation.
 * Replaces _align - kernels/moe_dispatch_fused.py:93-132 (bit-exact).
 *
 *   topk_ids [S] int64 (S = T*k, slot s = t*k + j), 0 <= id < E <= 1024; a
 *   negative id is a slot without an expert (an empty expert-parallel bucket
 *   entry): it is left out silently; an id >= E is left out and raises
 *   SIMSD_DEV_ERR_BAD_INDEX.  (The reference has no such slots.)
 *   counts [E], offsets [E+1] (exclusive prefix of counts), sorted_slots [S]
 *   (= argsort(ids, stable=True) over the kept slots, then -1), slot_to_row [S]
 *   (its inverse; -1 for a slot left out)
 *   slots_padded [num_tiles*block_m] and tile_expert [num_tiles]: optional (both NULL
 *   or both set) copies in the reference's padded layout (`slots`, `tile_expert`).
 *   `err_word`: device int that receives SIMSD_DEV_ERR bits, or NULL.
 */
int simsd_moe_align(const int64_t* topk_ids, int S, int E, int32_t* counts, int32_t* offsets,
                    int32_t* sorted_slots, int32_t* slot_to_row, int block_m, int num_tiles,
                    int32_t* slots_padded, int32_t* tile_expert, int* err_word, void* stream);

/* Workspace bytes simsd_moe_dispatch needs (header included). */
size_t simsd_moe_workspace_size(int T, int k, int E, int H, int I, int dtype);

/*
 * Fused MoE expert dispatch, CUDA-graph capturable (no host sync):
 *   out[t] = cast( sum_j fp32(down_e(silu(gate_e(x_t)) * up_e(x_t))) * topk_weight[t, j] )
 * with e = topk_ids[t, j]; when `add` is not NULL, out[t] = cast(cast(that sum) + add[t])
 * (the shared expert's output added in x.dtype, as the model does).
 * Replaces moe_dispatch(x, topk_ids, topk_weight, w_gate, w_up, w_down) -
 * kernels/moe_dispatch_fused.py:165-192 (stock moe_infer, transcribed at
 * kernels/workspace/moe_dispatch/build_oracle.py:34-67).
 *
 *   x [T, H] (row stride ldx), topk_ids [T, k] int64, topk_weight [T, k] fp32,
 *   w_gate, w_up [E, I, H]: element (e, i, h) at base + e*ldg_e + i*ldg_i + h
 *   w_down [E, H, I]:       element (e, h, i) at base + e*ldd_e + h*ldd_h + i
 *   out [T, H] (row stride ld_out), add [T, H] (row stride ld_add) or NULL.
 *   dtype: x, weights, out and add share it (SIMSD_BF16 | SIMSD_F16 | SIMSD_F32).
 * Slots whose id is negative contribute nothing (see simsd_moe_align).
 */
int simsd_moe_dispatch(const void* x, int64_t ldx, const int64_t* topk_ids,
                       const float* topk_weight, const void* w_gate, const void* w_up,
                       int64_t ldg_e, int64_t ldg_i, const void* w_down, int64_t ldd_e,
                       int64_t ldd_h, void* out, int64_t ld_out, const void* add,
                       int64_t ld_add, int T, int k, int E, int H, int I, int dtype,
                       void* workspace, size_t workspace_bytes, void* stream);

/*
 * simsd_moe_dispatch whose last routing column (k - 1) is an always-on shared
 * expert stacked as an expert of w_gate / w_up / w_down: its rows run in the
 * same grouped GEMMs as the routed experts, and the combine adds its output
 * unweighted to the rounded sum of the other columns — cast(cast(sum) +
 * shared), the reference model's `moe_infer(...) + shared_experts(x)`.
 */
int simsd_moe_dispatch_shared_last(const void* x, int64_t ldx, const int64_t* topk_ids, const float* topk_weight,
                                   const void* w_gate, const void* w_up, int64_t ldg_e, int64_t ldg_i,
                                   const void* w_down, int64_t ldd_e, int64_t ldd_h, void* out, int64_t ld_out,
                                   int T, int k, int E, int H, int I, int dtype, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* ---- column-parallel thin linear with the all-gather fused in (no counterpart in
 * the reference).  Each rank of a node holds rows [rank*N, (rank+1)*N) of the
 * full weight and writes its output columns straight into every rank's y
 * (NVLink peer stores).  The launch carries no signal and nothing waits inside
 * it: before reading y, every rank calls simsd_allgather_wait on the same
 * stream (one sync point may cover several launches).  All ranks must make the
 * same sequence of these calls with the same shapes. */

#define SIMSD_IPC_HANDLE_BYTES 64
#define SIMSD_SIGNAL_BYTES 256   /* one rank's signal block (zeroed by simsd_ipc_alloc) */

/* Device memory other processes of the node can map: cudaMalloc'd, zeroed. */
int simsd_ipc_alloc(size_t bytes, void** dev_ptr);
int simsd_ipc_free(void* dev_ptr);
/* Export a simsd_ipc_alloc block (SIMSD_IPC_HANDLE_BYTES bytes into `handle`). */
int simsd_ipc_handle(const void* dev_ptr, void* handle);
/* Map another process's exported block on the current device. */
int simsd_ipc_open(const void* handle, void** dev_ptr);
int simsd_ipc_close(void* dev_ptr);

/*
 * y_r[m, col_offset + n] = (x w^T)[m, n] (+ bias[n]) for every rank r, or the
 * SiLU*mul epilogue with w_up; n < N (this rank's output columns).
 *   peer_y [world]: every rank's y (same layout, row stride ldy), this rank's
 *   own at peer_y[rank].
 * plan_n > 0: split each output tile's K range exactly as simsd_thin_linear
 * would for an [M, plan_n] output (plan_n = the unsharded width), so every
 * element is summed in the single-GPU order and the gathered y is bit-identical
 * to the single-GPU result (at some cost in CTAs per rank); 0: plan for this
 * rank's N alone.
 * 1 < world <= 8, M <= 64, bf16/fp16 with TMA-describable layouts; other
 * requests return SIMSD_ERR_UNSUPPORTED (use simsd_thin_linear and a
 * collective instead).
 */
int simsd_thin_linear_allgather(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w,
                                int64_t ldw_n, int64_t ldw_k, const void* w_up, const void* bias,
                                void* const* peer_y, int64_t ldy, int col_offset, int M, int N,
                                int K, int dtype, int epilogue, int rank, int world,
                                int plan_n, void* workspace, size_t workspace_bytes,
                                void* stream);

/*
 * Sync point of simsd_thin_linear_allgather (no counterpart in the reference):
 * one single-thread kernel on `stream` that, once every earlier kernel on the
 * stream has completed (so this rank's peer stores are performed), adds 1 with
 * release to the arrival counter of every rank's signal block and then waits
 * until its own counter reaches world x this rank's count of sync points: every
 * rank has stored its columns of every fused launch it issued before the same
 * sync point.  Kernels after it on `stream` read the gathered outputs.  Every
 * rank calls it at the same points of the call sequence.  Counters are
 * cumulative, compared modulo 2^32.  The wait is bounded (2 s): a rank that
 * never arrives sets SIMSD_DEV_ERR_TIMEOUT in the workspace error word instead
 * of hanging.  peer_signal [world]: every rank's signal block (this rank's own
 * at peer_signal[rank]), each SIMSD_SIGNAL_BYTES zeroed bytes.
 */
int simsd_allgather_wait(void* const* peer_signal, int rank, int world, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * Greedy verify head: idx[m] = argmax_n round(x[m] . w[n] (+ bias[n])), the
 * rounding to `dtype` (the logits tensor the reference's lm_head returns), ties
 * to the lowest n (torch.argmax) — without writing the [M, N] logits.  Replaces
 * the reference's `lm_head(hidden)` followed by softmax / argmax on the accepted
 * rows (speculative_decoding/cache_aware.py:1193-1196, mrs.py:138): softmax is
 * monotonic, so its argmax is the logits' argmax.  M <= 64, K >= 64, bf16/fp16
 * with TMA-describable layouts, else SIMSD_ERR_UNSUPPORTED (use
 * simsd_thin_linear and an argmax).  Uses the workspace header's argmax slots
 * (zero between calls: after a device error, re-initialise the workspace).
 */
int simsd_thin_linear_argmax(const void* x, int64_t ldx_m, int64_t ldx_k, const void* w, int64_t ldw_n,
                             int64_t ldw_k, const void* bias, int64_t* idx, int M, int N, int K, int dtype,
                             void* workspace, size_t workspace_bytes, void* stream);

/*
 * Linears that share their input, in one launch: y[:, off_i : off_i + n[i]] =
 * x . w[i]^T for i < parts (<= 3), off_i = n[0] + ... + n[i-1] — the merged
 * q/k/v projection (the reference measured its merged qkv at -138 us per
 * forward, kernels/workspace/thin_linear/CONTRACT.md:287-289) without copying
 * the three weights into one.  w[i] [n[i], K] row-major with row stride
 * ldw_n[i] (unit K stride); every part but the last a multiple of 128 rows; y
 * row stride ldy >= the total width.  M <= 64, K >= 64, bf16/fp16 with
 * TMA-describable layouts, else SIMSD_ERR_UNSUPPORTED (use simsd_thin_linear
 * per part).
 */
int simsd_thin_linear_cat(const void* x, int64_t ldx_m, int64_t ldx_k, int parts, const void* const* w,
                          const int64_t* ldw_n, const int* n, void* y, int64_t ldy, int M, int K, int dtype,
                          void* workspace, size_t workspace_bytes, void* stream);

/*
 * Layer ops of the verify forward around its linears (sdar/modeling_sdar.py with
 * the fp32 RMSNorm of sdar/run_native_tp2.py:34-51):
 *
 * simsd_rmsnorm: per row r < rows, h = x[r] (res == NULL) or h = round(x[r] +
 * res[r]) (also stored to h_out when not NULL), y[r] = w * round(h_f32 *
 * rsqrt(mean(h_f32^2) + eps)), the product rounded to dtype.  n <= 16384.
 *
 * simsd_qk_norm_rope: the attention front end for L tokens at positions pos..
 * pos+L-1 of one sequence, head_dim 128.  qkv [L, (Hq + 2 Hk) * 128] (row stride
 * ldqkv; q heads, k heads, v heads) -> q_out [Hq, L, 128] = rope(rmsnorm(q)),
 * k_cache[g, pos + t] = rope(rmsnorm(k)), v_cache[g, pos + t] = v (caches
 * [Hk, cache_cap, 128]); rope(x) = round(round(x cos) + round(rotate_half(x) sin))
 * with cos/sin [L, 128] in dtype.  Replaces the per-layer q_norm / k_norm,
 * rotary embedding and KV-cache write (sdar/modeling_sdar.py:197-302 with the
 * reference's static cache writes, speculative_decoding/cache_aware.py).
 */
int simsd_rmsnorm(const void* x, int64_t ldx, const void* res, int64_t ldres, void* h_out, int64_t ldh,
                  const void* w, void* y, int64_t ldy, int rows, int n, float eps, int dtype, void* stream);
int simsd_qk_norm_rope(const void* qkv, int64_t ldqkv, int L, int Hq, int Hk, int head_dim, const void* q_weight,
                       const void* k_weight, const void* cos, const void* sin, float eps, void* q_out, void* k_cache,
                       void* v_cache, int64_t cache_cap, int pos, int dtype, void* stream);

/*
 * Verify attention over a static KV cache with native GQA (no expanded K/V):
 *   o[t, h, :] = softmax_j(scale * q[h, t] . k[g, j], keys j < Lk with
 *                mask[t * ldmask + j] != 0) v[g, j],  g = h / (Hq / Hk)
 * q [Hq, L, 128], k_cache / v_cache [Hk, cache_cap, 128], o [L, Hq, 128] (the
 * layout the output projection reads), all bf16 contiguous; mask bytes
 * (torch.bool) [L, ldmask].  Split over 128-key chunks (flash decoding) on the
 * tensor cores, chunks merged by a second kernel; fp32 softmax.  A row with
 * every key masked comes out as zeros.  (Hq / Hk) * L <= 128, else
 * SIMSD_ERR_UNSUPPORTED.  Replaces SDPA with enable_gqa over the reference's
 * expanded KV (speculative_decoding/cache_aware.py:195-215).
 */
size_t simsd_verify_attention_workspace_size(int Hq, int Hk, int L, int Lk);
int simsd_verify_attention(const void* q, const void* k_cache, const void* v_cache, int64_t cache_cap, int Hq,
                           int Hk, int L, int Lk, const uint8_t* mask, int64_t ldmask, float scale, void* o,
                           int dtype, void* workspace, size_t workspace_bytes, void* stream);

/* ---- expert parallelism (no counterpart in the reference, which runs the MoE
 * layer on one GPU): experts split over `world` ranks in contiguous blocks of
 * E / world, tokens routed on their owner rank, rows exchanged with all-to-all
 * in fixed-capacity per-peer buckets (so the exchange is CUDA-graph capturable),
 * each rank running simsd_moe_dispatch on the rows it receives (k = 1, weight 1,
 * negative id = empty entry), and the owner combining the returned rows. */

/*
 * Bucket plan of this rank's slots: for slot s = t*k + j with expert e =
 * topk_ids[s], peer = e / (E / world); in slot order each peer's slots take
 * positions 0, 1, ... of its bucket: send_slot[peer*capacity + i] = s,
 * send_expert[...] = e % (E / world), slot_pos[s] = peer*capacity + i.  Unused
 * bucket entries are -1.  A slot past `capacity` (SIMSD_DEV_ERR_CAPACITY) or with
 * an id outside [0, E) (SIMSD_DEV_ERR_BAD_INDEX for id >= E) gets slot_pos -1.
 * counts[peer] = slots bound for the peer.  E % world == 0, world <= 64.
 */
int simsd_moe_ep_plan(const int64_t* topk_ids, int S, int E, int world, int capacity,
                      int32_t* send_slot, int32_t* send_expert, int32_t* slot_pos,
                      int32_t* counts, int* err_word, void* stream);

/*
 * out[r, :] = x[slots[r] / k, :] for r < R; rows with slots[r] < 0 are left as
 * they are.  x [*, H] row stride ldx, out [R, H] row stride ld_out.
 */
int simsd_moe_gather_rows(const void* x, int64_t ldx, const int32_t* slots, int R, int k, int H,
                          int dtype, void* out, int64_t ld_out, void* stream);

/*
 * out[t] = cast( sum_j fp32(ys[slot_row[t*k + j]]) * topk_weight[t, j] ) over
 * j in order, rows -1 skipped; with `add`, out[t] = cast(cast(sum) + add[t]).
 * The combine step of simsd_moe_dispatch on rows the caller supplies.
 */
int simsd_moe_combine(const void* ys, int64_t ldys, const int32_t* slot_row,
                      const float* topk_weight, void* out, int64_t ld_out, const void* add,
                      int64_t ld_add, int T, int k, int H, int dtype, void* stream);

/*
 * The expert-parallel layer's exchanges as plain stores into every rank's
 * blocks (NVLink peer mappings from simsd_ipc_open; no counterpart in the
 * reference, which runs its MoE layer on one GPU).  Replaces the two
 * all-to-alls of fixed-capacity buckets: only occupied bucket entries move a
 * row, and nothing is staged in a send buffer.  Entry e = p * capacity + i of
 * this rank's buckets (send_slot / send_expert from simsd_moe_ep_plan) lands in
 * row rank * capacity + i of rank p's blocks.
 *
 * simsd_moe_ep_send: row x[send_slot[e] / k] into peer_rows[p] ([world *
 *   capacity, H], row stride H) for send_slot[e] >= 0, and send_expert[e]
 *   (the local expert id on p, -1 = empty) into peer_ids[p] for every e.
 * simsd_moe_ep_return: row y[e] ([world * capacity, H], row stride ldy) back
 *   into peer_back[p] at row rank * capacity + i for recv_expert[e] >= 0, where
 *   recv_expert is this rank's id block as the sends filled it.
 * Asynchronous: a sync point (simsd_allgather_wait on a signal block of the
 * same ranks) after each call makes every rank's stores complete before its
 * blocks are read.  Rows need 16-byte aligned bases and a row size (and ldx,
 * ldy in bytes) that is a multiple of 16 bytes; otherwise SIMSD_ERR_ALIGN
 * (use the all-to-all exchange).  world <= 8.
 */
int simsd_moe_ep_send(const void* x, int64_t ldx, const int32_t* send_slot, const int32_t* send_expert,
                      int k, int H, int capacity, int rank, int world, void* const* peer_rows,
                      void* const* peer_ids, int dtype, void* stream);
int simsd_moe_ep_return(const void* y, int64_t ldy, const int32_t* recv_expert, int H, int capacity,
                        int rank, int world, void* const* peer_back, int dtype, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* SIMSD_B200_H */
