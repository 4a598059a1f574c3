"""Thin-M linear on B200: a drop-in for `F.linear(x, w, bias)` when M is small.

Mirrors the interface of the reference module kernels/thin_linear_fused.py
(`thin_linear` :265-345, `pick_config` :217-228, `_tuned_for` :231-244,
`should_fuse` :348-377, `ThinLinear` :380-412, `reset_workspace` :193-195,
`make_bench_fn` :418) with the computation moved to libsimsd_b200.so:

* bf16/fp16 with TMA-describable layouts run the tcgen05 kernels: the weight
  rows stream through a TMA ring into the tensor cores (128 weight rows = MMA
  M, the activation rows = MMA N) with fp32 accumulation in TMEM; for M <= 64
  the K range of each output tile is split over the CTAs of a thread-block
  cluster and summed in fixed order over distributed shared memory
  (csrc/tc_cluster.cuh), above that a deterministic stream-K split with a
  fixed-order fixup (csrc/tc_gemm.cuh);
* fp32 with M <= 64 runs the same cluster kernel on the tensor cores with
  every operand split into two tf32 parts on chip (hi*hi + hi*lo + lo*hi,
  about 2^-21 relative per product, fp32 accumulation: far inside the
  reference's 1e-5 fp32 tolerance, never plain one-pass TF32);
* larger fp32, `config`-forced CUDA cores and layouts TMA cannot describe
  (transposed views, rows that are not 16-byte aligned) run the CUDA-core
  kernel (csrc/simt_gemm.cuh), IEEE fp32 FMA.

There is no CPU path: CUDA tensors only, and a missing library raises.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from ._lib import reset_workspace  # noqa: F401  (reference name)

# The tensor-core tile is fixed by the hardware mapping: 128 weight rows
# (tcgen05 M) x 64 K elements (one 128-byte swizzle row) per pipeline stage;
# the activation rows (tcgen05 N) are padded to a multiple of 16.
TILE_N = 128
TILE_K = 64

# Dispatch guard: `ThinLinear` routes M <= FUSE_MAX_M here and larger M to
# cuBLAS.  BASELINE's thin-M range is M = 4..64 (SDAR-8B verify runs M = 32).
FUSE_MAX_M = 64

# Kept for interface parity with the reference, where TUNED held searched
# Triton configs keyed by (K, N).  This kernel needs no per-shape table: the
# stream-K split balances any (K, N) over all SMs.  Entries, if a caller adds
# them, are (BLOCK_M, BLOCK_N, BLOCK_K, SPLIT_K, num_warps, num_stages) and only
# SPLIT_K is honoured.
TUNED: dict[tuple[int, int], tuple[int, int, int, int, int, int]] = {}


def _block_m(M: int) -> int:
    for b in (16, 32, 64, 128):
        if M <= b:
            return b
    return 256


def pick_config(M: int, N: int, K: int, itemsize: int = 2) -> tuple[int, int, int, int]:
    """(BLOCK_M, BLOCK_N, BLOCK_K, SPLIT_K) of the launch; SPLIT_K 0 = stream-K over all SMs."""
    full = _tuned_for(M, N, K)
    if full is not None:
        return full[0], full[1], full[2], full[3]
    return _heuristic_config(M, N, K)


def _tuned_for(M: int, N: int, K: int):
    """The TUNED entry for (K, N), only while M still fits its BLOCK_M."""
    c = TUNED.get((K, N))
    if c is None:
        return None
    return c if _block_m(max(M, 1)) == c[0] else None


def _heuristic_config(M: int, N: int, K: int) -> tuple[int, int, int, int]:
    return _block_m(max(M, 1)), TILE_N, TILE_K, 0


def thin_linear(x: torch.Tensor, w: torch.Tensor,
                bias: torch.Tensor | None = None,
                config: tuple[int, int, int, int] | None = None,
                num_warps: int | None = None,
                num_stages: int | None = None) -> torch.Tensor:
    """`F.linear(x, w, bias)` for thin x, via libsimsd_b200.

    x: [..., K] (leading dims flattened, strided views allowed)
    w: [N, K]   (nn.Linear weight layout; strided views allowed)
    -> [..., N] in x.dtype.  `config[3]` (SPLIT_K) > 0 forces that many K
    segments per output tile; `num_warps` / `num_stages` are accepted for
    signature compatibility and ignored (the kernel's warp roles are fixed).
    """
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad):
        raise RuntimeError(
            "thin_linear is a forward-only inference kernel; it has no backward. "
            "Call it under torch.no_grad() / torch.inference_mode(), or use F.linear "
            "for training.")
    if x.dtype != w.dtype:
        raise TypeError(f"dtype mismatch: x={x.dtype} w={w.dtype}")
    if w.ndim != 2:
        raise ValueError(f"w must be 2-D [N, K], got {tuple(w.shape)}")
    if x.ndim < 1:
        raise ValueError("x must have at least one dimension")
    code = _lib.dtype_code(x.dtype)
    N, K = w.shape
    if x.shape[-1] != K:
        raise ValueError(f"K mismatch: x[..., {x.shape[-1]}] vs w[{N}, {K}]")
    if bias is not None:
        if bias.dtype != x.dtype:
            raise TypeError(f"dtype mismatch: x={x.dtype} bias={bias.dtype}")
        if bias.shape != (N,):
            raise ValueError(f"bias must be [{N}], got {tuple(bias.shape)}")
    dev = _lib.require_cuda(x, w, bias)

    out_shape = (*x.shape[:-1], N)
    M = 1
    for d in x.shape[:-1]:
        M *= d
    y = torch.empty((M, N), device=dev, dtype=x.dtype)
    if M == 0 or N == 0:
        return y.view(out_shape)
    if K == 0:
        y.zero_()
        if bias is not None:
            y += bias
        return y.view(out_shape)
    x2 = x.reshape(M, K)
    if bias is not None and bias.stride(0) != 1:
        bias = bias.contiguous()

    split = 0
    if config is not None:
        split = int(config[3])
    else:
        tuned = _tuned_for(M, N, K)
        if tuned is not None:
            split = int(tuned[3])
    L = _lib.lib()
    with _lib.device_guard(dev):
        nbytes = _lib.thin_workspace_size(torch.cuda.current_device(), M, N, K, code, _lib.EPI_NONE, split)
        ws = _lib.workspace(dev, nbytes)
        rc = L.simsd_thin_linear(
            x2.data_ptr(), x2.stride(0), x2.stride(1),
            w.data_ptr(), w.stride(0), w.stride(1),
            None, bias.data_ptr() if bias is not None else None,
            y.data_ptr(), y.stride(0), M, N, K, code, _lib.EPI_NONE, split, _lib.PATH_AUTO,
            ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "thin_linear")
    return y.view(out_shape)


def thin_linear_silu_mul(x: torch.Tensor, w_gate: torch.Tensor, w_up: torch.Tensor,
                         split: int = 0) -> torch.Tensor:
    """`F.silu(F.linear(x, w_gate)) * F.linear(x, w_up)` in one pass over both weights.

    The SwiGLU front half of `SDARMLP.forward` (sdar/modeling_sdar.py:113-119)
    with the gate and up products kept in fp32 until the single rounding of the
    product.  w_gate and w_up: [I, K] with identical strides (they may be the two
    halves of one fused [2I, K] gate_up weight).  -> [..., I].
    """
    if torch.is_grad_enabled() and (x.requires_grad or w_gate.requires_grad or w_up.requires_grad):
        raise RuntimeError("thin_linear_silu_mul is a forward-only inference kernel.")
    if not (x.dtype == w_gate.dtype == w_up.dtype):
        raise TypeError(f"dtype mismatch: x={x.dtype} w_gate={w_gate.dtype} w_up={w_up.dtype}")
    if w_gate.ndim != 2 or w_gate.shape != w_up.shape:
        raise ValueError(f"w_gate {tuple(w_gate.shape)} and w_up {tuple(w_up.shape)} must be equal 2-D")
    if w_gate.stride() != w_up.stride():
        raise ValueError("w_gate and w_up must have identical strides")
    code = _lib.dtype_code(x.dtype)
    I, K = w_gate.shape
    if x.shape[-1] != K:
        raise ValueError(f"K mismatch: x[..., {x.shape[-1]}] vs w[{I}, {K}]")
    dev = _lib.require_cuda(x, w_gate, w_up)
    out_shape = (*x.shape[:-1], I)
    M = 1
    for d in x.shape[:-1]:
        M *= d
    y = torch.empty((M, I), device=dev, dtype=x.dtype)
    if M == 0 or I == 0:
        return y.view(out_shape)
    if K == 0:
        return y.zero_().view(out_shape)
    x2 = x.reshape(M, K)
    L = _lib.lib()
    with _lib.device_guard(dev):
        nbytes = _lib.thin_workspace_size(torch.cuda.current_device(), M, I, K, code, _lib.EPI_SILU_MUL, split)
        ws = _lib.workspace(dev, nbytes)
        rc = L.simsd_thin_linear(
            x2.data_ptr(), x2.stride(0), x2.stride(1),
            w_gate.data_ptr(), w_gate.stride(0), w_gate.stride(1),
            w_up.data_ptr(), None, y.data_ptr(), y.stride(0), M, I, K, code,
            _lib.EPI_SILU_MUL, split, _lib.PATH_AUTO, ws.data_ptr(), ws.numel(),
            _lib.stream_ptr(dev))
    _lib.check(rc, "thin_linear_silu_mul")
    return y.view(out_shape)


def thin_linear_argmax(x: torch.Tensor, w: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    """`F.linear(x, w, bias).argmax(-1)` without the [..., N] logits: the greedy
    verify head (lm_head then argmax, speculative_decoding/cache_aware.py:1193-1196,
    mrs.py:138).  Each logit is rounded to x.dtype as F.linear's output would be;
    ties go to the lowest index, as torch.argmax.  -> int64 [...].

    One launch of the M <= 64 tensor-core kernel whose epilogue keeps a running
    maximum per row; other requests (M > 64, fp32, odd layouts) run thin_linear
    and an argmax on the device.
    """
    if torch.is_grad_enabled() and (x.requires_grad or w.requires_grad or (bias is not None and bias.requires_grad)):
        raise RuntimeError("thin_linear_argmax is a forward-only inference kernel.")
    if x.dtype != w.dtype or (bias is not None and bias.dtype != x.dtype):
        raise TypeError(f"dtype mismatch: x={x.dtype} w={w.dtype}")
    if w.ndim != 2 or x.shape[-1] != w.shape[1]:
        raise ValueError(f"K mismatch: x[..., {x.shape[-1]}] vs w{tuple(w.shape)}")
    N, K = w.shape
    dev = _lib.require_cuda(x, w, bias)
    lead = x.shape[:-1]
    M = 1
    for d in lead:
        M *= d
    idx = torch.empty((M,), device=dev, dtype=torch.int64)
    if M == 0:
        return idx.view(lead)
    if N == 0:
        raise ValueError("argmax over zero output columns")
    x2 = x.reshape(M, K)
    if bias is not None and bias.stride(0) != 1:
        bias = bias.contiguous()
    rc = _lib.SIMSD_ERR_UNSUPPORTED
    if x.dtype in (torch.bfloat16, torch.float16):
        code = _lib.dtype_code(x.dtype)
        with _lib.device_guard(dev):
            ws = _lib.workspace(dev, _lib.lib().simsd_workspace_header_bytes())
            rc = _lib.lib().simsd_thin_linear_argmax(
                x2.data_ptr(), x2.stride(0), x2.stride(1), w.data_ptr(), w.stride(0), w.stride(1),
                bias.data_ptr() if bias is not None else None, idx.data_ptr(), M, N, K, code,
                ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    if rc == _lib.SIMSD_ERR_UNSUPPORTED:
        return thin_linear(x2, w, bias).argmax(-1).view(lead)
    _lib.check(rc, "thin_linear_argmax")
    return idx.view(lead)


def thin_linear_cat(x: torch.Tensor, weights, whole: bool = False):
    """[F.linear(x, w) for w in weights] (up to three weights of the same K) from
    one launch, as views into one [..., sum N] output — the merged q/k/v
    projection without concatenating the weights.  Falls back to one
    thin_linear per weight when the kernel cannot take the request (M > 64,
    fp32, a part other than the last not a multiple of 128 rows, odd layouts).
    `whole=True` returns the concatenated [..., sum N] output instead.
    """
    ws_ = list(weights)
    if torch.is_grad_enabled() and (x.requires_grad or any(w.requires_grad for w in ws_)):
        raise RuntimeError("thin_linear_cat is a forward-only inference kernel.")
    if not 1 <= len(ws_) <= 3:
        raise ValueError("one to three weights")
    K = x.shape[-1]
    for w in ws_:
        if w.dtype != x.dtype:
            raise TypeError(f"dtype mismatch: x={x.dtype} w={w.dtype}")
        if w.ndim != 2 or w.shape[1] != K:
            raise ValueError(f"K mismatch: x[..., {K}] vs w{tuple(w.shape)}")
    dev = _lib.require_cuda(x, *ws_)
    lead = x.shape[:-1]
    M = 1
    for d in lead:
        M *= d
    ns = [w.shape[0] for w in ws_]
    y = torch.empty((M, sum(ns)), device=dev, dtype=x.dtype)
    rc = _lib.SIMSD_ERR_UNSUPPORTED
    if M > 0 and x.dtype in (torch.bfloat16, torch.float16) and all(w.stride(1) == 1 for w in ws_):
        x2 = x.reshape(M, K)
        P = len(ws_)
        wp = (ctypes.c_void_p * P)(*[w.data_ptr() for w in ws_])
        lw = (ctypes.c_int64 * P)(*[w.stride(0) for w in ws_])
        nn_ = (ctypes.c_int * P)(*ns)
        with _lib.device_guard(dev):
            nbytes = _lib.thin_workspace_size(torch.cuda.current_device(), M, sum(ns), K,
                                              _lib.dtype_code(x.dtype), _lib.EPI_NONE, 0)
            ws = _lib.workspace(dev, nbytes)
            rc = _lib.lib().simsd_thin_linear_cat(
                x2.data_ptr(), x2.stride(0), x2.stride(1), P, wp, lw, nn_, y.data_ptr(), y.stride(0), M, K,
                _lib.dtype_code(x.dtype), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    outs, off = [], 0
    if rc == _lib.SIMSD_ERR_UNSUPPORTED:
        for w in ws_:
            outs.append(thin_linear(x, w))
        return torch.cat(outs, -1) if whole else outs
    _lib.check(rc, "thin_linear_cat")
    if whole:
        return y.view(*lead, sum(ns))
    for n in ns:
        outs.append(y[:, off:off + n].view(*lead, n))
        off += n
    return outs


def should_fuse(M: int, N: int, K: int) -> bool:
    """Route this call to the thin kernel (True) or to cuBLAS `F.linear` (False).

    The kernel streams the weight once per 256 activation rows and is built for
    the decode/verify regime M <= FUSE_MAX_M; prefill-sized M goes to cuBLAS,
    which the reference's guard also does above its searched range
    (kernels/thin_linear_fused.py:348-377).
    """
    return 1 <= M <= FUSE_MAX_M


class ThinLinear(torch.nn.Module):
    """Replacement for one `nn.Linear` whose forward runs on libsimsd_b200.

    The module registers the *same* Parameter objects as the linear it
    replaces, so the swap allocates nothing, the optimiser-free inference
    model keeps one copy of every weight, and `state_dict()` has the same keys
    and tensors before and after.  Calls with an activation height inside
    `should_fuse` (or any height when `config` pins a split or `always_fuse`
    is set) take the thin-M kernel; the rest take cuBLAS through `F.linear`.
    """

    def __init__(self, linear: torch.nn.Linear,
                 config: tuple[int, int, int, int] | None = None,
                 always_fuse: bool = False):
        super().__init__()
        self.in_features, self.out_features = linear.in_features, linear.out_features
        self.weight, self.bias = linear.weight, linear.bias
        self.config, self.always_fuse = config, always_fuse

    def _thin(self, x: torch.Tensor) -> bool:
        if self.config is not None or self.always_fuse:
            return True
        rows = x.numel() // x.shape[-1] if x.shape[-1] else 0
        return should_fuse(rows, self.out_features, self.in_features)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self._thin(x):
            return thin_linear(x, self.weight, self.bias, config=self.config)
        return torch.nn.functional.linear(x, self.weight, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, fused=tcgen05 thin GEMM "
                f"(M<={FUSE_MAX_M} unless always_fuse)")


def make_bench_fn(x, pool, sh):
    """Timing hook taking (activations, weight pool, shape); the returned
    callable's i-th call multiplies by pool[i], so a pool larger than L2 makes
    every call stream its weight from HBM.  `sh` is unused here."""
    def call(i):
        return thin_linear(x, pool[i])
    return call
