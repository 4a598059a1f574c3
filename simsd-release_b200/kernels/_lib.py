"""ctypes binding of libsimsd_b200.so (the C ABI in include/simsd_b200.h).

This module is the only place that touches the shared library.  It has no CPU
fallback: if the library is missing, every operator raises.  Workspaces are
cached per device and reused serially, like the reference's split-K staging
buffer (kernels/thin_linear_fused.py:173-190); `reset_workspace()` drops them
(call it before re-capturing graphs into a new memory pool).
"""
from __future__ import annotations

import contextlib
import ctypes
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libsimsd_b200.so")

SIMSD_OK = 0
SIMSD_ERR_SHAPE = -1
SIMSD_ERR_DTYPE = -2
SIMSD_ERR_WORKSPACE = -3
SIMSD_ERR_LAUNCH = -4
SIMSD_ERR_ALIGN = -5
SIMSD_ERR_DEVICE = -6
SIMSD_ERR_UNSUPPORTED = -7
SIMSD_ERR_SCRATCH_LIMIT = -8

SIMSD_BF16, SIMSD_F16, SIMSD_F32 = 0, 1, 2
EPI_NONE, EPI_SILU_MUL = 0, 1
PATH_AUTO, PATH_TC, PATH_SIMT = 0, 1, 2

LAUNCH_PDL = 1
LAUNCH_INKERNEL_REDUCE = 2
LAUNCH_GROUPED_FIXUP = 4
LAUNCH_MOE_SIZE_CLASSES = 8
IPC_HANDLE_BYTES = 64
SIGNAL_BYTES = 256

DEV_ERR_TIMEOUT = 1
DEV_ERR_BAD_INDEX = 2
DEV_ERR_CAPACITY = 4

_DTYPE = {torch.bfloat16: SIMSD_BF16, torch.float16: SIMSD_F16, torch.float32: SIMSD_F32}

# name -> (restype, argtypes); every symbol include/simsd_b200.h declares
_P, _I, _L, _S, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_size_t, ctypes.c_float
SIGNATURES: dict[str, tuple] = {
    "simsd_version": (ctypes.c_char_p, []),
    "simsd_status_string": (ctypes.c_char_p, [_I]),
    "simsd_device_sm_count": (_I, []),
    "simsd_set_launch_flags": (_I, [_I]),
    "simsd_get_launch_flags": (_I, []),
    "simsd_debug_cluster_plan": (_I, [_I, _I, _I, _I, _P, _P, _P]),
    "simsd_debug_set_trace": (_I, [_P, _S]),
    "simsd_workspace_header_bytes": (_S, []),
    "simsd_workspace_init": (_I, [_P, _S, _P]),
    "simsd_workspace_error": (_I, [_P, _P, ctypes.POINTER(_I)]),
    "simsd_thin_linear_workspace_size": (_S, [_I, _I, _I, _I, _I, _I]),
    "simsd_thin_linear": (_I, [_P, _L, _L, _P, _L, _L, _P, _P, _P, _L, _I, _I, _I, _I, _I, _I, _I,
                               _P, _S, _P]),
    "simsd_thin_linear_noalloc": (_I, [_P, _L, _L, _P, _L, _L, _P, _P, _P, _L, _I, _I, _I, _I, _I, _P]),
    "simsd_thin_linear_noalloc_error": (_I, [_P, ctypes.POINTER(_I)]),
    "simsd_moe_route_ex": (_I, [_P, _L, _I, _P, _L, _I, _P, _I, _I, _I, _I, _I, _F, _P, _P, _L, _I, _P, _P]),
    "simsd_moe_route": (_I, [_P, _L, _I, _P, _L, _I, _P, _I, _I, _I, _I, _I, _F, _P, _P, _P, _P]),
    "simsd_moe_align": (_I, [_P, _I, _I, _P, _P, _P, _P, _I, _I, _P, _P, _P, _P]),
    "simsd_moe_workspace_size": (_S, [_I, _I, _I, _I, _I, _I]),
    "simsd_moe_dispatch_shared_last": (_I, [_P, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _L, _I, _I, _I, _I, _I, _I, _P, _S, _P]),
    "simsd_moe_dispatch": (_I, [_P, _L, _P, _P, _P, _P, _L, _L, _P, _L, _L, _P, _L, _P, _L, _I, _I,
                                _I, _I, _I, _I, _P, _S, _P]),
    "simsd_ipc_alloc": (_I, [_S, ctypes.POINTER(_P)]),
    "simsd_ipc_free": (_I, [_P]),
    "simsd_ipc_handle": (_I, [_P, _P]),
    "simsd_ipc_open": (_I, [_P, ctypes.POINTER(_P)]),
    "simsd_ipc_close": (_I, [_P]),
    "simsd_thin_linear_argmax": (_I, [_P, _L, _L, _P, _L, _L, _P, _P, _I, _I, _I, _I, _P, _S, _P]),
    "simsd_thin_linear_cat": (_I, [_P, _L, _L, _I, _P, _P, _P, _P, _L, _I, _I, _I, _P, _S, _P]),
    "simsd_rmsnorm": (_I, [_P, _L, _P, _L, _P, _L, _P, _P, _L, _I, _I, _F, _I, _P]),
    "simsd_qk_norm_rope": (_I, [_P, _L, _I, _I, _I, _I, _P, _P, _P, _P, _F, _P, _P, _P, _L, _I, _I, _P]),
    "simsd_verify_attention_workspace_size": (_S, [_I, _I, _I, _I]),
    "simsd_verify_attention": (_I, [_P, _P, _P, _L, _I, _I, _I, _I, _P, _L, _F, _P, _I, _P, _S, _P]),
    "simsd_allgather_wait": (_I, [_P, _I, _I, _P, _S, _P]),
    "simsd_thin_linear_allgather": (_I, [_P, _L, _L, _P, _L, _L, _P, _P, _P, _L, _I, _I, _I, _I, _I, _I, _I, _I,
                                         _I, _P, _S, _P]),
    "simsd_moe_ep_plan": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _P, _P, _P]),
    "simsd_moe_gather_rows": (_I, [_P, _L, _P, _I, _I, _I, _I, _P, _L, _P]),
    "simsd_moe_combine": (_I, [_P, _L, _P, _P, _P, _L, _P, _L, _I, _I, _I, _I, _P]),
    "simsd_moe_ep_send": (_I, [_P, _L, _P, _P, _I, _I, _I, _I, _I, _P, _P, _I, _P]),
    "simsd_moe_ep_return": (_I, [_P, _L, _P, _I, _I, _I, _I, _P, _I, _P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """Load libsimsd_b200.so once; raise if it has not been built."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise RuntimeError(
                f"{LIB_PATH.name} is not built; run `python simsd-release_b200/build.py` "
                "(nvcc, sm_100a). There is no CPU fallback.")
        L = ctypes.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}; expected bfloat16, float16 or float32") from None


def check(rc: int, what: str) -> None:
    if rc == SIMSD_OK:
        return
    msg = f"{what}: {lib().simsd_status_string(rc).decode()} (status {rc})"
    if rc == SIMSD_ERR_SHAPE:
        raise ValueError(msg)
    if rc == SIMSD_ERR_DTYPE:
        raise TypeError(msg)
    raise RuntimeError(msg)


def stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


_SIDE_STREAMS: dict[torch.device, torch.cuda.Stream] = {}


def side_stream(dev: torch.device) -> torch.cuda.Stream:
    """A second stream per device for work that overlaps the caller's stream
    (callers order it with wait_stream on both sides)."""
    s = _SIDE_STREAMS.get(dev)
    if s is None:
        s = _SIDE_STREAMS[dev] = torch.cuda.Stream(device=dev)
    return s


def device_guard(dev: torch.device):
    """`torch.cuda.device(dev)` when `dev` is not the current device (tensors of a
    sharded model may live elsewhere); a no-op context otherwise, which keeps the
    common call cheap."""
    if dev.index is None or dev.index == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(dev)


_WS_SIZES: dict[tuple, int] = {}


def thin_workspace_size(dev_index: int, M: int, N: int, K: int, code: int, epilogue: int, split: int) -> int:
    """simsd_thin_linear_workspace_size, memoised (pure arithmetic for a device)."""
    key = (dev_index, M, N, K, code, epilogue, split)
    v = _WS_SIZES.get(key)
    if v is None:
        v = _WS_SIZES[key] = lib().simsd_thin_linear_workspace_size(M, N, K, code, epilogue, split)
    return v


def require_cuda(*tensors: torch.Tensor) -> torch.device:
    dev = tensors[0].device
    if dev.type != "cuda":
        raise RuntimeError(
            "the simsd_b200 operators run on CUDA tensors only (no CPU fallback); "
            f"got a tensor on {dev}")
    for t in tensors[1:]:
        if t is not None and t.device != dev:
            raise RuntimeError(f"all tensors must be on {dev}; got one on {t.device}")
    return dev


# ------------------------------------------------------------------ workspaces
_WORKSPACES: dict[torch.device, torch.Tensor] = {}
# Outgrown workspaces stay alive until reset_workspace(): a CUDA graph captured
# earlier may still hold their addresses.
_RETIRED: list[torch.Tensor] = []


def workspace(dev: torch.device, nbytes: int) -> torch.Tensor:
    """Per-device scratch of at least `nbytes`, header zeroed (grows, never shrinks)."""
    buf = _WORKSPACES.get(dev)
    if buf is None or buf.numel() < nbytes:
        size = max(nbytes, 0 if buf is None else buf.numel())
        size = (size + (1 << 20) - 1) & ~((1 << 20) - 1)
        if buf is not None:
            _RETIRED.append(buf)
        buf = torch.zeros(size, dtype=torch.uint8, device=dev)
        _WORKSPACES[dev] = buf
    return buf


def reset_workspace() -> None:
    """Drop the cached workspaces (call before re-capturing graphs in a new pool)."""
    _WORKSPACES.clear()
    _RETIRED.clear()


def device_error(dev: torch.device | None = None) -> int:
    """OR of the device error bits recorded in `dev`'s workspace (synchronises)."""
    dev = torch.device("cuda", torch.cuda.current_device()) if dev is None else dev
    buf = _WORKSPACES.get(dev)
    if buf is None:
        return 0
    out = ctypes.c_int(0)
    with torch.cuda.device(dev):
        check(lib().simsd_workspace_error(buf.data_ptr(), stream_ptr(dev), ctypes.byref(out)),
              "simsd_workspace_error")
    return out.value


def clear_device_error(dev: torch.device | None = None) -> None:
    """Zero `dev`'s workspace header (error word and tile counters), stream-ordered."""
    dev = torch.device("cuda", torch.cuda.current_device()) if dev is None else dev
    buf = _WORKSPACES.get(dev)
    if buf is None:
        return
    with torch.cuda.device(dev):
        check(lib().simsd_workspace_init(buf.data_ptr(), buf.numel(), stream_ptr(dev)),
              "simsd_workspace_init")


def _set_flag(bit: int, enable: bool) -> bool:
    L = lib()
    old = L.simsd_get_launch_flags()
    L.simsd_set_launch_flags((old | bit) if enable else (old & ~bit))
    return bool(old & bit)


def set_pdl(enable: bool) -> bool:
    """Launch kernels as programmatic dependents (weights must not be written by the
    kernel right before each call on the same stream).  Returns the previous setting."""
    return _set_flag(LAUNCH_PDL, enable)


def set_grouped_fixup(enable: bool) -> bool:
    """MoE grouped GEMMs: sum split tiles in a separate reduction kernel instead of
    inside the GEMM (the default); same bits.  Returns the previous setting."""
    return _set_flag(LAUNCH_GROUPED_FIXUP, enable)


def set_inkernel_reduce(enable: bool) -> bool:
    """Sum split-K tiles inside the GEMM (last contributor) instead of in a separate
    reduction kernel; the bits are the same either way.  Returns the previous setting."""
    return _set_flag(LAUNCH_INKERNEL_REDUCE, enable)


class moe_size_classes:
    """Context manager: MoE dispatches issued (or captured) in its body split
    each grouped GEMM by expert size (SIMSD_LAUNCH_MOE_SIZE_CLASSES)."""

    def __init__(self, enable: bool = True):
        self.enable = enable

    def __enter__(self):
        self.prev = _set_flag(LAUNCH_MOE_SIZE_CLASSES, self.enable)
        return self

    def __exit__(self, *exc):
        _set_flag(LAUNCH_MOE_SIZE_CLASSES, self.prev)
        return False


class weights_static:
    """Context manager enabling programmatic dependent launch for its body."""

    def __init__(self, enable: bool = True):
        self.enable = enable

    def __enter__(self):
        self.prev = set_pdl(self.enable)
        return self

    def __exit__(self, *exc):
        set_pdl(self.prev)
        return False
