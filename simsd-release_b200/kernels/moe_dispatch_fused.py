"""Fused MoE expert dispatch on B200, CUDA-graph capturable.

Mirrors kernels/moe_dispatch_fused.py of the reference (`moe_dispatch`
:165-192, `_align` :93-132, `_num_tiles` :135-137, `stack_expert_weights`
:195-217, `FusedMoEDispatch` :220-231) and adds the on-GPU router that feeds it
(`moe_route`) plus a whole-layer helper (`moe_layer`: router + routed experts +
shared expert).

One `moe_dispatch` call is five launches on the current stream, none of which
syncs with the host:
  align   (1 CTA) counts, offsets and the stable slot permutation;
  gather  token rows into expert order;
  gate/up grouped tcgen05 GEMM with the SiLU*mul epilogue (both weights read
          once per active expert, fp32 until the single rounding);
  down    grouped tcgen05 GEMM;
  combine fp32 weighted sum over the k experts of each token.
Every buffer size depends only on (T, k, E, H, I); only the values depend on
the routing, so the call can be captured once and replayed.  fp32 inputs and
shapes below one 64-wide K block use the CUDA-core grouped kernel instead.
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib

# Row padding of the reference's slot layout (`slots` / `tile_expert`).
BLOCK_M = 16


def _num_tiles(M: int, E: int) -> int:
    """Worst-case tile count of the reference layout: every active group costs >= 1 tile."""
    return min(E, M) + (M + BLOCK_M - 1) // BLOCK_M


def _err_ptr(dev: torch.device) -> int:
    ws = _lib.workspace(dev, _lib.lib().simsd_workspace_header_bytes())
    return ws.data_ptr() + _lib.lib().simsd_workspace_header_bytes() - 64


def align(topk_ids: torch.Tensor, E: int, block_m: int = BLOCK_M, num_tiles: int | None = None,
          reference_layout: bool = True) -> dict[str, torch.Tensor]:
    """Expert counts, offsets and the stable slot permutation of `topk_ids` [T, k].

    Returns int32 tensors: counts [E], offsets [E+1], sorted_slots [T*k]
    (== argsort(ids.flatten(), stable=True)), slot_to_row [T*k] (its inverse),
    and, with `reference_layout`, the reference's padded `slots`
    [num_tiles*block_m] (-1 = padding) and `tile_expert` [num_tiles].
    """
    if topk_ids.dtype != torch.int64:
        raise TypeError(f"topk_ids must be int64, got {topk_ids.dtype}")
    dev = _lib.require_cuda(topk_ids)
    flat = topk_ids.reshape(-1).contiguous()
    S = flat.numel()
    if num_tiles is None:
        num_tiles = min(E, S) + (S + block_m - 1) // block_m
    i32 = dict(dtype=torch.int32, device=dev)
    out = {
        "counts": torch.empty(E, **i32),
        "offsets": torch.empty(E + 1, **i32),
        "sorted_slots": torch.empty(S, **i32),
        "slot_to_row": torch.empty(S, **i32),
    }
    if reference_layout:
        out["slots"] = torch.empty(num_tiles * block_m, **i32)
        out["tile_expert"] = torch.empty(num_tiles, **i32)
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_moe_align(
            flat.data_ptr(), S, E, out["counts"].data_ptr(), out["offsets"].data_ptr(),
            out["sorted_slots"].data_ptr(), out["slot_to_row"].data_ptr(), block_m, num_tiles,
            out["slots"].data_ptr() if reference_layout else None,
            out["tile_expert"].data_ptr() if reference_layout else None,
            _err_ptr(dev), _lib.stream_ptr(dev))
    _lib.check(rc, "moe align")
    return out


def _align(topk_ids: torch.Tensor, E: int, num_tiles: int):
    """Reference-layout (slots, tile_expert), as kernels/moe_dispatch_fused.py:93-132 returns."""
    a = align(topk_ids, E, BLOCK_M, num_tiles, reference_layout=True)
    return a["slots"], a["tile_expert"]


def moe_route(x: torch.Tensor, w_router: torch.Tensor, bias: torch.Tensor | None = None,
              k: int = 8, renorm: bool = True, scale: float = 1.0,
              return_logits: bool = False, extra_expert: int | None = None):
    """Top-k sigmoid router: (topk_ids [T,k] int64, topk_weight [T,k] fp32[, logits [T,E] fp32]).

    score = sigmoid(x . w_router^T) in fp32; experts chosen by score + bias
    (ties to the lower id); weights = chosen scores, renormalised (+1e-20) when
    `renorm` and k > 1, then times `scale` (the routed scaling factor).
    `extra_expert` (an id): a (k+1)-th column of that id with weight 1 is
    appended to every row (the always-on shared expert of moe_layer).
    """
    if x.ndim != 2 or w_router.ndim != 2 or x.shape[1] != w_router.shape[1]:
        raise ValueError(f"x [T,H] and w_router [E,H] expected, got {tuple(x.shape)} / {tuple(w_router.shape)}")
    T, H = x.shape
    E = w_router.shape[0]
    if not 1 <= k <= min(E, 32):
        raise ValueError(f"k must be in [1, min(E, 32)], got {k}")
    if bias is not None:
        if bias.shape != (E,):
            raise ValueError(f"bias must be [{E}]")
        bias = bias.to(torch.float32).contiguous()
    dev = _lib.require_cuda(x, w_router, bias)
    if x.stride(1) != 1:
        x = x.contiguous()
    if w_router.stride(1) != 1:
        w_router = w_router.contiguous()
    kc = k + (1 if extra_expert is not None else 0)
    ids = torch.empty((T, kc), dtype=torch.int64, device=dev)
    wts = torch.empty((T, kc), dtype=torch.float32, device=dev)
    # always handed to the library: with few tokens it splits the experts over
    # blocks and passes the logits through this buffer to its top-k kernel
    logits = torch.empty((T, E), dtype=torch.float32, device=dev)
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_moe_route_ex(
            x.data_ptr(), x.stride(0), _lib.dtype_code(x.dtype),
            w_router.data_ptr(), w_router.stride(0), _lib.dtype_code(w_router.dtype),
            bias.data_ptr() if bias is not None else None, T, H, E, k, int(bool(renorm)),
            ctypes.c_float(scale), ids.data_ptr(), wts.data_ptr(), kc,
            -1 if extra_expert is None else int(extra_expert), logits.data_ptr(), _lib.stream_ptr(dev))
    _lib.check(rc, "moe_route")
    return (ids, wts, logits) if return_logits else (ids, wts)


def moe_dispatch(x, topk_ids, topk_weight, w_gate, w_up, w_down, add=None, shared_last: bool = False,
                 size_classes: bool = False):
    """Drop-in for ``LLaDA2MoeSparseMoeBlock.moe_infer`` on stacked weights.

    x (T, H); topk_ids (T, k) int64; topk_weight (T, k) fp32;
    w_gate/w_up (E, I, H); w_down (E, H, I) -> (T, H) in x.dtype.
    `add` (T, H), optional: added in x.dtype after the combine (shared expert).
    `shared_last`: the last column of topk_ids names a shared expert stacked
    with the routed ones (moe_route(..., extra_expert=E)); its output is added
    unweighted after the routed sum is rounded, as `add` would be, but it runs
    inside the same grouped GEMMs.
    `size_classes`: for skewed routing (a few experts take most tokens), each
    grouped GEMM runs twice, the experts that outgrow the planned tile height
    with 256-row tiles (SIMSD_LAUNCH_MOE_SIZE_CLASSES).
    """
    if x.ndim != 2 or topk_ids.ndim != 2 or topk_weight.shape != topk_ids.shape:
        raise ValueError("x (T,H), topk_ids (T,k) and topk_weight (T,k) expected")
    if topk_ids.dtype != torch.int64:
        raise TypeError(f"topk_ids must be int64, got {topk_ids.dtype}")
    if topk_weight.dtype != torch.float32:
        raise TypeError(f"topk_weight must be float32, got {topk_weight.dtype}")
    if not (x.dtype == w_gate.dtype == w_up.dtype == w_down.dtype):
        raise TypeError("x and the expert weights must share a dtype")
    T, H = x.shape
    k = topk_ids.shape[1]
    E, I, H2 = w_gate.shape
    if H2 != H or w_up.shape != w_gate.shape or tuple(w_down.shape) != (E, H, I):
        raise ValueError(f"w_gate/w_up (E,I,H) and w_down (E,H,I) expected; got "
                         f"{tuple(w_gate.shape)} {tuple(w_up.shape)} {tuple(w_down.shape)}")
    if topk_ids.shape[0] != T:
        raise ValueError("topk_ids rows must equal x rows")
    if torch.is_grad_enabled() and any(t.requires_grad for t in (x, w_gate, w_up, w_down)):
        raise RuntimeError("moe_dispatch is a forward-only inference kernel.")
    dev = _lib.require_cuda(x, topk_ids, topk_weight, w_gate, w_up, w_down, add)
    code = _lib.dtype_code(x.dtype)
    if x.stride(1) != 1:
        x = x.contiguous()
    if w_gate.stride(2) != 1 or w_up.stride() != w_gate.stride():
        w_gate, w_up = w_gate.contiguous(), w_up.contiguous()
    if w_down.stride(2) != 1:
        w_down = w_down.contiguous()
    ids = topk_ids.contiguous()
    wts = topk_weight.contiguous()
    out = torch.empty((T, H), dtype=x.dtype, device=dev)
    if T == 0:
        return out
    if add is not None:
        if add.shape != (T, H) or add.dtype != x.dtype:
            raise ValueError("add must be (T, H) in x.dtype")
        if add.stride(1) != 1:
            add = add.contiguous()
    L = _lib.lib()
    if size_classes:
        with _lib.moe_size_classes(True):
            return moe_dispatch(x, topk_ids, topk_weight, w_gate, w_up, w_down, add, shared_last)
    if shared_last:
        if add is not None or k < 2:
            raise ValueError("shared_last takes no `add` and needs at least one routed column")
        with _lib.device_guard(dev):
            ws = _lib.workspace(dev, L.simsd_moe_workspace_size(T, k, E, H, I, code))
            rc = L.simsd_moe_dispatch_shared_last(
                x.data_ptr(), x.stride(0), ids.data_ptr(), wts.data_ptr(),
                w_gate.data_ptr(), w_up.data_ptr(), w_gate.stride(0), w_gate.stride(1),
                w_down.data_ptr(), w_down.stride(0), w_down.stride(1), out.data_ptr(), out.stride(0),
                T, k, E, H, I, code, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        _lib.check(rc, "moe_dispatch")
        return out
    with _lib.device_guard(dev):
        nbytes = L.simsd_moe_workspace_size(T, k, E, H, I, code)
        ws = _lib.workspace(dev, nbytes)
        rc = L.simsd_moe_dispatch(
            x.data_ptr(), x.stride(0), ids.data_ptr(), wts.data_ptr(),
            w_gate.data_ptr(), w_up.data_ptr(), w_gate.stride(0), w_gate.stride(1),
            w_down.data_ptr(), w_down.stride(0), w_down.stride(1),
            out.data_ptr(), out.stride(0),
            add.data_ptr() if add is not None else None, add.stride(0) if add is not None else 0,
            T, k, E, H, I, code, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "moe_dispatch")
    return out


def stack_shared_expert(w_gate, w_up, w_down, shared: tuple):
    """The routed experts' stacked weights with the shared expert (w_gate_s,
    w_up_s, w_down_s) appended as expert E (a copy, made once at install time),
    for moe_layer(..., shared_stacked=True)."""
    sg, su, sd = shared
    return (torch.cat([w_gate, sg[None]]), torch.cat([w_up, su[None]]), torch.cat([w_down, sd[None]]))


def moe_layer(x, w_router, router_bias, k, w_gate, w_up, w_down,
              shared: tuple | None = None, renorm: bool = True, scale: float = 1.0,
              shared_stacked: bool = False, size_classes: bool = False):
    """Router + routed experts + optional shared expert (w_gate_s, w_up_s, w_down_s).

    The shared expert is the dense SwiGLU `down(silu(gate(x)) * up(x))`, run as
    two thin-linear launches; its output is added to the routed output in x.dtype.
    It does not depend on the routing, so it runs on a side stream while the
    router runs on the caller's stream (the router's kernels use a few SMs; the
    shared expert's weight stream fills the rest); the caller's stream waits
    for it before the dispatch.  Both orders of work are graph-capturable.
    """
    from .thin_linear_fused import thin_linear, thin_linear_silu_mul
    if shared_stacked:
        # the shared expert is expert E of the stacked weights (stack_shared_expert):
        # the router adds it as an always-on last column and it runs in the
        # dispatch's grouped GEMMs with the routed experts
        E = w_router.shape[0]
        if w_gate.shape[0] != E + 1:
            raise ValueError(f"shared_stacked: {E} routed experts + 1 shared expected, got {w_gate.shape[0]}")
        ids, wts = moe_route(x, w_router, router_bias, k=k, renorm=renorm, scale=scale, extra_expert=E)
        return moe_dispatch(x, ids, wts, w_gate, w_up, w_down, shared_last=True, size_classes=size_classes)
    add = None
    if shared is not None:
        sg, su, sd = shared
        main = torch.cuda.current_stream(x.device)
        side = _lib.side_stream(x.device)
        side.wait_stream(main)
        with torch.cuda.stream(side):
            add = thin_linear(thin_linear_silu_mul(x, sg, su), sd)
    ids, wts = moe_route(x, w_router, router_bias, k=k, renorm=renorm, scale=scale)
    if add is not None:
        main.wait_stream(side)
        add.record_stream(main)
    return moe_dispatch(x, ids, wts, w_gate, w_up, w_down, add=add, size_classes=size_classes)


def stack_expert_weights(experts, free_originals: bool = True):
    """(E,I,H), (E,I,H), (E,H,I) stacked from per-expert gate/up/down Linears.

    One projection at a time; with `free_originals` each expert's weight is
    released as soon as its projection is stacked, so the extra memory peaks at
    one projection of the layer.  Destructive: the per-expert modules cannot run
    afterwards (as in the reference, kernels/moe_dispatch_fused.py:195-217).
    """
    out = []
    for name in ("gate_proj", "up_proj", "down_proj"):
        mats = [getattr(e, name).weight.data for e in experts]
        stacked = torch.stack(mats).contiguous()
        del mats
        if free_originals:
            for e in experts:
                getattr(e, name).weight.data = stacked.new_empty(0)
        out.append(stacked)
    return tuple(out)


class FusedMoEDispatch(torch.nn.Module):
    """Holds one layer's stacked expert weights (non-persistent buffers, so
    checkpoints are unaffected) and applies `moe_dispatch` with them to the
    routing it is given."""

    def __init__(self, w_gate, w_up, w_down):
        super().__init__()
        for name, t in (("w_gate", w_gate), ("w_up", w_up), ("w_down", w_down)):
            self.register_buffer(name, t, persistent=False)

    def forward(self, x, topk_ids, topk_weight):
        packed = (self.w_gate, self.w_up, self.w_down)
        return moe_dispatch(x, topk_ids, topk_weight, *packed)
