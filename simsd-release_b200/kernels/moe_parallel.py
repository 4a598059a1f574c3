"""Expert-parallel MoE layer over a process group.

E experts are split over the g ranks of a group in contiguous blocks (rank r
holds experts [r E/g, (r+1) E/g)); every rank owns T_r tokens.  One layer:

1. route the owned tokens (simsd_moe_route: sigmoid + bias top-k, renormalised);
2. plan per-peer buckets of fixed capacity (simsd_moe_ep_plan): slot s = t*k + j
   goes to the rank holding its expert, in slot order;
3. gather the slots' token rows into the send buffer [g * capacity, H]
   (simsd_moe_gather_rows) and exchange rows and local expert ids with
   all_to_all_single (NCCL over NVLink on GPUs);
4. run the received rows through the local experts: simsd_moe_dispatch with
   k = 1 and weight 1 (so each row comes back as its expert's bf16 output, the
   same rounding the single-GPU path applies before its weighted sum), empty
   bucket entries carrying expert id -1;
5. return the rows with a second all_to_all_single and combine them on the
   owner (simsd_moe_combine): out[t] = cast(sum_j fp32(y[t, j]) * w[t, j]) in j
   order, plus the shared expert (computed data-parallel on the owner).

With a PeerExchange, steps 3 and 5 are plain NVLink peer stores of the
occupied bucket entries only (simsd_moe_ep_send / simsd_moe_ep_return), each
followed by a sync point, instead of all-to-alls of the whole fixed-capacity
buckets.  Fixed capacities make the exchange shape static, so the whole layer
can be captured in a CUDA graph.  The default capacity T_r * k never drops a slot; a
smaller one may, which raises SIMSD_DEV_ERR_CAPACITY in the device error word.
The reference runs its MoE layer on one GPU (kernels/moe_dispatch_fused.py,
moe_infer's per-expert loop); this layer reproduces that computation's
routing and combine order across ranks.

`ep_moe_layer(..., ops=...)` takes the five compute steps as an object so the
collective plumbing can be exercised with CPU stand-ins under gloo; the default
ops are the CUDA kernels (no CPU fallback).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .moe_dispatch_fused import _err_ptr, moe_dispatch, moe_route
from .thin_linear_fused import thin_linear, thin_linear_silu_mul


def expert_range(E: int, rank: int, world: int) -> tuple[int, int]:
    """Experts [lo, hi) held by `rank`."""
    if E % world != 0:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    per = E // world
    return rank * per, (rank + 1) * per


def ep_plan(topk_ids: torch.Tensor, E: int, world: int, capacity: int) -> dict[str, torch.Tensor]:
    """Per-peer buckets of this rank's slots (see simsd_moe_ep_plan).

    Returns int32 tensors send_slot [world*capacity], send_expert
    [world*capacity] (local expert id on the peer, -1 = empty), slot_pos
    [T*k] (bucket position of each slot, -1 = not sent) and counts [world].
    """
    if topk_ids.dtype != torch.int64:
        raise TypeError(f"topk_ids must be int64, got {topk_ids.dtype}")
    expert_range(E, 0, world)
    dev = _lib.require_cuda(topk_ids)
    flat = topk_ids.reshape(-1).contiguous()
    i32 = dict(dtype=torch.int32, device=dev)
    out = {"send_slot": torch.empty(world * capacity, **i32), "send_expert": torch.empty(world * capacity, **i32),
           "slot_pos": torch.empty(flat.numel(), **i32), "counts": torch.empty(world, **i32)}
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_moe_ep_plan(
            flat.data_ptr(), flat.numel(), E, world, capacity, out["send_slot"].data_ptr(),
            out["send_expert"].data_ptr(), out["slot_pos"].data_ptr(), out["counts"].data_ptr(), _err_ptr(dev),
            _lib.stream_ptr(dev))
    _lib.check(rc, "moe_ep_plan")
    return out


def gather_rows(x: torch.Tensor, slots: torch.Tensor, k: int) -> torch.Tensor:
    """[R, H] with row r = x[slots[r] // k]; rows of negative slots are left unset."""
    dev = _lib.require_cuda(x, slots)
    if slots.dtype != torch.int32:
        raise TypeError("slots must be int32")
    if x.stride(-1) != 1:
        x = x.contiguous()
    R, H = slots.numel(), x.shape[-1]
    out = torch.empty((R, H), dtype=x.dtype, device=dev)
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_moe_gather_rows(x.data_ptr(), x.stride(0), slots.data_ptr(), R, k, H,
                                              _lib.dtype_code(x.dtype), out.data_ptr(), out.stride(0),
                                              _lib.stream_ptr(dev))
    _lib.check(rc, "moe_gather_rows")
    return out


def combine(ys: torch.Tensor, slot_row: torch.Tensor, topk_weight: torch.Tensor,
            add: torch.Tensor | None = None) -> torch.Tensor:
    """out[t] = cast(sum_j fp32(ys[slot_row[t*k+j]]) * w[t, j]) (+ add), j in order."""
    dev = _lib.require_cuda(ys, slot_row, topk_weight, add)
    T, k = topk_weight.shape
    H = ys.shape[-1]
    w = topk_weight.contiguous()
    rows = slot_row.reshape(-1).contiguous()
    out = torch.empty((T, H), dtype=ys.dtype, device=dev)
    if add is not None and add.stride(-1) != 1:
        add = add.contiguous()
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_moe_combine(ys.data_ptr(), ys.stride(0), rows.data_ptr(), w.data_ptr(), out.data_ptr(),
                                          out.stride(0), add.data_ptr() if add is not None else None,
                                          add.stride(0) if add is not None else 0, T, k, H,
                                          _lib.dtype_code(ys.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "moe_combine")
    return out


_ONES: dict[tuple, torch.Tensor] = {}


def _ones(n: int, dev: torch.device) -> torch.Tensor:
    t = _ONES.get((n, dev))
    if t is None:
        t = _ONES[(n, dev)] = torch.ones((n, 1), dtype=torch.float32, device=dev)
    return t


class CudaOps:
    """The layer's compute steps on the CUDA kernels of libsimsd_b200."""

    @staticmethod
    def route(x, w_router, bias, k, renorm, scale):
        return moe_route(x, w_router, bias, k=k, renorm=renorm, scale=scale)

    @staticmethod
    def plan(ids, E, world, capacity):
        return ep_plan(ids, E, world, capacity)

    @staticmethod
    def gather(x, slots, k):
        return gather_rows(x, slots, k)

    @staticmethod
    def experts(rows, expert_ids, w_gate, w_up, w_down):
        ids = expert_ids.to(torch.int64).reshape(-1, 1)
        return moe_dispatch(rows, ids, _ones(ids.shape[0], rows.device), w_gate, w_up, w_down)

    @staticmethod
    def combine(ys, slot_pos, w, add):
        return combine(ys, slot_pos, w, add)

    @staticmethod
    def shared(x, w_gate, w_up, w_down):
        return thin_linear(thin_linear_silu_mul(x, w_gate, w_up), w_down)


class PeerExchange:
    """The layer's two exchanges as NVLink peer stores (simsd_moe_ep_send /
    simsd_moe_ep_return) instead of all-to-alls of the fixed-capacity buckets.

    Every rank maps every rank's row, id and return blocks ([world * capacity]
    entries, cudaIpc mappings): a send stores each occupied bucket entry's
    token row straight from x into the receiving rank's row block (no send
    buffer) and every entry's expert id into its id block; a return stores
    each received row's expert output back into its owner's return block.  A
    sync point (simsd_allgather_wait on this object's signal block) follows
    each, so only occupied entries cross NVLink and the layer stays capturable
    (no sizes reach the host).  The blocks are reused by every call: a call's
    sends overwrite rows the ranks read in the previous call only after every
    rank has passed that call's second sync point, which it reaches only after
    its reads.  Collective: every rank constructs it with the same capacity,
    and every rank calls `send` and `give_back` at the same points.
    """

    def __init__(self, capacity: int, H: int, dtype: torch.dtype = torch.bfloat16, group=None):
        from .parallel import SymmetricBlock, _group_info
        self.rank, self.world = _group_info(group)
        self.cap, self.H, self.dtype = capacity, H, dtype
        n = self.world * capacity
        esz = torch.empty((), dtype=dtype).element_size()
        self.rows = SymmetricBlock(n * H * esz, group)
        self.back = SymmetricBlock(n * H * esz, group)
        self.ids = SymmetricBlock(n * 4, group)
        self.sig = SymmetricBlock(_lib.SIGNAL_BYTES, group)
        arr = lambda blk: (ctypes.c_void_p * self.world)(*blk.ptrs)
        self._rows, self._back, self._ids, self._sig = arr(self.rows), arr(self.back), arr(self.ids), arr(self.sig)
        self.recv = self.rows.tensor.view(dtype).view(n, H)
        self.recv_expert = self.ids.tensor.view(torch.int32)[:n]
        self.returned = self.back.tensor.view(dtype).view(n, H)

    def _sync(self, dev) -> None:
        ws = _lib.workspace(dev, _lib.lib().simsd_workspace_header_bytes())
        _lib.check(_lib.lib().simsd_allgather_wait(self._sig, self.rank, self.world, ws.data_ptr(), ws.numel(),
                                                   _lib.stream_ptr(dev)), "moe_ep sync")

    def send(self, x: torch.Tensor, plan: dict, k: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Rows and local expert ids of every rank's buckets for this rank:
        views [world * capacity, H] and [world * capacity] of this rank's blocks."""
        dev = _lib.require_cuda(x)
        if x.stride(-1) != 1:
            x = x.contiguous()
        with _lib.device_guard(dev):
            _lib.check(_lib.lib().simsd_moe_ep_send(
                x.data_ptr(), x.stride(0), plan["send_slot"].data_ptr(), plan["send_expert"].data_ptr(), k,
                self.H, self.cap, self.rank, self.world, self._rows, self._ids, _lib.dtype_code(x.dtype),
                _lib.stream_ptr(dev)), "moe_ep_send")
            self._sync(dev)
        return self.recv, self.recv_expert

    def give_back(self, y: torch.Tensor) -> torch.Tensor:
        """Expert outputs of this rank's sent slots, laid out as the buckets
        (view [world * capacity, H] of this rank's return block)."""
        dev = _lib.require_cuda(y)
        with _lib.device_guard(dev):
            _lib.check(_lib.lib().simsd_moe_ep_return(
                y.data_ptr(), y.stride(0), self.recv_expert.data_ptr(), self.H, self.cap, self.rank, self.world,
                self._back, _lib.dtype_code(y.dtype), _lib.stream_ptr(dev)), "moe_ep_return")
            self._sync(dev)
        return self.returned

    def close(self) -> None:
        for blk in (self.rows, self.back, self.ids, self.sig):
            blk.close()


def ep_moe_layer(x: torch.Tensor, w_router: torch.Tensor, router_bias: torch.Tensor | None, k: int,
                 w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor, E: int, group=None,
                 capacity: int | None = None, shared: tuple | None = None, renorm: bool = True,
                 scale: float = 1.0, ops=CudaOps, size_classes: bool = False,
                 exchange: PeerExchange | None = None) -> torch.Tensor:
    """One expert-parallel MoE layer for this rank's tokens x [T_r, H].

    w_gate, w_up [E/g, I, H] and w_down [E/g, H, I] are this rank's experts;
    w_router [E, H] and router_bias [E] are replicated.  `capacity` (rows per
    peer bucket) must be the same on every rank; default T_r * k.
    `size_classes`: as moe_dispatch's, for skewed routing.  `exchange`: a
    PeerExchange of this capacity and H (NVLink peer stores); without it the
    buckets cross with all_to_all_single.
    """
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = expert_range(E, rank, world)
    if w_gate.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds experts [{lo}, {hi}) but got {w_gate.shape[0]} gate matrices")
    T, H = x.shape
    cap = capacity if capacity is not None else T * k
    ids, w = ops.route(x, w_router, router_bias, k, renorm, scale)
    plan = ops.plan(ids, E, world, cap)
    if exchange is not None:
        if exchange.cap != cap or exchange.H != H or exchange.world != world:
            raise ValueError(f"exchange holds {exchange.world} x {exchange.cap} rows of {exchange.H}; "
                             f"this layer needs {world} x {cap} rows of {H}")
        recv, recv_e = exchange.send(x, plan, k)
    else:
        send = ops.gather(x, plan["send_slot"], k)
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=group)
        recv_e = torch.empty_like(plan["send_expert"])
        dist.all_to_all_single(recv_e, plan["send_expert"], group=group)
    if size_classes:
        from . import _lib
        with _lib.moe_size_classes(True):
            y = ops.experts(recv, recv_e, w_gate, w_up, w_down)
    else:
        y = ops.experts(recv, recv_e, w_gate, w_up, w_down)
    if exchange is not None:
        back = exchange.give_back(y)
    else:
        back = torch.empty_like(y)
        dist.all_to_all_single(back, y, group=group)
    add = ops.shared(x, *shared) if shared is not None else None
    return ops.combine(back, plan["slot_pos"], w, add)
