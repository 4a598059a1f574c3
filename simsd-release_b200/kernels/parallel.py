"""Thin linears split across GPUs: column-parallel weight shards + all-gather.

The SDAR target verify and draft linears have few activation rows (M = 4..64)
and large weights, so they shard naturally by output column: rank r of a
g-rank group holds rows [r N/g, (r+1) N/g) of each nn.Linear weight (its
output columns), computes its [M, N/g] slice with the thin-M kernel and the
group all-gathers the slices (NCCL over NVLink on GPUs).  For the SwiGLU front
half, gate and up are split at the same rows so SiLU(gate) * up stays local.
No counterpart exists in the reference's kernel package; its TP=2 baselines
shard through transformers' `tp_plan="auto"` (main_table/run_native_tp2_cache.py:96),
whose column-wise plan splits nn.Linear weights the same way.

`gather_columns` and the shard helpers are plain tensor/collective code and
run under any backend (the CPU tests use gloo); the local product is the
CUDA thin-M kernel.
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .thin_linear_fused import thin_linear, thin_linear_silu_mul


def _group_info(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def column_range(n: int, rank: int, world: int) -> tuple[int, int]:
    """Output columns [lo, hi) of `rank` for an n-column linear split `world` ways."""
    if n % world != 0:
        raise ValueError(f"{n} output columns do not split evenly over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def column_shard(w: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """This rank's rows of an nn.Linear weight [N, K] (its output columns), contiguous."""
    lo, hi = column_range(w.shape[0], rank, world)
    return w[lo:hi].contiguous()


def bias_shard(b: torch.Tensor | None, rank: int, world: int) -> torch.Tensor | None:
    if b is None:
        return None
    lo, hi = column_range(b.shape[0], rank, world)
    return b[lo:hi].contiguous()


def gather_columns(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather per-rank column slices [M, n] into the full [M, world * n].

    Rank r's slice lands at columns [r n, (r+1) n), matching `column_shard`.
    One all_gather_into_tensor into [world * M, n], then one transpose copy.
    """
    rank, world = _group_info(group)
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    M, n = y_local.shape
    buf = torch.empty((world * M, n), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local, group=group)
    return buf.view(world, M, n).permute(1, 0, 2).reshape(M, world * n)


class ColumnParallelThinLinear(torch.nn.Module):
    """nn.Linear split by output column over a process group.

    forward(x [..., K]) -> [..., N] on every rank: thin_linear on the local
    shard, then gather_columns.  The shard is a copy of this rank's rows (the
    full weight may be dropped afterwards).
    """

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None = None, group=None):
        super().__init__()
        self.group = group
        rank, world = _group_info(group)
        self.out_features = weight.shape[0]
        self.weight = torch.nn.Parameter(column_shard(weight, rank, world), requires_grad=False)
        b = bias_shard(bias, rank, world)
        self.bias = torch.nn.Parameter(b, requires_grad=False) if b is not None else None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y = thin_linear(x.reshape(-1, x.shape[-1]), self.weight, self.bias)
        return gather_columns(y, self.group).reshape(*lead, self.out_features)


class ColumnParallelGateUp(torch.nn.Module):
    """SiLU(x w_gate^T) * (x w_up^T) with gate and up split at the same rows."""

    def __init__(self, w_gate: torch.Tensor, w_up: torch.Tensor, group=None):
        super().__init__()
        if w_gate.shape != w_up.shape:
            raise ValueError("gate and up weights must have the same shape")
        self.group = group
        rank, world = _group_info(group)
        self.out_features = w_gate.shape[0]
        self.w_gate = torch.nn.Parameter(column_shard(w_gate, rank, world), requires_grad=False)
        self.w_up = torch.nn.Parameter(column_shard(w_up, rank, world), requires_grad=False)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y = thin_linear_silu_mul(x.reshape(-1, x.shape[-1]), self.w_gate, self.w_up)
        return gather_columns(y, self.group).reshape(*lead, self.out_features)


# ------------------------------------------------------------------ fused all-gather
class _CudaArray:
    """A raw device pointer seen by torch through __cuda_array_interface__."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False), "version": 3}


class SymmetricBlock:
    """One device block per rank, mapped into every rank of the group
    (simsd_ipc_alloc / cudaIpc handles exchanged with all_gather_object).
    Collective: every rank constructs it with the same size, in the same order."""

    def __init__(self, nbytes: int, group=None):
        L = _lib.lib()
        self.rank, self.world = _group_info(group)
        own = ctypes.c_void_p()
        _lib.check(L.simsd_ipc_alloc(nbytes, ctypes.byref(own)), "ipc_alloc")
        self.nbytes = nbytes
        self.own = own.value
        handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
        _lib.check(L.simsd_ipc_handle(self.own, handle), "ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, handle.raw, group=group)
        self.ptrs: list[int] = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.own)
            else:
                p = ctypes.c_void_p()
                _lib.check(L.simsd_ipc_open(ctypes.create_string_buffer(h, len(h)), ctypes.byref(p)), "ipc_open")
                self.ptrs.append(p.value)
        self.tensor = torch.as_tensor(_CudaArray(self.own, nbytes), device=f"cuda:{torch.cuda.current_device()}")

    def close(self) -> None:
        if not self.ptrs:
            return
        L = _lib.lib()
        for r, p in enumerate(self.ptrs):
            if r != self.rank:
                L.simsd_ipc_close(p)
        self.ptrs = []
        self.tensor = None
        L.simsd_ipc_free(self.own)


class FusedAllGather:
    """Column-parallel thin linears whose all-gather is fused into the GEMM
    (simsd_thin_linear_allgather): each rank stores its columns straight into
    every rank's output over NVLink.  The launches carry no signal; at a sync
    point (`wait`, simsd_allgather_wait) every rank counts itself on every
    rank's signal block and waits for the others, so ranks only meet where an
    output is actually read, and one sync point covers every launch before it.

    `linear(x, w_local, w_up_local=None, bias_local=None, wait=True)` returns
    the full [M, world * n] output; with `wait=False` the output is complete
    only after a later `wait()` on the same stream (several launches may share
    one wait).  Outputs live in buffers this object owns, two per output shape
    used in turn, so a result stays valid until the second-next call with the
    same shape.  Peers write into them: consume each result before issuing the
    call after next with the same shape, and keep at most one unwaited call
    per shape in flight.  Calls are collective: every rank makes the same
    sequence of calls with the same shapes.  Shapes the fused kernel does not
    take (M > 64, fp32, odd layouts) fall back to thin_linear and
    gather_columns (NCCL), which are complete on return.
    """

    def __init__(self, group=None):
        self.group = group
        self.rank, self.world = _group_info(group)
        self.sig = SymmetricBlock(_lib.SIGNAL_BYTES, group)
        self.outs: dict[tuple, SymmetricBlock] = {}
        self._sig_arr = (ctypes.c_void_p * self.world)(*self.sig.ptrs)
        self._out_arrs: dict[tuple, ctypes.Array] = {}
        self._calls: dict[tuple, int] = {}

    def _out(self, M: int, N: int, dtype: torch.dtype):
        calls = self._calls.get((M, N, dtype), 0)
        self._calls[(M, N, dtype)] = calls + 1
        key = (M, N, dtype, calls & 1)
        blk = self.outs.get(key)
        if blk is None:
            esz = torch.empty((), dtype=dtype).element_size()
            blk = self.outs[key] = SymmetricBlock(M * N * esz, self.group)
            self._out_arrs[key] = (ctypes.c_void_p * self.world)(*blk.ptrs)
        return blk.tensor.view(dtype).view(M, N), self._out_arrs[key]

    def linear(self, x: torch.Tensor, w: torch.Tensor, w_up: torch.Tensor | None = None,
               bias: torch.Tensor | None = None, wait: bool = True, plan_n: int = 0) -> torch.Tensor:
        """`plan_n` > 0 (the unsharded output width): split K exactly as one GPU
        would for that width, so the gathered output is bit-identical to the
        single-GPU thin linear."""
        M, K = x.shape
        n = w.shape[0]
        N = n * self.world
        code = _lib.dtype_code(x.dtype)
        y, peers = self._out(M, N, x.dtype)
        dev = x.device
        ws = _lib.workspace(dev, _lib.lib().simsd_workspace_header_bytes())
        rc = _lib.lib().simsd_thin_linear_allgather(
            x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), w.stride(0), w.stride(1),
            w_up.data_ptr() if w_up is not None else None, bias.data_ptr() if bias is not None else None,
            peers, N, self.rank * n, M, n, K, code, _lib.EPI_SILU_MUL if w_up is not None else _lib.EPI_NONE,
            self.rank, self.world, plan_n, ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
        if rc == _lib.SIMSD_ERR_UNSUPPORTED:
            local = thin_linear_silu_mul(x, w, w_up) if w_up is not None else thin_linear(x, w, bias)
            return gather_columns(local, self.group)
        _lib.check(rc, "thin_linear_allgather")
        if wait:
            self.wait(dev)
        return y

    def wait(self, dev: torch.device | None = None) -> None:
        """Make every fused output issued so far on the current stream complete
        on this rank (one bounded device-side sync point; no host
        synchronisation).  Collective: every rank calls it at the same point
        of the call sequence."""
        dev = dev or torch.device("cuda", torch.cuda.current_device())
        ws = _lib.workspace(dev, _lib.lib().simsd_workspace_header_bytes())
        _lib.check(_lib.lib().simsd_allgather_wait(self._sig_arr, self.rank, self.world, ws.data_ptr(),
                                                   ws.numel(), _lib.stream_ptr(dev)), "allgather_wait")

    def close(self) -> None:
        for blk in self.outs.values():
            blk.close()
        self.outs.clear()
        self.sig.close()
