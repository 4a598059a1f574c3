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

import torch
import torch.distributed as dist

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
