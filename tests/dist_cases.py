"""Multi-process cases run under torch.distributed.run by test_parallel_cpu.py.

Each rank asserts; a failing rank exits non-zero, which fails the launcher.
Backend gloo on CPU: the local linear is F.linear in fp32 (the CPU stand-in
for the thin-M kernel), so the check isolates the sharding and collective
layout of kernels/parallel.py and kernels/moe_parallel.py.
"""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

REPO = Path(__file__).resolve().parents[1]
for p in (str(REPO / "simsd-release_b200"), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402
import torch.nn.functional as F  # noqa: E402


def case_column():
    from kernels import parallel as P
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator().manual_seed(0)
    M, K, N = 7, 96, 64
    x = torch.randn(M, K, generator=g)
    w = torch.randn(N, K, generator=g)
    b = torch.randn(N, generator=g)
    wg, wu = torch.randn(N, K, generator=g), torch.randn(N, K, generator=g)
    # plain linear with bias
    y_local = F.linear(x, P.column_shard(w, rank, world), P.bias_shard(b, rank, world))
    y = P.gather_columns(y_local)
    assert y.shape == (M, N)
    assert torch.equal(y, F.linear(x, w, b)), "column-parallel linear differs from the full linear"
    # SwiGLU front half, gate and up split at the same rows
    h_local = F.silu(F.linear(x, P.column_shard(wg, rank, world))) * F.linear(x, P.column_shard(wu, rank, world))
    h = P.gather_columns(h_local)
    assert torch.equal(h, F.silu(F.linear(x, wg)) * F.linear(x, wu))
    # the module keeps exactly this rank's rows
    mod = P.ColumnParallelThinLinear(w, b)
    lo, hi = P.column_range(N, rank, world)
    assert torch.equal(mod.weight.data, w[lo:hi]) and torch.equal(mod.bias.data, b[lo:hi])
    gu = P.ColumnParallelGateUp(wg, wu)
    assert torch.equal(gu.w_gate.data, wg[lo:hi]) and torch.equal(gu.w_up.data, wu[lo:hi])


CASES = {"column": case_column}


def main():
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        CASES[sys.argv[1]]()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
