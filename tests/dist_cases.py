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

import numpy as np  # noqa: E402
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


class CpuEpOps:
    """CPU stand-ins for the expert-parallel layer's compute steps (fp32, one
    row at a time, so a row's result never depends on what it is batched with)."""

    @staticmethod
    def route(x, w_router, bias, k, renorm, scale):
        from oracle.torch_eager import route
        return route(x, w_router, bias, k, renorm=renorm, scale=scale)

    @staticmethod
    def plan(ids, E, world, cap):
        from oracle import oracle as O
        return {k: torch.from_numpy(v) for k, v in O.ep_plan(ids.numpy(), E, world, cap).items()}

    @staticmethod
    def gather(x, slots, k):
        out = torch.zeros((slots.numel(), x.shape[1]), dtype=x.dtype)
        for r, s in enumerate(slots.tolist()):
            if s >= 0:
                out[r] = x[s // k]
        return out

    @staticmethod
    def expert_row(row, wg, wu, wd):
        return F.linear(F.silu(F.linear(row, wg)) * F.linear(row, wu), wd)

    @staticmethod
    def experts(rows, expert_ids, w_gate, w_up, w_down):
        out = torch.zeros_like(rows)
        for r, e in enumerate(expert_ids.tolist()):
            if e >= 0:
                out[r] = CpuEpOps.expert_row(rows[r:r + 1], w_gate[e], w_up[e], w_down[e])[0]
        return out

    @staticmethod
    def combine(ys, slot_pos, w, add):
        T, k = w.shape
        out = torch.zeros((T, ys.shape[1]), dtype=torch.float32)
        for t in range(T):
            for j in range(k):
                p = int(slot_pos[t * k + j])
                if p >= 0:
                    out[t] += ys[p].float() * w[t, j]
        if add is not None:
            out = out + add
        return out.to(ys.dtype)

    @staticmethod
    def shared(x, w_gate, w_up, w_down):
        return F.linear(F.silu(F.linear(x, w_gate)) * F.linear(x, w_up), w_down)


class CpuExchange:
    """CPU stand-in with PeerExchange's contract: persistent receive and return
    blocks of [world * capacity] rows in which only occupied bucket entries are
    rewritten (the rest keep whatever an earlier call left there), and an id
    block rewritten in full by every send (-1 = empty)."""

    def __init__(self, capacity, H, world):
        self.cap, self.H, self.world = capacity, H, world
        n = world * capacity
        self.recv = torch.full((n, H), float("nan"))
        self.recv_expert = torch.full((n,), -7, dtype=torch.int32)
        self.returned = torch.full((n, H), float("nan"))

    def send(self, x, plan, k):
        rows = CpuEpOps.gather(x, plan["send_slot"], k)
        rows[plan["send_slot"] < 0] = float("nan")          # what an empty entry would carry
        got = torch.empty_like(rows)
        dist.all_to_all_single(got, rows)
        dist.all_to_all_single(self.recv_expert, plan["send_expert"].to(torch.int32))
        occ = self.recv_expert >= 0
        self.recv[occ] = got[occ]
        return self.recv, self.recv_expert

    def give_back(self, y):
        sent = y.clone()
        sent[self.recv_expert < 0] = float("nan")
        got = torch.empty_like(sent)
        dist.all_to_all_single(got, sent)
        keep = ~torch.isnan(got).any(dim=1)
        self.returned[keep] = got[keep]
        return self.returned


def case_ep_moe():
    """Expert-parallel layer (2 ranks, CPU ops) == the same computation done
    token by token on one process, for every rank's tokens; plus the bucket
    plan's invariants."""
    from kernels import moe_parallel as MP
    from oracle import oracle as O
    rank, world = dist.get_rank(), dist.get_world_size()
    T, H, E, k, I = 6, 16, 8, 3, 8
    g = torch.Generator().manual_seed(1)
    wr = torch.randn(E, H, generator=g) * 0.3
    bias = torch.randn(E, generator=g) * 0.5
    wg, wu = torch.randn(E, I, H, generator=g) * 0.3, torch.randn(E, I, H, generator=g) * 0.3
    wd = torch.randn(E, H, I, generator=g) * 0.3
    sh = (torch.randn(I, H, generator=g) * 0.3, torch.randn(I, H, generator=g) * 0.3,
          torch.randn(H, I, generator=g) * 0.3)
    xs = [torch.randn(T, H, generator=g) for _ in range(world)]   # every rank's tokens
    lo, hi = MP.expert_range(E, rank, world)
    for capacity, shared in ((None, None), (None, sh), (T * k + 5, None)):
        out = MP.ep_moe_layer(xs[rank], wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, capacity=capacity,
                              shared=shared, ops=CpuEpOps)
        ids, w = CpuEpOps.route(xs[rank], wr, bias, k, True, 1.0)
        ref = torch.zeros(T, H)
        for t in range(T):
            for j in range(k):
                e = int(ids[t, j])
                ref[t] += CpuEpOps.expert_row(xs[rank][t:t + 1], wg[e], wu[e], wd[e])[0] * w[t, j]
        if shared is not None:
            ref = ref + CpuEpOps.shared(xs[rank], *shared)
        assert torch.equal(out, ref), (rank, capacity, (out - ref).abs().max())
    # the peer-store exchange's contract (only occupied entries rewritten, the
    # rest stale): the same output as the all-to-all layer, call after call
    xch = CpuExchange(T * k, H, world)
    for i in range(3):
        xi = torch.randn(T, H, generator=g) * (i + 1)
        want = MP.ep_moe_layer(xi, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, shared=sh, ops=CpuEpOps)
        got = MP.ep_moe_layer(xi, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, shared=sh, ops=CpuEpOps,
                              exchange=xch)
        assert torch.equal(got, want), (rank, i, (got - want).abs().max())
    try:
        MP.ep_moe_layer(xs[rank], wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, capacity=T * k + 1,
                        ops=CpuEpOps, exchange=xch)
        raise AssertionError("a capacity other than the exchange's must be refused")
    except ValueError:
        pass
    # plan invariants: every slot sent once, to the rank holding its expert, in slot order
    ids = torch.randint(0, E, (T, k), generator=g)
    p = O.ep_plan(ids.numpy(), E, world, T * k)
    flat = ids.reshape(-1).numpy()
    for s, pos in enumerate(p["slot_pos"]):
        peer = pos // (T * k)
        assert peer == flat[s] // (E // world) and p["send_slot"][pos] == s
        assert p["send_expert"][pos] == flat[s] % (E // world)
    for peer in range(world):
        sent = [v for v in p["send_slot"][peer * T * k:(peer + 1) * T * k] if v >= 0]
        assert sent == sorted(sent) and len(sent) == p["counts"][peer]
    # a capacity below a bucket's load drops the slots past it
    q = O.ep_plan(np.zeros(5, np.int64), E, world, 2)
    assert list(q["slot_pos"]) == [0, 1, -1, -1, -1] and q["counts"][0] == 5


CASES = {"column": case_column, "ep_moe": case_ep_moe}


def main():
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    try:
        CASES[sys.argv[1]]()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
