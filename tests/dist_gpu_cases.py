"""Multi-GPU cases (one process per GPU, NCCL) run by test_multi_gpu.py.

Each rank checks its own result against the single-GPU path on the same
inputs; a failing rank exits non-zero.
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


def _close(a, b, rel=1e-2):
    return float((a.float() - b.float()).abs().max()) <= rel * float(b.float().abs().max())


def case_column(dev):
    from kernels.parallel import ColumnParallelGateUp, ColumnParallelThinLinear
    from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul
    g = torch.Generator(device=dev).manual_seed(0)       # same weights on every rank
    bf = torch.bfloat16
    x = torch.randn(32, 4096, generator=g, device=dev).to(bf)
    w = (torch.randn(6144, 4096, generator=g, device=dev) * 0.02).to(bf)
    wg, wu = [(torch.randn(3072, 4096, generator=g, device=dev) * 0.02).to(bf) for _ in range(2)]
    with torch.inference_mode():
        y = ColumnParallelThinLinear(w)(x)
        h = ColumnParallelGateUp(wg, wu)(x)
        assert _close(y, thin_linear(x, w)) and _close(h, thin_linear_silu_mul(x, wg, wu))


def case_ep(dev):
    from kernels.moe_dispatch_fused import moe_layer
    from kernels.moe_parallel import ep_moe_layer, expert_range
    rank, world = dist.get_rank(), dist.get_world_size()
    T, k, E, H, I = 64, 8, 64, 1024, 512
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(1)       # same model on every rank
    wr = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(bf)
    bias = torch.randn(E, generator=g, device=dev) * 0.5
    wg, wu = [(torch.randn(E, I, H, generator=g, device=dev) * 0.02).to(bf) for _ in range(2)]
    wd = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(bf)
    gx = torch.Generator(device=dev).manual_seed(10 + rank)
    x = torch.randn(T, H, generator=gx, device=dev).to(bf)
    lo, hi = expert_range(E, rank, world)
    with torch.inference_mode():
        got = ep_moe_layer(x, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E)
        ref = moe_layer(x, wr, bias, k, wg, wu, wd)
        torch.cuda.synchronize()
    assert _close(got, ref), (rank, float((got.float() - ref.float()).abs().max()))
    # the buckets exchanged by NVLink peer stores: the same rows reach the same
    # experts, so the output is the all-to-all layer's bit for bit, call after
    # call with different tokens (the blocks are reused) and inside a CUDA graph
    from kernels.moe_parallel import PeerExchange
    xch = PeerExchange(T * k, H, bf)
    try:
        with torch.inference_mode():
            for i in range(4):
                xi = torch.randn(T, H, generator=gx, device=dev).to(bf)
                a2a = ep_moe_layer(xi, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E)
                p2p = ep_moe_layer(xi, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, exchange=xch)
                torch.cuda.synchronize()
                assert torch.equal(p2p, a2a), (rank, i, float((p2p.float() - a2a.float()).abs().max()))
            xs = torch.randn(T, H, generator=gx, device=dev).to(bf)
            want = ep_moe_layer(xs, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                yg = ep_moe_layer(xs, wr, bias, k, wg[lo:hi], wu[lo:hi], wd[lo:hi], E, exchange=xch)
            for _ in range(3):
                gr.replay()
            torch.cuda.synchronize()
            assert torch.equal(yg, want), rank
            del gr
            torch.cuda.synchronize()
        dist.barrier()
        from kernels import _lib
        assert _lib.device_error(dev) == 0
    finally:
        xch.close()


def case_fused(dev):
    """All-gather fused into the GEMM (NVLink peer stores + a sync point):
    equal to the single-GPU thin linear within tolerance, stable over repeated
    calls (both output buffers, many counter slots) and inside a CUDA graph."""
    from kernels.parallel import FusedAllGather, column_shard
    from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul
    rank, world = dist.get_rank(), dist.get_world_size()
    g = torch.Generator(device=dev).manual_seed(2)
    bf = torch.bfloat16
    # NX different inputs in turn (NX odd): an output buffer is reused every
    # second call, so a read that saw a peer's columns of an earlier call
    # instead of this one's would not match this call's reference
    NX = 5
    xs = [torch.randn(16, 4096, generator=g, device=dev).to(bf) for _ in range(NX)]
    w = (torch.randn(4096, 4096, generator=g, device=dev) * 0.02).to(bf)
    wg, wu = [(torch.randn(2048, 4096, generator=g, device=dev) * 0.02).to(bf) for _ in range(2)]
    x64s = [torch.randn(64, 12288, generator=g, device=dev).to(bf) for _ in range(NX)]
    wd = (torch.randn(4096, 12288, generator=g, device=dev) * 0.02).to(bf)
    x = xs[0]
    ag = FusedAllGather()
    try:
        with torch.inference_mode():
            refs = [thin_linear(v, w) for v in xs]
            refs_h = [thin_linear_silu_mul(v, wg, wu) for v in xs]
            refs_d = [thin_linear(v, wd) for v in x64s]
            ref_h = refs_h[0]
            wl, wgl, wul, wdl = (column_shard(t, rank, world) for t in (w, wg, wu, wd))
            for i in range(40):          # many launches on the cumulative counters
                j = i % NX
                y = ag.linear(xs[j], wl)
                h = ag.linear(xs[j], wgl, wul)
                d = ag.linear(x64s[j], wdl)
                assert _close(y, refs[j]) and _close(h, refs_h[j]) and _close(d, refs_d[j]), i
            # deferred: three launches, one sync point
            for i in range(10):
                j = i % NX
                y = ag.linear(xs[j], wl, wait=False)
                h = ag.linear(xs[j], wgl, wul, wait=False)
                d = ag.linear(x64s[j], wdl, wait=False)
                ag.wait()
                assert _close(y, refs[j]) and _close(h, refs_h[j]) and _close(d, refs_d[j]), i
            torch.cuda.synchronize()
            first = ag.linear(x, wl).clone()
            assert torch.equal(first, ag.linear(x, wl))          # bit-identical across calls
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr):
                yg = ag.linear(x, wl, wait=False)
                hg = ag.linear(x, wgl, wul, wait=False)
                ag.wait()
            for _ in range(5):
                gr.replay()
            torch.cuda.synchronize()
            assert torch.equal(yg, first) and _close(hg, ref_h)
            del gr
            torch.cuda.synchronize()
        dist.barrier()
        from kernels import _lib
        assert _lib.device_error(dev) == 0
    finally:
        ag.close()


def case_verify_tp(dev):
    """The verify forward with every linear column-split (fused all-gather, K
    split pinned to the single-GPU plan): hidden states and greedy tokens equal
    to the single-GPU fused forward bit for bit, on 3 SDAR-8B-wide layers."""
    from kernels import fused_toggle
    from kernels.sdar_verify import SDARShape, SDARVerifyModel, VerifyHarness
    from kernels.sdar_verify_tp import ShardedVerify
    s = SDARShape(layers=3)
    K, BL, P = 4, 4, 128
    model = SDARVerifyModel.random_init(s, dev, seed=5)
    g = torch.Generator().manual_seed(6)
    prompt = torch.randint(0, s.vocab, (P,), generator=g).tolist()
    drafts = [torch.randint(0, s.vocab, (BL,), generator=g).tolist() for _ in range(K)]
    smaps = [torch.randperm(BL, generator=g).tolist() for _ in range(K)]
    h = VerifyHarness(model, prompt, drafts, smaps, BL)
    sv = ShardedVerify(model)
    try:
        fused_toggle.apply_to_model(model, True, fuse_gate_up=True, fuse_qkv=True)
        with torch.inference_mode():
            for trial in range(3):
                d = [[(t * 7 + trial) % s.vocab for t in blk] for blk in drafts]
                h.set_drafts(d, smaps)
                h.fused = True
                h1, id1 = h.window_hidden().clone(), h.window_argmax().clone()
                h.fused = False
                hg, idg = sv.window_hidden(h).clone(), sv.window_argmax(h).clone()
                torch.cuda.synchronize()
                assert torch.equal(h1, hg), ("hidden", trial, float((h1.float() - hg.float()).abs().max()))
                assert torch.equal(id1, idg), ("argmax", trial)
        fused_toggle.apply_to_model(model, False)
        dist.barrier()
        from kernels import _lib
        assert _lib.device_error(dev) == 0
    finally:
        sv.close()


CASES = {"column": case_column, "ep": case_ep, "fused": case_fused, "verify_tp": case_verify_tp}


def main():
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        for name in sys.argv[1:]:
            CASES[name](dev)
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
