"""Expert-parallel MoE kernels on the GPU: bucket plan (bit-exact vs the
oracle), row gather, combine, dropped slots, and the layer on a one-rank
NCCL group against the single-GPU layer."""
from __future__ import annotations

import datetime
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.nn.functional as F

from kernels import _lib
from kernels import moe_parallel as MP
from kernels.moe_dispatch_fused import moe_dispatch, moe_layer
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ids(T, k, E, seed, lo=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randint(lo, E, (T, k), device=DEV, generator=g)


@pytest.mark.parametrize("T,k,E,world,cap", [(1, 1, 8, 1, 1), (37, 8, 256, 8, 296), (1024, 8, 256, 8, 8192),
                                             (3000, 8, 256, 4, 6000), (513, 4, 64, 2, 40), (64, 8, 256, 8, 9)])
def test_ep_plan_bit_exact_vs_oracle(T, k, E, world, cap):
    ids = _ids(T, k, E, seed=T + E)
    got = MP.ep_plan(ids, E, world, cap)
    ref = O.ep_plan(ids.cpu().numpy(), E, world, cap)
    for key in ("send_slot", "send_expert", "slot_pos", "counts"):
        assert np.array_equal(got[key].cpu().numpy(), ref[key]), key


def test_ep_plan_flags_overflow_and_bad_ids():
    dev = torch.device(DEV, torch.cuda.current_device())
    torch.cuda.synchronize()
    _lib.clear_device_error(dev)
    ids = torch.tensor([[0, 1], [-1, 9], [0, 0]], device=DEV)     # E = 8: -1 empty, 9 bad
    got = MP.ep_plan(ids, 8, 2, 2)
    ref = O.ep_plan(ids.cpu().numpy(), 8, 2, 2)
    torch.cuda.synchronize()
    for key in ref:
        assert np.array_equal(got[key].cpu().numpy(), ref[key]), key
    err = _lib.device_error(dev)
    assert err & _lib.DEV_ERR_BAD_INDEX and err & _lib.DEV_ERR_CAPACITY
    _lib.clear_device_error(dev)


def test_gather_rows_and_combine_exact():
    T, k, H = 50, 4, 256
    g = torch.Generator(device=DEV).manual_seed(3)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    slots = torch.randint(-1, T * k, (300,), device=DEV, generator=g, dtype=torch.int32)
    rows = MP.gather_rows(x, slots, k)
    ok = slots >= 0
    assert torch.equal(rows[ok], x[(slots[ok] // k).long()])
    ys = torch.randn(300, H, device=DEV, generator=g).to(torch.bfloat16)
    pos = torch.randint(-1, 300, (T * k,), device=DEV, generator=g, dtype=torch.int32)
    w = torch.rand(T, k, device=DEV, generator=g)
    add = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    for a in (None, add):
        out = MP.combine(ys, pos, w, a)
        acc = torch.zeros(T, H, device=DEV)
        for j in range(k):
            p = pos.view(T, k)[:, j].long()
            y = torch.where((p >= 0)[:, None], ys[p.clamp(min=0)].float(), torch.zeros_like(acc))
            acc = acc + y * w[:, j:j + 1]
        ref = acc.to(torch.bfloat16)
        if a is not None:
            ref = (ref.float() + a.float()).to(torch.bfloat16)
        assert torch.equal(out, ref)


def test_dispatch_negative_ids_are_empty_slots():
    T, k, E, H, I = 40, 4, 16, 256, 128
    g = torch.Generator(device=DEV).manual_seed(5)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    ids = _ids(T, k, E, seed=6)
    drop = torch.rand(T, k, device=DEV, generator=g) < 0.3
    w = torch.rand(T, k, device=DEV, generator=g)
    wg, wu = [(torch.randn(E, I, H, device=DEV, generator=g) * 0.05).to(torch.bfloat16) for _ in range(2)]
    wd = (torch.randn(E, H, I, device=DEV, generator=g) * 0.05).to(torch.bfloat16)
    dev = torch.device(DEV, torch.cuda.current_device())
    torch.cuda.synchronize()
    _lib.clear_device_error(dev)
    with torch.inference_mode():
        got = moe_dispatch(x, torch.where(drop, torch.full_like(ids, -1), ids), w, wg, wu, wd)
        ref = moe_dispatch(x, ids, torch.where(drop, torch.zeros_like(w), w), wg, wu, wd)
    torch.cuda.synchronize()
    assert _lib.device_error(dev) == 0
    assert float((got.float() - ref.float()).abs().max()) <= 1e-2 * float(ref.float().abs().max())


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_ep_layer_one_rank_group_matches_single_gpu_layer():
    """The full exchange path on a one-rank NCCL group (the multi-rank exchange
    is exercised by the gloo CPU tests and by the multi-GPU bench)."""
    T, k, E, H, I = 96, 8, 64, 512, 256
    g = torch.Generator(device=DEV).manual_seed(7)
    bf = torch.bfloat16
    x = torch.randn(T, H, device=DEV, generator=g).to(bf)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(bf)
    bias = torch.randn(E, device=DEV, generator=g) * 0.5
    wg, wu = [(torch.randn(E, I, H, device=DEV, generator=g) * 0.02).to(bf) for _ in range(2)]
    wd = (torch.randn(E, H, I, device=DEV, generator=g) * 0.02).to(bf)
    sh = tuple((torch.randn(*s, device=DEV, generator=g) * 0.02).to(bf) for s in ((I, H), (I, H), (H, I)))
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ["MASTER_PORT"] = str(_free_port())
    dist.init_process_group("nccl", rank=0, world_size=1, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device(DEV, torch.cuda.current_device()))
    try:
        with torch.inference_mode():
            got = MP.ep_moe_layer(x, wr, bias, k, wg, wu, wd, E, shared=sh)
            ref = moe_layer(x, wr, bias, k, wg, wu, wd, shared=sh)
            torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    assert float((got.float() - ref.float()).abs().max()) <= 1e-2 * float(ref.float().abs().max())
