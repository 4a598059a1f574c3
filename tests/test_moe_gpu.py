"""GPU parity of the MoE path: router, align and fused dispatch.

* align: bit-exact against the reference's `_align` (golden vectors) and the
  CPU oracle (counts, offsets, stable permutation, padded layout);
* router: bit-exact against the oracle's fixed-order arithmetic (logits,
  ids and weights compared as bits);
* dispatch: the reference tolerance against `reference_moe_dispatch` (golden
  vectors; kernels/workspace/moe_dispatch/duipai.py:37-60), the fp64 accuracy
  gate of duipai.py:88-116, 1e-2 max relative error against the fp32-accumulated
  oracle, and CUDA-graph capture with routing that changes between replays.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from kernels import _lib
from kernels.moe_dispatch_fused import BLOCK_M, _align, _num_tiles, align, moe_dispatch, moe_layer, moe_route
from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


def to_np(t):
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def from_np(a, dtype):
    if dtype == torch.bfloat16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.int16).copy()).view(torch.bfloat16).to(DEV)
    if dtype == torch.float16:
        return torch.from_numpy(np.ascontiguousarray(a).view(np.float16).copy()).to(DEV)
    return torch.from_numpy(np.ascontiguousarray(a).copy()).to(DEV)


def routing(T, k, E, seed, conc=None, device=DEV):
    """Routing as kernels/workspace/moe_dispatch/build_oracle.py:71-90 draws it."""
    g = torch.Generator(device=device).manual_seed(seed)
    if conc is None:
        logits = torch.randn(T, E, device=device, generator=g)
    else:
        pool = max(1, int(E * conc))
        logits = torch.randn(T, E, device=device, generator=g) - 8.0
        hot = torch.randperm(E, device=device, generator=g)[:pool]
        logits[:, hot] += 8.0
    ids = logits.topk(k, dim=-1).indices.contiguous()
    s = torch.sigmoid(logits.float()).gather(1, ids)
    w = s / (s.sum(-1, keepdim=True) + 1e-20) if k > 1 else s
    return ids, (w * 2.5).float()


def experts(E, H, I, dtype, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    mk = lambda *s: (torch.randn(*s, device=DEV, generator=g) * 0.02).to(dtype)  # noqa: E731
    return mk(E, I, H), mk(E, I, H), mk(E, H, I)


def tol(ref):
    m = float(ref.abs().max())
    if ref.dtype == torch.float32:
        return 1e-5 * max(1.0, m)
    return 2 ** -6 * m + 1e-3


# ------------------------------------------------------------------ align
def test_align_matches_reference_golden():
    z = np.load(GOLDEN / "align.npz")
    for c in sorted({k.split(".")[0] for k in z.files}):
        ids = torch.from_numpy(z[f"{c}.ids"]).to(DEV)
        E, nt = int(z[f"{c}.E"]), int(z[f"{c}.num_tiles"])
        slots, tile_expert = _align(ids, E, nt)
        assert np.array_equal(slots.cpu().numpy(), z[f"{c}.slots"]), c
        assert np.array_equal(tile_expert.cpu().numpy(), z[f"{c}.tile_expert"]), c


@pytest.mark.parametrize("T,k,E,conc", [(1, 8, 256, None), (16, 8, 256, 0.1), (64, 8, 256, None),
                                        (1024, 8, 256, 0.5), (4096, 8, 256, 0.3), (333, 3, 13, None),
                                        (100, 1, 1, None), (64, 8, 1024, None)])
def test_align_matches_oracle(T, k, E, conc):
    ids, _ = routing(T, k, E, seed=T + E, conc=conc)
    a = align(ids, E)
    o = O.align(to_np(ids), E, BLOCK_M, _num_tiles(T * k, E))
    for key in ("counts", "offsets", "sorted_slots", "slot_to_row", "slots", "tile_expert"):
        assert np.array_equal(a[key].cpu().numpy(), o[key]), key


def test_align_duplicate_ids_are_stable():
    ids = torch.tensor([[3, 3, 1], [1, 3, 0], [0, 0, 0]], device=DEV)
    a = align(ids, 4)
    flat = ids.flatten().cpu()
    assert torch.equal(a["sorted_slots"].cpu().long(), torch.argsort(flat, stable=True))


def test_align_flags_bad_ids_without_faulting():
    dev = torch.device(DEV, torch.cuda.current_device())
    torch.cuda.synchronize()
    _lib.clear_device_error(dev)
    ids = torch.tensor([[0, 5], [9, 1]], device=DEV)     # 9 >= E = 8
    a = align(ids, 8)
    torch.cuda.synchronize()
    assert a["slot_to_row"][2].item() == -1 and a["counts"].sum().item() == 3
    assert a["sorted_slots"][3].item() == -1
    assert _lib.device_error(dev) & _lib.DEV_ERR_BAD_INDEX
    _lib.clear_device_error(dev)
    assert _lib.device_error(dev) == 0


# ------------------------------------------------------------------ router
def _route_case(T, H, E, bias_std, seed, dtype=torch.bfloat16, wdtype=None):
    g = torch.Generator(device=DEV).manual_seed(seed)
    x = torch.randn(T, H, device=DEV, generator=g).to(dtype)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(wdtype or dtype)
    b = torch.randn(E, device=DEV, generator=g) * bias_std if bias_std else None
    return x, wr, b


@pytest.mark.parametrize("T,H,E,k,bias_std", [(16, 2048, 256, 8, 0.1), (1024, 2048, 256, 8, 0.1),
                                              (64, 4096, 256, 8, 0.5), (7, 130, 13, 3, 0.0),
                                              (33, 1000, 64, 1, 0.2), (5, 64, 1024, 32, 0.1)])
def test_router_bit_exact_vs_oracle(T, H, E, k, bias_std):
    x, wr, b = _route_case(T, H, E, bias_std, seed=T + H)
    ids, wts, lg = moe_route(x, wr, b, k=k, renorm=True, scale=2.5, return_logits=True)
    oi, ow, ol = O.route(to_np(x), to_np(wr), None if b is None else b.cpu().numpy(), k, True, 2.5)
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), ol.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ow.view(np.uint32))


# token-group sizes 4 / 8 / 16 of the fast router (T >= 4 and 16 x 148 SMs pick
# 8 and 16), 16-bit activations with bf16, fp16 or fp32 router weights
@pytest.mark.parametrize("T,H,E,k,dtype,wdtype", [
    (700, 1000, 40, 4, torch.bfloat16, torch.float32),
    (2400, 512, 24, 2, torch.float16, None),
    (2400, 256, 36, 3, torch.bfloat16, torch.float32),
    (40, 520, 72, 6, torch.float16, torch.float32),
    (3000, 264, 20, 5, torch.bfloat16, None)])
def test_router_fast_variants_bit_exact(T, H, E, k, dtype, wdtype):
    x, wr, b = _route_case(T, H, E, 0.2, seed=T + E, dtype=dtype, wdtype=wdtype)
    ids, wts, lg = moe_route(x, wr, b, k=k, renorm=True, scale=1.5, return_logits=True)
    oi, ow, ol = O.route(to_np(x), to_np(wr), b.cpu().numpy(), k, True, 1.5)
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), ol.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ow.view(np.uint32))


def test_router_fp32_inputs_and_no_renorm():
    x, wr, b = _route_case(20, 512, 48, 0.3, seed=9, dtype=torch.float32)
    ids, wts, lg = moe_route(x, wr, b, k=4, renorm=False, scale=1.0, return_logits=True)
    oi, ow, ol = O.route(to_np(x), to_np(wr), b.cpu().numpy(), 4, False, 1.0)
    assert np.array_equal(lg.cpu().numpy().view(np.uint32), ol.view(np.uint32))
    assert np.array_equal(ids.cpu().numpy(), oi)
    assert np.array_equal(wts.cpu().numpy().view(np.uint32), ow.view(np.uint32))


def test_router_ties_pick_lower_id():
    x, wr, _ = _route_case(4, 256, 32, 0.0, seed=3)
    wr[17] = wr[4]
    wr[30] = wr[11]
    b = torch.zeros(32, device=DEV)
    b[[4, 17, 11, 30]] = 10.0
    ids, _ = moe_route(x, wr, b, k=4)
    for row in ids.cpu().tolist():
        assert sorted(row) == [4, 11, 17, 30]
        assert row.index(4) < row.index(17) and row.index(11) < row.index(30)


def _choice_bound(x, wr):
    """Per row: how far any fp32 evaluation of score + bias can be from the exact
    value.  Each logit is a sum of H exact bf16 x bf16 products, so any fp32
    summation order is within gamma_H * sum|x_h w_h| of the exact sum
    (gamma_n = n u / (1 - n u), u = 2^-24); sigmoid has slope <= 1/4; the
    sigmoid evaluation and the bias add cost at most 2^-21 + 2^-23 more."""
    H = x.shape[1]
    u = 2.0 ** -24
    gamma = H * u / (1 - H * u)
    absdot = x.double().abs() @ wr.double().abs().T           # [T, E]
    return gamma * absdot.max(1).values / 4 + 2.0 ** -21 + 2.0 ** -23


def _compare_with_torch_restatement(x, wr, b, ids, wts, k, rid, rw):
    """Rows where the device router and the torch restatement pick different
    ids, each checked against the rounding bound on the exact (fp64) choice
    values; returns the fraction of rows with identical ids."""
    exact = torch.sigmoid(x.double() @ wr.double().T) + b.double()
    bound = _choice_bound(x, wr)
    got, rid = ids.cpu(), torch.as_tensor(rid).cpu()
    diff = torch.nonzero((got != rid).any(1)).flatten().tolist()
    for t in diff:
        j = int(torch.nonzero(got[t] != rid[t]).flatten()[0])
        a, c = int(got[t, j]), int(rid[t, j])
        gap = float((exact[t, a] - exact[t, c]).abs())
        print(f"row {t}: rank {j} id {a} vs {c}, exact choice gap {gap:.3e}, bound {2 * float(bound[t]):.3e}")
        assert gap <= 2 * float(bound[t]), (t, j, gap, float(bound[t]))
    same = (got == rid).all(1)
    np.testing.assert_allclose(wts.cpu()[same].numpy(), torch.as_tensor(rw).cpu()[same].numpy(), rtol=2e-6, atol=1e-7)
    return 1.0 - len(diff) / got.shape[0]


def test_router_golden_torch_restatement():
    """Against the reference-side torch restatement run in the build container
    (tests/golden/router.npz): identical ids except where the exact choice
    values are closer than two rounding bounds."""
    z = np.load(GOLDEN / "router.npz")
    for c in sorted({k.split(".")[0] for k in z.files}):
        x, wr = from_np(z[f"{c}.x"], torch.bfloat16), from_np(z[f"{c}.wr"], torch.bfloat16)
        b = torch.from_numpy(z[f"{c}.bias"]).to(DEV)
        rid, rw = z[f"{c}.ids"], z[f"{c}.w"]
        k = rid.shape[1]
        ids, wts = moe_route(x, wr, b, k=k)
        frac = _compare_with_torch_restatement(x, wr, b, ids, wts, k, rid, rw)
        print(f"{c}: ids identical to the torch restatement on {100 * frac:.2f} % of rows")


@pytest.mark.parametrize("cfg,T", [("cfg2", 16), ("cfg2", 64), ("cfg2", 256), ("cfg2", 1024),
                                   ("cfg4", 64), ("cfg4", 256), ("cfg4", 1024), ("cfg4", 4096)])
def test_router_vs_torch_restatement_at_benchmark_sizes(cfg, T):
    """BASELINE configs[2] / configs[4] routers on the benchmark's own seeds,
    against the torch restatement (sigmoid(x.float() @ Wr.float().T), top-k of
    score + bias, renormalised) evaluated by cuBLAS in fp32 on the GPU and by
    the CPU."""
    from kernels.moe_dispatch_fused import moe_route as route_dev
    from oracle.torch_eager import route as route_torch
    if cfg == "cfg2":
        H, E, std, seed, order = 2048, 256, 0.1, 2024, (16, 64, 256, 1024)
    else:
        H, E, std, seed, order = 4096, 256, 0.5, 77, (64, 256, 1024, 4096)
    g = torch.Generator(device=DEV).manual_seed(seed)
    wr = (torch.randn(E, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, generator=g, device=DEV) * std
    gx = torch.Generator(device=DEV).manual_seed(seed + T)
    x = torch.randn(T, H, generator=gx, device=DEV).to(torch.bfloat16)
    ids, wts = route_dev(x, wr, b, k=8)
    for where in ("cuda", "cpu"):
        rid, rw = route_torch(x.to(where), wr.to(where), b.to(where), 8)
        frac = _compare_with_torch_restatement(x, wr, b, ids, wts, 8, rid, rw)
        print(f"{cfg} T={T}: ids identical to the torch restatement ({where}) on {100 * frac:.2f} % of rows")


# ------------------------------------------------------------------ dispatch
def test_dispatch_golden_reference_outputs():
    z = np.load(GOLDEN / "moe_dispatch.npz")
    for c in sorted({k.split(".")[0] for k in z.files}):
        dt = {"torch.bfloat16": torch.bfloat16, "torch.float32": torch.float32,
              "torch.float16": torch.float16}[str(z[f"{c}.dtype"])]
        x, wg, wu, wd, ref = (from_np(z[f"{c}.{k}"], dt) for k in ("x", "wg", "wu", "wd", "ref"))
        ids = torch.from_numpy(z[f"{c}.ids"]).to(DEV)
        w = torch.from_numpy(z[f"{c}.w"]).to(DEV)
        with torch.inference_mode():
            out = moe_dispatch(x, ids, w, wg, wu, wd)
        err = float((out.float() - ref.float()).abs().max())
        assert out.dtype == ref.dtype and err <= tol(ref), f"{c}: {err} > {tol(ref)}"


@pytest.mark.parametrize("T,k,E,H,I,conc", [(16, 8, 256, 2048, 512, None), (64, 8, 256, 2048, 512, 0.2),
                                            (32, 4, 16, 256, 128, None), (8, 8, 64, 512, 192, 0.05),
                                            (1024, 2, 8, 512, 256, None),     # ~256 rows per expert: 256-row tiles
                                            (600, 4, 16, 256, 192, 0.3)])     # busy experts split in 128/256-row chunks
@pytest.mark.parametrize("size_classes", [False, True], ids=["one-class", "size-classes"])
def test_dispatch_vs_oracle(T, k, E, H, I, conc, size_classes):
    ids, w = routing(T, k, E, seed=T * k + E, conc=conc)
    g = torch.Generator(device=DEV).manual_seed(E + H)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=I)
    with torch.inference_mode():
        out = moe_dispatch(x, ids, w, wg, wu, wd, size_classes=size_classes)
    args = [to_np(t) for t in (x, ids, w, wg, wu, wd)]
    acc1, _ = O.moe_dispatch(*args, mode=1)          # same rounding points as the kernel
    _, ref0 = O.moe_dispatch(*args, mode=0)          # stock moe_infer rounding
    got = out.float().cpu().numpy()
    scale = float(np.abs(acc1).max())
    assert float(np.abs(got - acc1).max()) <= 1e-2 * scale
    r0 = O.bf16_bits_to_f32(ref0)
    assert float(np.abs(got - r0).max()) <= 2 ** -6 * float(np.abs(r0).max()) + 1e-3


def test_dispatch_accuracy_vs_fp64_not_worse_than_stock():
    """duipai.py:88-116: fused error vs fp64 truth <= max(1.5 x stock error, 2^-12 scale)."""
    T, k, E, H, I = 32, 4, 16, 256, 128
    ids, w = routing(T, k, E, seed=5)
    g = torch.Generator(device=DEV).manual_seed(6)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=7)
    with torch.inference_mode():
        out = moe_dispatch(x, ids, w, wg, wu, wd).double().cpu()
    xd, wgd, wud, wdd = (t.double().cpu() for t in (x, wg, wu, wd))
    truth = torch.zeros(T, H, dtype=torch.float64)
    for t in range(T):
        for j in range(k):
            e = int(ids[t, j])
            h = F.silu(xd[t] @ wgd[e].T) * (xd[t] @ wud[e].T)
            truth[t] += (h @ wdd[e].T) * float(w[t, j])
    _, stock = O.moe_dispatch(*[to_np(t) for t in (x, ids, w, wg, wu, wd)], mode=0)
    e_stock = float((torch.from_numpy(O.bf16_bits_to_f32(stock)).double() - truth).abs().max())
    e_fused = float((out - truth).abs().max())
    assert e_fused <= max(1.5 * e_stock, 2 ** -12 * float(truth.abs().max()))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_dispatch_other_dtypes(dtype):
    T, k, E, H, I = 12, 3, 10, 192, 96
    ids, w = routing(T, k, E, seed=11)
    g = torch.Generator(device=DEV).manual_seed(12)
    x = torch.randn(T, H, device=DEV, generator=g).to(dtype)
    wg, wu, wd = experts(E, H, I, dtype, seed=13)
    with torch.inference_mode():
        out = moe_dispatch(x, ids, w, wg, wu, wd)
    a = [to_np(t) for t in (x, ids, w, wg, wu, wd)]
    acc, _ = O.moe_dispatch(*a, mode=1)
    assert float(np.abs(out.float().cpu().numpy() - acc).max()) <= (
        1e-5 if dtype == torch.float32 else 1e-2) * max(1.0, float(np.abs(acc).max()))


def test_dispatch_add_shared_expert_rounding():
    T, k, E, H, I = 8, 2, 8, 256, 128
    ids, w = routing(T, k, E, seed=21)
    g = torch.Generator(device=DEV).manual_seed(22)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    add = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=23)
    with torch.inference_mode():
        base = moe_dispatch(x, ids, w, wg, wu, wd)
        both = moe_dispatch(x, ids, w, wg, wu, wd, add=add)
    assert torch.equal(both, base + add)


def test_dispatch_deterministic_and_noncontiguous_x():
    T, k, E, H, I = 64, 8, 256, 2048, 512
    ids, w = routing(T, k, E, seed=31)
    g = torch.Generator(device=DEV).manual_seed(32)
    big = torch.randn(T, 2 * H, device=DEV, generator=g).to(torch.bfloat16)
    x = big[:, :H]
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=33)
    with torch.inference_mode():
        a = moe_dispatch(x, ids, w, wg, wu, wd)
        b = moe_dispatch(x.contiguous(), ids, w, wg, wu, wd)
        c = moe_dispatch(x, ids, w, wg, wu, wd)
    assert torch.equal(a, b) and torch.equal(a, c)


@pytest.mark.parametrize("T,conc", [(1, None), (2, None), (4, 0.3), (64, None), (300, 0.05)])
def test_dispatch_inkernel_reduction_matches_fixup_kernel_bitwise(T, conc):
    """Grouped GEMM tiles split over CTAs (few tokens: fewer tiles than two per
    CTA) give the same bits whether their last contributor (the default) or the
    separate reduction kernel sums them."""
    k, E, H, I = 8, 256, 2048, 512
    ids, w = routing(T, k, E, seed=T, conc=conc)
    g = torch.Generator(device=DEV).manual_seed(T + 1)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=T + 2)
    with torch.inference_mode():
        got = moe_dispatch(x, ids, w, wg, wu, wd)
        prev = _lib.set_grouped_fixup(True)
        try:
            ref = moe_dispatch(x, ids, w, wg, wu, wd)
        finally:
            _lib.set_grouped_fixup(prev)
        again = moe_dispatch(x, ids, w, wg, wu, wd)      # counters left at zero: same again
    assert torch.equal(got, ref) and torch.equal(again, ref)


def test_dispatch_all_tokens_one_expert_and_empty():
    T, E, H, I = 300, 16, 256, 128
    ids = torch.zeros(T, 1, dtype=torch.long, device=DEV)
    w = torch.ones(T, 1, device=DEV)
    g = torch.Generator(device=DEV).manual_seed(41)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=42)
    with torch.inference_mode():
        out = moe_dispatch(x, ids, w, wg, wu, wd)
        ref = F.linear(F.silu(F.linear(x.float(), wg[0].float())) * F.linear(x.float(), wu[0].float()),
                       wd[0].float())
        empty = moe_dispatch(x[:0], ids[:0], w[:0], wg, wu, wd)
    assert float((out.float() - ref).abs().max()) <= 1e-2 * float(ref.abs().max())
    assert empty.shape == (0, H)


def test_cuda_graph_capture_with_changing_routing():
    T, k, E, H, I = 32, 8, 256, 2048, 512
    ids, w = routing(T, k, E, seed=51, conc=0.15)
    g = torch.Generator(device=DEV).manual_seed(52)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=53)
    with torch.inference_mode():
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                moe_dispatch(x, ids, w, wg, wu, wd)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            out = moe_dispatch(x, ids, w, wg, wu, wd)
        gr.replay()
        torch.cuda.synchronize()
        first = moe_dispatch(x, ids, w, wg, wu, wd)
        assert torch.equal(out, first)
        ids2, w2 = routing(T, k, E, seed=99, conc=None)
        ids.copy_(ids2)
        w.copy_(w2)
        gr.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, moe_dispatch(x, ids, w, wg, wu, wd))


def test_moe_layer_router_experts_shared():
    """BASELINE configs[2] shape at T=64: router + 256 experts (top-8) + one shared expert."""
    T, H, E, k, I = 64, 2048, 256, 8, 512
    g = torch.Generator(device=DEV).manual_seed(61)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, device=DEV, generator=g) * 0.1
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=62)
    sg, su, sd = (t[0] for t in experts(1, H, I, torch.bfloat16, seed=63))
    with torch.inference_mode():
        out = moe_layer(x, wr, b, k, wg, wu, wd, shared=(sg, su, sd))
        ids, wts = moe_route(x, wr, b, k=k)
        shared = thin_linear(thin_linear_silu_mul(x, sg, su), sd)
        ref = moe_dispatch(x, ids, wts, wg, wu, wd) + shared
    assert torch.equal(out, ref)
    oi, ow, _ = O.route(to_np(x), to_np(wr), b.cpu().numpy(), k)
    assert np.array_equal(ids.cpu().numpy(), oi)


def test_programmatic_dependent_launch_moe_chain_is_exact():
    T, H, E, k, I = 64, 2048, 256, 8, 512
    g = torch.Generator(device=DEV).manual_seed(71)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, device=DEV, generator=g) * 0.1
    wg, wu, wd = experts(E, H, I, torch.bfloat16, seed=72)
    sg, su, sd = (t[0] for t in experts(1, H, I, torch.bfloat16, seed=73))
    with torch.inference_mode():
        ref = moe_layer(x, wr, b, k, wg, wu, wd, shared=(sg, su, sd))
        with _lib.weights_static():
            got = moe_layer(x, wr, b, k, wg, wu, wd, shared=(sg, su, sd))
            got2 = moe_layer(got, wr, b, k, wg, wu, wd)
        ref2 = moe_layer(ref, wr, b, k, wg, wu, wd)
        torch.cuda.synchronize()
    assert torch.equal(got, ref) and torch.equal(got2, ref2)


def test_no_device_errors_recorded():
    assert _lib.device_error(torch.device(DEV, torch.cuda.current_device())) == 0


# ------------------------------------------------------------------ stacked shared expert
def test_route_extra_column_for_the_shared_expert():
    T, H, E, k = 100, 512, 64, 6
    g = torch.Generator(device=DEV).manual_seed(71)
    x = torch.randn(T, H, device=DEV, generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(torch.bfloat16)
    b = torch.randn(E, device=DEV, generator=g) * 0.1
    with torch.inference_mode():
        ids, w = moe_route(x, wr, b, k=k)
        ids2, w2 = moe_route(x, wr, b, k=k, extra_expert=E)
    assert ids2.shape == (T, k + 1)
    assert torch.equal(ids2[:, :k], ids) and torch.equal(w2[:, :k], w)
    assert bool((ids2[:, k] == E).all()) and bool((w2[:, k] == 1.0).all())


@pytest.mark.parametrize("T", [16, 256, 1024])
def test_moe_layer_with_stacked_shared_expert(T):
    """The shared expert stacked as expert E (one set of grouped GEMMs) against
    the separate shared-expert launches: the same layer to within the bf16
    rounding of the shared expert's own output."""
    from kernels.moe_dispatch_fused import moe_layer, stack_shared_expert
    H, E, k, I = 2048, 256, 8, 512
    g = torch.Generator(device=DEV).manual_seed(T + 81)
    bf = torch.bfloat16
    x = torch.randn(T, H, device=DEV, generator=g).to(bf)
    wr = (torch.randn(E, H, device=DEV, generator=g) * 0.02).to(bf)
    b = torch.randn(E, device=DEV, generator=g) * 0.1
    wg, wu, wd = experts(E, H, I, bf, seed=T + 82)
    shared = tuple((torch.randn(*sh, device=DEV, generator=g) * 0.02).to(bf) for sh in ((I, H), (I, H), (H, I)))
    with torch.inference_mode():
        ref = moe_layer(x, wr, b, k, wg, wu, wd, shared=shared)
        st = stack_shared_expert(wg, wu, wd, shared)
        got = moe_layer(x, wr, b, k, *st, shared_stacked=True)
        got2 = moe_layer(x, wr, b, k, *st, shared_stacked=True)
    torch.cuda.synchronize()
    assert torch.equal(got, got2)
    err = float((got.float() - ref.float()).abs().max())
    assert err <= 2 ** -7 * float(ref.float().abs().max()) + 1e-3, err
