"""The CPU oracle pinned against the reference's own outputs (tests/golden/*.npz).

Golden vectors come from the reference's code run in the build container
(tests/golden/make_golden.py): `_align` and `reference_moe_dispatch` imported
from the reference, F.linear as the reference's thin-linear ground truth.
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle as O

G = Path(__file__).resolve().parent / "golden"


def _load(name):
    return np.load(G / f"{name}.npz")


def _cases(z):
    return sorted({k.split(".")[0] for k in z.files})


def _f32(a, dtype_str):
    if "bfloat16" in dtype_str:
        return O.bf16_bits_to_f32(a)
    return a.astype(np.float32)


def test_align_matches_reference_bit_exact():
    z = _load("align")
    for c in _cases(z):
        ids, E, nt = z[f"{c}.ids"], int(z[f"{c}.E"]), int(z[f"{c}.num_tiles"])
        a = O.align(ids, E, 16, nt)
        assert a["status"] == 0
        np.testing.assert_array_equal(a["slots"], z[f"{c}.slots"], err_msg=c)
        np.testing.assert_array_equal(a["tile_expert"], z[f"{c}.tile_expert"], err_msg=c)
        flat = ids.reshape(-1)
        np.testing.assert_array_equal(a["sorted_slots"], np.argsort(flat, kind="stable"), err_msg=c)
        np.testing.assert_array_equal(a["counts"], np.bincount(flat, minlength=E), err_msg=c)
        np.testing.assert_array_equal(a["slot_to_row"][a["sorted_slots"]], np.arange(flat.size), err_msg=c)


def test_align_flags_out_of_range_ids():
    a = O.align(np.array([[0, 5], [9, 1]]), 8)
    assert a["status"] == -1
    assert a["slot_to_row"][2] == -1 and a["counts"].sum() == 3


def _moe_tol(ref, dtype_str):
    m = float(np.abs(ref).max())
    if "float32" in dtype_str:
        return 1e-5 * max(1.0, m)           # kernels/workspace/moe_dispatch/duipai.py:58-59
    return 2 ** -6 * m + 1e-3                # duipai.py:60


def test_moe_dispatch_oracle_matches_reference():
    z = _load("moe_dispatch")
    for c in _cases(z):
        dt = str(z[f"{c}.dtype"])
        if "float16" in dt and "bfloat16" not in dt:
            cast = lambda a: a.view(np.float16)  # noqa: E731
        else:
            cast = lambda a: a  # noqa: E731
        args = [cast(z[f"{c}.{k}"]) for k in ("x", "ids", "w", "wg", "wu", "wd")]
        args[1] = z[f"{c}.ids"]
        args[2] = z[f"{c}.w"]
        _, out = O.moe_dispatch(*args, mode=0)
        ref = _f32(z[f"{c}.ref"], dt) if "float16" not in dt or "bfloat16" in dt else z[f"{c}.ref"].view(np.float16).astype(np.float32)
        got = _f32(out, dt) if out.dtype != np.float16 else out.astype(np.float32)
        err = float(np.abs(got - ref).max())
        assert err <= _moe_tol(ref, dt), f"{c}: {err} > {_moe_tol(ref, dt)}"


@pytest.mark.parametrize("via", ["c", "grouped"])
def test_moe_dispatch_grouped_oracle_matches_reference(via):
    """The grouped numpy restatement against the same golden outputs as the C loop."""
    z = _load("moe_dispatch")
    for c in _cases(z):
        dt = str(z[f"{c}.dtype"])
        if "float16" in dt and "bfloat16" not in dt:
            cast = lambda a: a.view(np.float16)  # noqa: E731
        else:
            cast = lambda a: a  # noqa: E731
        args = [cast(z[f"{c}.{k}"]) for k in ("x", "ids", "w", "wg", "wu", "wd")]
        args[1] = z[f"{c}.ids"]
        args[2] = z[f"{c}.w"]
        fn = O.moe_dispatch if via == "c" else O.moe_dispatch_grouped
        _, out = fn(*args, mode=0)
        ref = _f32(z[f"{c}.ref"], dt) if "float16" not in dt or "bfloat16" in dt else z[f"{c}.ref"].view(np.float16).astype(np.float32)
        got = _f32(out, dt) if out.dtype != np.float16 else out.astype(np.float32)
        err = float(np.abs(got - ref).max())
        assert err <= _moe_tol(ref, dt), f"{c}: {err} > {_moe_tol(ref, dt)}"


@pytest.mark.parametrize("mode", [0, 1])
def test_moe_dispatch_grouped_oracle_matches_c_loop(mode):
    """Same rounding points, different summation order inside each dot product:
    the fp32 combines agree to a few fp32 ulps of the scale and almost every
    bf16 output has the same bits (a rounding boundary crossed by the order
    change moves one output by one bf16 ulp)."""
    rng = np.random.default_rng(7)
    T, k, E, H, I = 48, 4, 12, 256, 192
    x = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    wg, wu = (O.f32_to_bf16_bits((rng.standard_normal((E, I, H)) * 0.02).astype(np.float32)) for _ in range(2))
    wd = O.f32_to_bf16_bits((rng.standard_normal((E, H, I)) * 0.02).astype(np.float32))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int64)
    ids[3, 1] = -1                         # an empty slot (expert-parallel buckets) contributes nothing
    w = rng.random((T, k)).astype(np.float32)
    add = O.f32_to_bf16_bits(rng.standard_normal((T, H)).astype(np.float32))
    a_c, o_c = O.moe_dispatch(x, ids, w, wg, wu, wd, add=add, mode=mode)
    a_g, o_g = O.moe_dispatch_grouped(x, ids, w, wg, wu, wd, add=add, mode=mode)
    scale = float(np.abs(a_c).max())
    assert float(np.abs(a_c - a_g).max()) <= 2 ** -8 * scale       # bf16 rounding of h may differ
    assert float((o_c == o_g).mean()) >= 0.98
    assert float(np.abs(O.bf16_bits_to_f32(o_c) - O.bf16_bits_to_f32(o_g)).max()) <= 2 ** -7 * float(
        np.abs(O.bf16_bits_to_f32(o_c)).max())


def _lin_tol(ref, dtype_str):
    m = float(np.abs(ref).max())
    if "float32" in dtype_str:
        return 1e-5 * max(1.0, m)            # kernels/thin_linear_fused_test.py:28-32
    return 2 ** -7 * m + 1e-3


def test_thin_linear_oracle_matches_f_linear():
    z = _load("thin_linear")
    for c in _cases(z):
        dt = str(z[f"{c}.dtype"])
        if dt == "torch.float16":
            x, w = z[f"{c}.x"].view(np.float16), z[f"{c}.w"].view(np.float16)
            ref = z[f"{c}.y"].view(np.float16).astype(np.float32)
        else:
            x, w = z[f"{c}.x"], z[f"{c}.w"]
            ref = _f32(z[f"{c}.y"], dt)
        b = z[f"{c}.b"] if f"{c}.b" in z.files else None
        acc, y = O.thin_linear(x, w, b)
        got = y.astype(np.float32) if y.dtype == np.float16 else _f32(y, dt)
        err = float(np.abs(got - ref).max())
        assert err <= _lin_tol(ref, dt), f"{c}: {err} > {_lin_tol(ref, dt)}"


def test_router_oracle_matches_torch_restatement():
    z = _load("router")
    for c in _cases(z):
        x, wr, b = z[f"{c}.x"], z[f"{c}.wr"], z[f"{c}.bias"]
        ref_ids, ref_w = z[f"{c}.ids"], z[f"{c}.w"]
        k = ref_ids.shape[1]
        ids, w, logits = O.route(x, wr, b, k, renorm=True, scale=1.0)
        # logits agree with an fp64 evaluation to fp32 accumulation noise
        l64 = O.bf16_bits_to_f32(x).astype(np.float64) @ O.bf16_bits_to_f32(wr).astype(np.float64).T
        assert np.abs(logits - l64).max() <= 1e-5 * max(1.0, np.abs(l64).max())
        choice = 1.0 / (1.0 + np.exp(-logits.astype(np.float64))) + b
        srt = np.sort(choice, axis=1)[:, ::-1]
        clear = (srt[:, k - 1] - srt[:, k]) > 1e-5           # no near-tie at the k-th place
        assert clear.mean() > 0.9
        for t in np.nonzero(clear)[0]:
            assert set(ids[t]) == set(ref_ids[t]), (c, t)
            np.testing.assert_array_equal(ids[t], ref_ids[t])  # both sorted by choice, descending
            np.testing.assert_allclose(w[t], ref_w[t], rtol=2e-6, atol=1e-7)


def test_router_ties_go_to_lower_expert_id():
    rng = np.random.RandomState(0)
    H, E, k = 64, 16, 4
    x = O.f32_to_bf16_bits(rng.randn(3, H).astype(np.float32))
    w = rng.randn(E, H).astype(np.float32) * 0.02
    w[9] = w[2]          # experts 2 and 9 tie exactly, as do 5 and 12
    w[12] = w[5]
    w = O.f32_to_bf16_bits(w)
    bias = np.zeros(E, np.float32)
    bias[[2, 9, 5, 12]] = 10.0    # force all four into the top-4
    ids, wts, _ = O.route(x, w, bias, k)
    for t in range(3):
        row = list(ids[t])
        assert sorted(row) == [2, 5, 9, 12]
        assert row.index(2) < row.index(9) and row.index(5) < row.index(12)
    np.testing.assert_allclose(wts.sum(1), 1.0, rtol=1e-6)


def test_router_scale_and_no_renorm():
    rng = np.random.RandomState(1)
    x = O.f32_to_bf16_bits(rng.randn(5, 96).astype(np.float32))
    w = O.f32_to_bf16_bits(rng.randn(12, 96).astype(np.float32) * 0.1)
    ids, w1, lg = O.route(x, w, None, 3, renorm=False, scale=2.5)
    s = 1.0 / (1.0 + np.exp(-lg.astype(np.float64)))
    np.testing.assert_allclose(w1, 2.5 * np.take_along_axis(s, ids, 1), rtol=3e-7)
    ids1, wk1, _ = O.route(x, w, None, 1, renorm=True)      # k = 1: never renormalised
    np.testing.assert_allclose(wk1[:, 0], np.take_along_axis(s, ids1, 1)[:, 0], rtol=3e-7)


def test_silu_mul_oracle_is_fp32_product():
    rng = np.random.RandomState(2)
    x = rng.randn(4, 128).astype(np.float32)
    wg = rng.randn(32, 128).astype(np.float32) * 0.05
    wu = rng.randn(32, 128).astype(np.float32) * 0.05
    acc, _ = O.thin_linear_silu_mul(x, wg, wu)
    g, u = x.astype(np.float64) @ wg.T, x.astype(np.float64) @ wu.T
    np.testing.assert_allclose(acc, g / (1 + np.exp(-g)) * u, rtol=1e-5, atol=1e-6)


def test_torch_eager_restatement_matches_reference_moe():
    """The CPU baseline's stock-path restatement (oracle/torch_eager.py) against the
    reference's reference_moe_dispatch outputs."""
    import torch
    from oracle import torch_eager as TE
    z = _load("moe_dispatch")
    for c in _cases(z):
        dt = str(z[f"{c}.dtype"])
        tdt = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16,
               "torch.float32": torch.float32}[dt]

        def t(a):
            if tdt == torch.bfloat16:
                return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16)
            if tdt == torch.float16:
                return torch.from_numpy(a.view(np.float16).copy())
            return torch.from_numpy(a.copy())
        x, wg, wu, wd, ref = (t(z[f"{c}.{k}"]) for k in ("x", "wg", "wu", "wd", "ref"))
        ids = torch.from_numpy(z[f"{c}.ids"])
        w = torch.from_numpy(z[f"{c}.w"])
        with torch.inference_mode():
            got = TE.moe_infer(x, ids, w, wg, wu, wd)
        err = float((got.float() - ref.float()).abs().max())
        assert err <= _moe_tol(ref.float().numpy(), dt), c
