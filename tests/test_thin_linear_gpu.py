"""GPU parity of the thin-M linear (the test intents of the reference's
kernels/thin_linear_fused_test.py, run against libsimsd_b200 on a B200).

Three references:
  * F.linear on the GPU (cuBLAS), the reference's own ground truth, with its
    tolerance 2^-7 * max|ref| + 1e-3 in bf16 and 1e-5 * max(1, max|ref|) in fp32
    (kernels/thin_linear_fused_test.py:28-32);
  * the CPU oracle (fp32 accumulation in K order): bf16 outputs within max
    relative error 1e-2 of it, plus the reference tolerance;
  * the golden vectors of tests/golden/thin_linear.npz (F.linear outputs recorded
    in the build container).
"""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from kernels import _lib, fused_toggle
from kernels.thin_linear_fused import (FUSE_MAX_M, ThinLinear, should_fuse, thin_linear, thin_linear_argmax,
                                      thin_linear_cat, thin_linear_silu_mul)
from oracle import oracle as O

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"

# (K, N): SDAR-1.7B draft projections, SDAR-8B target projections
DEPLOYED = [(2048, 2048), (2048, 1024), (2048, 6144), (6144, 2048), (2048, 4096),
            (4096, 6144), (4096, 4096), (12288, 4096)]


def tol(ref: torch.Tensor) -> float:
    if ref.dtype == torch.float32:
        return 1e-5 * max(1.0, float(ref.abs().max()))
    return 2 ** -7 * float(ref.abs().max()) + 1e-3


def rnd(*shape, dtype=torch.bfloat16, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV, dtype=torch.float32) * scale).to(dtype)


def assert_matches(x, w, b=None, **kw):
    with torch.inference_mode():
        ref = F.linear(x, w, b)
        got = thin_linear(x, w, b, **kw)
    assert got.shape == ref.shape and got.dtype == ref.dtype
    err = float((got.float() - ref.float()).abs().max())
    assert err <= tol(ref), f"max_err {err:.3e} > tol {tol(ref):.3e}"
    return got, err


def to_np(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def assert_oracle(x, w, got, silu_up=None):
    """Within 1e-2 max relative error of the fp32-accumulated oracle, and the reference tolerance."""
    if silu_up is None:
        acc, _ = O.thin_linear(to_np(x), to_np(w))
    else:
        acc, _ = O.thin_linear_silu_mul(to_np(x), to_np(w), to_np(silu_up))
    g = got.float().cpu().numpy()
    scale = float(np.abs(acc).max())
    rel = float(np.abs(g - acc).max()) / max(scale, 1e-30)
    assert rel <= 1e-2, f"relative error {rel:.3e} vs oracle"
    assert float(np.abs(g - acc).max()) <= 2 ** -7 * scale + 1e-3


@pytest.mark.parametrize("K,N", DEPLOYED)
@pytest.mark.parametrize("M", [1, 2, 4, 8, 16, 32, 64])
def test_deployed_shapes(M, K, N):
    assert_matches(rnd(M, K, seed=M), rnd(N, K, scale=0.02, seed=K + N))


def test_lm_head_shape():
    assert_matches(rnd(4, 2048, seed=3), rnd(151936, 2048, scale=0.02, seed=4))


@pytest.mark.parametrize("K,N", [(1000, 1531), (2049, 129), (6143, 2047), (127, 65), (1, 1), (2048, 1),
                                 (3, 4096), (1021, 769), (4096, 1), (64, 129), (72, 200)])
def test_odd_dims(K, N):
    """Non-power-of-2 / degenerate dims must be masked, not rounded."""
    assert_matches(rnd(4, K, seed=K), rnd(N, K, scale=0.02, seed=N))


@pytest.mark.parametrize("M", [1, 4, 16, 33, 64])
def test_oracle_parity_small(M):
    x, w = rnd(M, 1024, seed=100 + M), rnd(640, 1024, scale=0.02, seed=200 + M)
    got, _ = assert_matches(x, w)
    assert_oracle(x, w, got)


def test_baseline_config0_qkv_1p7b():
    """x [16, 2048] ~N(0,1), W [4096, 2048] ~N(0,0.02), seed 0."""
    x, w = rnd(16, 2048, seed=0), rnd(4096, 2048, scale=0.02, seed=0)
    got, _ = assert_matches(x, w)
    assert_oracle(x, w, got)


def test_golden_vectors():
    z = np.load(GOLDEN / "thin_linear.npz")
    for c in sorted({k.split(".")[0] for k in z.files}):
        dt = str(z[f"{c}.dtype"])
        tdt = {"torch.bfloat16": torch.bfloat16, "torch.float16": torch.float16,
               "torch.float32": torch.float32}[dt]
        def dev(a):
            if tdt == torch.bfloat16:
                return torch.from_numpy(a.view(np.int16).copy()).view(torch.bfloat16).to(DEV)
            if tdt == torch.float16:
                return torch.from_numpy(a.view(np.float16).copy()).to(DEV)
            return torch.from_numpy(a.copy()).to(DEV)
        x, w, ref = dev(z[f"{c}.x"]), dev(z[f"{c}.w"]), dev(z[f"{c}.y"])
        b = dev(z[f"{c}.b"]) if f"{c}.b" in z.files else None
        with torch.inference_mode():
            got = thin_linear(x, w, b)
        err = float((got.float() - ref.float()).abs().max())
        assert err <= tol(ref), f"{c}: {err} > {tol(ref)}"


def test_fp32_ieee():
    """fp32 must be IEEE fp32 accumulation, not TF32 (~1e-3 relative)."""
    x, w = rnd(4, 2048, dtype=torch.float32), rnd(2048, 2048, scale=0.02, dtype=torch.float32, seed=3)
    got, err = assert_matches(x, w)
    ref_max = float(F.linear(x, w).abs().max())
    assert err / ref_max < 1e-5


def test_fp16():
    assert_matches(rnd(8, 4096, dtype=torch.float16, seed=5), rnd(2048, 4096, dtype=torch.float16,
                                                                     scale=0.02, seed=6))


@pytest.mark.parametrize("scale", [1e-6, 1e-3, 1.0, 1e2, 1e4])
def test_magnitudes(scale):
    assert_matches(rnd(4, 2048, scale=scale, seed=int(scale) + 1), rnd(2048, 2048, scale=0.02, seed=9))


def test_zeros():
    z = torch.zeros(4, 2048, device=DEV, dtype=torch.bfloat16)
    with torch.inference_mode():
        out = thin_linear(z, rnd(2048, 2048, scale=0.02))
    assert torch.all(out == 0)


def test_noncontiguous_x_and_w():
    """A transposed activation view (CUDA-core path), an offset weight view and a
    strided weight view (tensor-core path through TMA strides)."""
    assert_matches(rnd(2048, 4, seed=11).t(), rnd(2048, 2048, scale=0.02, seed=12))
    big = rnd(4096, 2048, scale=0.02, seed=13)
    assert_matches(rnd(4, 2048, seed=14), big[1024:3072])
    assert_matches(rnd(4, 2048, seed=15), big[::2])
    xs = rnd(8, 4096, seed=16)[:, :2048]           # row stride 4096, inner stride 1
    assert_matches(xs, big[:1024])


def test_leading_dims_preserved():
    x, w = rnd(2, 3, 2048, seed=16), rnd(512, 2048, scale=0.02, seed=17)
    with torch.inference_mode():
        got, ref = thin_linear(x, w), F.linear(x, w)
    assert got.shape == (2, 3, 512) == ref.shape
    assert float((got.float() - ref.float()).abs().max()) <= tol(ref)


def test_bias_applied():
    x, w = rnd(4, 512, seed=18), rnd(256, 512, scale=0.02, seed=19)
    b = rnd(256, scale=0.5, seed=20)
    assert_matches(x, w, b)
    assert_matches(x.float(), w.float(), b.float())


def test_empty_inputs():
    w = rnd(256, 512, scale=0.02)
    with torch.inference_mode():
        assert thin_linear(torch.empty(0, 512, device=DEV, dtype=torch.bfloat16), w).shape == (0, 256)
        y = thin_linear(torch.empty(3, 0, device=DEV, dtype=torch.bfloat16),
                        torch.empty(5, 0, device=DEV, dtype=torch.bfloat16))
        assert y.shape == (3, 5) and torch.all(y == 0)


def test_rejects_grad_mode():
    x = rnd(4, 512, seed=21).requires_grad_(True)
    w = rnd(256, 512, scale=0.02, seed=22)
    with pytest.raises(RuntimeError, match="forward-only"):
        thin_linear(x, w)
    with torch.no_grad():
        thin_linear(x, w)


def test_dtype_mismatch_rejected():
    with pytest.raises(TypeError):
        with torch.inference_mode():
            thin_linear(rnd(4, 512), rnd(256, 512, dtype=torch.float32))


@pytest.mark.parametrize("split_k", [0, 1, 2, 8])
def test_reduction_is_deterministic(split_k):
    """Bit-identical outputs across calls, for the stream-K split and forced splits."""
    x, w = rnd(4, 6144, seed=23), rnd(2048, 6144, scale=0.02, seed=24)
    cfg = (16, 128, 64, split_k)
    with torch.inference_mode():
        first = thin_linear(x, w, config=cfg)
        for _ in range(8):
            assert torch.equal(thin_linear(x, w, config=cfg), first)
        ref = F.linear(x, w)
        assert float((first.float() - ref.float()).abs().max()) <= tol(ref)


def test_split_count_changes_nothing_beyond_rounding():
    x, w = rnd(16, 4096, seed=31), rnd(4096, 4096, scale=0.02, seed=32)
    with torch.inference_mode():
        outs = [thin_linear(x, w, config=(16, 128, 64, s)) for s in (0, 1, 3, 16)]
    for o in outs[1:]:
        assert float((o.float() - outs[0].float()).abs().max()) <= tol(outs[0])


def test_large_M_is_correct_when_forced():
    """always_fuse at prefill sizes: chunks of 256 rows, still within tolerance."""
    lin = nn.Linear(2048, 1024, bias=False).to(DEV, torch.bfloat16).eval()
    for M in (96, 97, 300, 600):
        x = rnd(M, 2048, seed=M)
        with torch.inference_mode():
            got = ThinLinear(lin, always_fuse=True)(x)
            ref = F.linear(x, lin.weight)
        assert float((got.float() - ref.float()).abs().max()) <= tol(ref), M


def test_dispatch_falls_back_above_guard():
    lin = nn.Linear(2048, 2048, bias=False).to(DEV, torch.bfloat16).eval()
    mod = ThinLinear(lin)
    assert should_fuse(4, 2048, 2048) and should_fuse(FUSE_MAX_M, 2048, 2048)
    assert not should_fuse(FUSE_MAX_M + 1, 2048, 2048)
    with torch.inference_mode():
        for M, fused in ((4, True), (32, True), (64, True), (65, False), (96, False)):
            x = rnd(M, 2048, seed=M)
            got, ref = mod(x), F.linear(x, lin.weight)
            if fused:
                assert float((got.float() - ref.float()).abs().max()) <= tol(ref)
            else:
                assert torch.equal(got, ref), f"M={M} should have used F.linear"
        x3 = rnd(1, 96, 2048, seed=7)
        assert torch.equal(mod(x3), F.linear(x3, lin.weight))


def test_silu_mul_epilogue():
    x = rnd(16, 4096, seed=40)
    wgu = rnd(2 * 1536, 4096, scale=0.02, seed=41)     # one fused gate_up weight, two halves
    wg, wu = wgu[:1536], wgu[1536:]
    with torch.inference_mode():
        got = thin_linear_silu_mul(x, wg, wu)
        ref32 = F.silu(F.linear(x.float(), wg.float())) * F.linear(x.float(), wu.float())
        eager = F.silu(F.linear(x, wg)) * F.linear(x, wu)          # SDARMLP's bf16 chain
    assert float((got.float() - ref32).abs().max()) <= 2 ** -7 * float(ref32.abs().max()) + 1e-3
    assert float((got.float() - eager.float()).abs().max()) <= 2 ** -6 * float(eager.abs().max()) + 1e-3
    assert_oracle(x, wg, got, silu_up=wu)


@pytest.mark.parametrize("M", [4, 16, 64])
def test_silu_mul_single_k_block(M):
    """K = 64 is one K block, so every cluster is a single CTA (whole tiles) and
    the gate and up rows meet through the staging rows of the epilogue; N = 1000
    leaves a ragged last tile."""
    x = rnd(M, 64, seed=60 + M)
    wg, wu = rnd(1000, 64, scale=0.02, seed=61), rnd(1000, 64, scale=0.02, seed=62)
    with torch.inference_mode():
        got = thin_linear_silu_mul(x, wg, wu)
        ref32 = F.silu(F.linear(x.float(), wg.float())) * F.linear(x.float(), wu.float())
    assert got.shape == (M, 1000)
    assert float((got.float() - ref32).abs().max()) <= 2 ** -7 * float(ref32.abs().max()) + 1e-3
    assert_oracle(x, wg, got, silu_up=wu)


@pytest.mark.parametrize("M", [4, 32, 64])
def test_silu_mul_sdar8b(M):
    x = rnd(M, 4096, seed=50 + M)
    wg, wu = rnd(12288, 4096, scale=0.02, seed=51), rnd(12288, 4096, scale=0.02, seed=52)
    with torch.inference_mode():
        got = thin_linear_silu_mul(x, wg, wu)
        ref = F.silu(F.linear(x.float(), wg.float())) * F.linear(x.float(), wu.float())
    err = float((got.float() - ref).abs().max())
    assert err <= 1e-2 * float(ref.abs().max())


def test_cuda_graph_capture_and_replay():
    x, w = rnd(4, 2048, seed=25), rnd(2048, 2048, scale=0.02, seed=26)
    with torch.inference_mode():
        ref = F.linear(x, w)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                thin_linear(x, w)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = thin_linear(x, w)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
    assert float((out.float() - ref.float()).abs().max()) <= tol(ref)
    with torch.inference_mode():
        x.mul_(2.0)
        g.replay()
        torch.cuda.synchronize()
        assert float((out.float() - F.linear(x, w).float()).abs().max()) <= tol(ref) * 2


def test_graph_capture_with_multiple_shapes_shares_workspace():
    xs = [(rnd(4, 2048, seed=30), rnd(1024, 2048, scale=0.02, seed=31)),
          (rnd(4, 6144, seed=32), rnd(2048, 6144, scale=0.02, seed=33)),
          (rnd(32, 4096, seed=34), rnd(6144, 4096, scale=0.02, seed=35))]
    with torch.inference_mode():
        refs = [F.linear(x, w) for x, w in xs]
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(3):
                for x, w in xs:
                    thin_linear(x, w)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            outs = [thin_linear(x, w) for x, w in xs]
        for _ in range(4):
            g.replay()
        torch.cuda.synchronize()
    for out, ref in zip(outs, refs):
        assert float((out.float() - ref.float()).abs().max()) <= tol(ref)


def test_non_current_device_guard():
    """The operator runs on the tensors' device even when another device is current."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    x = rnd(4, 1024).to("cuda:1")
    w = rnd(512, 1024, scale=0.02).to("cuda:1")
    with torch.cuda.device(0), torch.inference_mode():
        got, ref = thin_linear(x, w), F.linear(x, w)
    assert float((got.float() - ref.float()).abs().max()) <= tol(ref)


class _Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(512, 512, bias=False)
        self.gate_proj = nn.Linear(512, 1024, bias=False)
        self.other = nn.Linear(512, 8, bias=False)

    def forward(self, x):
        return self.gate_proj(self.q_proj(x)), self.other(x)


def test_toggle_swaps_and_restores_on_gpu():
    m = _Tiny().to(DEV, torch.bfloat16).eval()
    x = rnd(4, 512, seed=40)
    with torch.inference_mode():
        ref = m(x)
    assert fused_toggle.apply_to_model(m, True) == 2
    fused_toggle.warmup(m, block_length=4)
    with torch.inference_mode():
        got = m(x)
    for a, b in zip(got, ref):
        assert float((a.float() - b.float()).abs().max()) <= tol(b)
    assert fused_toggle.apply_to_model(m, False) == 2


class _SwiGLU(nn.Module):
    def __init__(self, H=1024, I=2048):
        super().__init__()
        self.gate_proj = nn.Linear(H, I, bias=False)
        self.up_proj = nn.Linear(H, I, bias=False)
        self.down_proj = nn.Linear(I, H, bias=False)
        self.act_fn = nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


def test_toggle_fused_gate_up_mlp():
    m = _SwiGLU().to(DEV, torch.bfloat16).eval()
    x = rnd(8, 1024, seed=60)
    with torch.inference_mode():
        ref = m(x)
    fused_toggle.apply_to_model(m, True, fuse_gate_up=True)
    with torch.inference_mode():
        got = m(x)
    fused_toggle.apply_to_model(m, False)
    assert float((got.float() - ref.float()).abs().max()) <= 2 ** -6 * float(ref.abs().max()) + 1e-3


def _chain(x, ws):
    h = x
    for i, w in enumerate(ws):
        h = thin_linear(h, w)
        if i % 3 == 2:
            h = h * 0.5                  # a torch kernel between two of ours
    return h


def test_programmatic_dependent_launch_chain_is_exact():
    """With PDL each launch streams its weights before the previous kernel ends;
    a dependent chain must still see every activation, bit for bit."""
    ws = [rnd(2048, 2048, scale=0.03, seed=70 + i) for i in range(8)]
    x = rnd(16, 2048, seed=80)
    with torch.inference_mode():
        ref = _chain(x, ws)
        with _lib.weights_static():
            got = _chain(x, ws)
            h = thin_linear_silu_mul(got[:4], ws[0], ws[1])
        h_ref = thin_linear_silu_mul(ref[:4], ws[0], ws[1])
        torch.cuda.synchronize()
    assert torch.equal(got, ref) and torch.equal(h, h_ref)
    assert not _lib.set_pdl(False)


def test_programmatic_dependent_launch_in_graph():
    ws = [rnd(4096, 2048, scale=0.02, seed=90), rnd(2048, 4096, scale=0.02, seed=91)]
    x = rnd(8, 2048, seed=92)
    with torch.inference_mode():
        ref = thin_linear(thin_linear(x, ws[0]), ws[1])
        with _lib.weights_static():
            for _ in range(3):
                thin_linear(thin_linear(x, ws[0]), ws[1])
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                out = thin_linear(thin_linear(x, ws[0]), ws[1])
        for _ in range(5):
            g.replay()
        torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("M,K,N,silu", [(4, 4096, 4096, False), (16, 4096, 6144, False), (32, 12288, 4096, False),
                                         (64, 4096, 4096, False), (16, 4096, 12288, True), (64, 4096, 3072, True),
                                         (200, 2048, 512, False), (3, 100, 300, False)])
def test_inkernel_reduction_matches_fixup_kernel_bitwise(M, K, N, silu):
    """Split tiles summed by their last contributor inside the GEMM give the same
    bits as the separate reduction kernel (same slots, same order)."""
    x = rnd(M, K, seed=M + 7)
    ws = [rnd(N, K, scale=0.02, seed=N + K + i) for i in range(2 if silu else 1)]
    f = (lambda: thin_linear_silu_mul(x, *ws)) if silu else (lambda: thin_linear(x, ws[0]))
    with torch.inference_mode():
        ref = f()
        prev = _lib.set_inkernel_reduce(True)
        try:
            got = [f() for _ in range(2)]
        finally:
            _lib.set_inkernel_reduce(prev)
        torch.cuda.synchronize()
    assert all(torch.equal(g, ref) for g in got)


# ------------------------------------------------------------------ greedy head
# thin_linear_argmax = argmax over the rounded logits that thin_linear itself
# returns (same plan, same summation order), ties to the lowest column.
@pytest.mark.parametrize("M,N,K,dtype,bias", [
    (32, 151936, 4096, torch.bfloat16, False),   # SDAR-8B lm_head over the 32 verify rows
    (4, 151936, 4096, torch.bfloat16, False),
    (1, 1000, 64, torch.bfloat16, False),
    (16, 12345, 1024, torch.float16, True),      # ragged last tile, fp16, bias
    (64, 50000, 512, torch.bfloat16, True),
    (7, 300, 130, torch.bfloat16, False),        # K*2 not a multiple of 16: the device-argmax path
])
def test_argmax_head_equals_argmax_of_thin_linear(M, N, K, dtype, bias):
    x = rnd(M, K, dtype=dtype, seed=M + N)
    w = rnd(N, K, dtype=dtype, scale=0.02, seed=K)
    b = rnd(N, dtype=dtype, scale=0.1, seed=3) if bias else None
    with torch.inference_mode():
        ref = thin_linear(x, w, b).argmax(-1)
        got = thin_linear_argmax(x, w, b)
        again = thin_linear_argmax(x, w, b)      # the argmax slots are zero again after a call
    torch.cuda.synchronize()
    assert got.dtype == torch.int64 and got.shape == (M,)
    assert torch.equal(got, ref) and torch.equal(again, ref)


def test_argmax_head_ties_and_zeros():
    M, N, K = 8, 4096, 1024
    x = rnd(M, K, seed=11)
    w = rnd(N, K, scale=0.02, seed=12)
    w[300] = (x[0].float() * 0.05).to(w.dtype)   # row 0's maximum, by far
    w[3000] = w[300]                             # an exact tie: the lower column wins
    w[77] = w[300] * 0                           # all-zero row
    with torch.inference_mode():
        got = thin_linear_argmax(x, w)
        zero = thin_linear_argmax(torch.zeros_like(x), w)
    torch.cuda.synchronize()
    assert int(got[0]) == 300
    assert torch.equal(got, thin_linear(x, w).argmax(-1))
    assert torch.equal(zero, torch.zeros(M, dtype=torch.int64, device=DEV))   # all logits 0: column 0


def test_argmax_head_vs_fp32_reference():
    """Against a plain fp32 reference: the same column, or a near-tie (the two
    logits within 2 bf16 ulps of the larger, where rounding decides)."""
    M, N, K = 32, 151936, 4096
    x = rnd(M, K, seed=21)
    w = rnd(N, K, scale=0.02, seed=22)
    with torch.inference_mode():
        got = thin_linear_argmax(x, w).cpu()
    ref_logits = (x.float() @ w.float().T).to(torch.bfloat16).float().cpu()
    ref = ref_logits.argmax(-1)
    for m in range(M):
        g, r = int(got[m]), int(ref[m])
        if g != r:
            a, c = float(ref_logits[m, g]), float(ref_logits[m, r])
            assert abs(a - c) <= 2 * 2 ** -7 * max(abs(a), abs(c)), (m, g, r, a, c)


def test_argmax_head_in_graph_replay():
    x = rnd(32, 4096, seed=31)
    w = rnd(20000, 4096, scale=0.02, seed=32)
    with torch.inference_mode():
        ref = thin_linear_argmax(x, w)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            thin_linear_argmax(x, w)
        torch.cuda.current_stream().wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            out = thin_linear_argmax(x, w)
        for _ in range(3):
            g.replay()
        torch.cuda.synchronize()
    assert torch.equal(out, ref)


# ------------------------------------------------------------------ merged q/k/v
@pytest.mark.parametrize("M,K,ns,dtype", [
    (32, 4096, (4096, 1024, 1024), torch.bfloat16),   # SDAR-8B q/k/v at the verify M
    (4, 4096, (4096, 1024, 1024), torch.bfloat16),
    (64, 4096, (4096, 1024, 1024), torch.bfloat16),
    (1, 2048, (2048, 1024, 1024), torch.float16),     # SDAR-1.7B draft
    (16, 1024, (256, 1000), torch.bfloat16),          # two parts, ragged last
    (8, 512, (384,), torch.bfloat16),                 # one part
    (8, 512, (100, 128, 64), torch.bfloat16),         # first part not 128-aligned: per-part fallback
    (96, 1024, (256, 128, 128), torch.bfloat16),      # M > 64: per-part fallback
])
def test_qkv_cat_matches_f_linear(M, K, ns, dtype):
    x = rnd(M, K, dtype=dtype, seed=M + K)
    ws = [rnd(n, K, dtype=dtype, scale=0.02, seed=10 + i) for i, n in enumerate(ns)]
    with torch.inference_mode():
        outs = thin_linear_cat(x, ws)
        again = thin_linear_cat(x, ws)
        refs = [F.linear(x, w) for w in ws]
    torch.cuda.synchronize()
    for o, a, r in zip(outs, again, refs):
        assert o.shape == r.shape and o.dtype == r.dtype
        assert float((o.float() - r.float()).abs().max()) <= tol(r)
        assert torch.equal(o, a)                      # bit-identical across calls
    assert_oracle(x, torch.cat(ws, 0), torch.cat([o.reshape(M, -1) for o in outs], -1))


def test_qkv_merge_in_attention_module():
    class Attn(nn.Module):
        def __init__(self):
            super().__init__()
            self.q_proj = nn.Linear(4096, 4096, bias=False)
            self.k_proj = nn.Linear(4096, 1024, bias=False)
            self.v_proj = nn.Linear(4096, 1024, bias=False)

        def forward(self, h):
            return self.q_proj(h), self.k_proj(h), self.v_proj(h)

    m = Attn().to(DEV, torch.bfloat16)
    h = rnd(1, 32, 4096, seed=5)
    with torch.inference_mode():
        ref = m(h)
        assert fused_toggle.apply_to_model(m, True, fuse_qkv=True) == 3
        got = m(h)
        got2 = m(h.clone())                           # a new input tensor: a new merged launch
        fused_toggle.apply_to_model(m, False)
    for g, g2, r in zip(got, got2, ref):
        assert g.shape == r.shape
        assert float((g.float() - r.float()).abs().max()) <= tol(r)
        assert torch.equal(g, g2)


def test_no_device_errors_recorded():
    assert _lib.device_error(torch.device(DEV, torch.cuda.current_device())) == 0
