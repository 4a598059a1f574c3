"""fp32 thin linears on the tensor cores (tf32 hi/lo split in the cluster kernel).

The reference requires fp32 results within 1e-5 of the maximum of an IEEE fp32
`F.linear` (kernels/thin_linear_fused_test.py:28-32, :65-71: "not TF32").  For
M <= 64 this build runs fp32 through tc_cluster_kernel with each operand split
on chip into two tf32 parts (hi*hi + hi*lo + lo*hi, fp32 accumulation); these
tests hold it to that tolerance, to a tighter bound against an fp64 product,
and to the CUDA-core IEEE path (SIMSD_PATH_SIMT) of the same library.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from kernels import _lib
from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rnd(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return torch.randn(*shape, generator=g, device=DEV, dtype=torch.float32) * scale


def tol(ref):
    return 1e-5 * max(1.0, float(ref.abs().max()))


def call(x, w, path, w_up=None, bias=None):
    """simsd_thin_linear through the C ABI with an explicit path."""
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, N, device=DEV, dtype=torch.float32)
    dev = x.device
    epi = _lib.EPI_SILU_MUL if w_up is not None else _lib.EPI_NONE
    nbytes = _lib.thin_workspace_size(torch.cuda.current_device(), M, N, K, _lib.SIMSD_F32, epi, 0)
    ws = _lib.workspace(dev, nbytes)
    rc = _lib.lib().simsd_thin_linear(
        x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), w.stride(0), w.stride(1),
        w_up.data_ptr() if w_up is not None else None, bias.data_ptr() if bias is not None else None,
        y.data_ptr(), y.stride(0), M, N, K, _lib.SIMSD_F32, epi, 0, path, ws.data_ptr(), ws.numel(),
        _lib.stream_ptr(dev))
    return rc, y


@pytest.mark.parametrize("K,N", [(2048, 2048), (4096, 6144), (12288, 4096), (2048, 151936 // 8)])
@pytest.mark.parametrize("M", [1, 4, 16, 32, 64])
def test_fp32_tensor_core_within_reference_tolerance(M, K, N):
    x, w = rnd(M, K, seed=M), rnd(N, K, scale=0.02, seed=K + N)
    with torch.inference_mode():
        rc, got = call(x, w, _lib.PATH_TC)          # refused before this path existed (fp32 had no TC path)
        torch.cuda.synchronize()
        assert rc == _lib.SIMSD_OK
        ref = F.linear(x, w)
        truth = (x.double() @ w.double().T)
        auto = thin_linear(x, w)
    scale = float(truth.abs().max())
    assert float((got - ref).abs().max()) <= tol(ref)
    # and within the same bound of the exact (fp64) product
    e_tc = float((got.double() - truth).abs().max())
    e_ieee = float((ref.double() - truth).abs().max())
    print(f"M={M} K={K} N={N}: |tc - exact| {e_tc / scale:.2e}, |cuBLAS fp32 - exact| {e_ieee / scale:.2e} "
          f"(relative to max |y|)")
    assert e_tc <= 1e-5 * max(1.0, scale)
    assert torch.equal(auto, got)                     # the default path is the tensor-core one


def test_fp32_tensor_core_matches_ieee_cuda_core_path():
    x, w = rnd(8, 4096, seed=3), rnd(4096, 4096, scale=0.02, seed=4)
    with torch.inference_mode():
        rc1, tc = call(x, w, _lib.PATH_TC)
        rc2, simt = call(x, w, _lib.PATH_SIMT)
        torch.cuda.synchronize()
    assert rc1 == _lib.SIMSD_OK and rc2 == _lib.SIMSD_OK
    assert float((tc - simt).abs().max()) <= tol(simt)


@pytest.mark.parametrize("K", [32, 33, 72, 1000, 2049])
def test_fp32_odd_k(K):
    """K not a multiple of the 32-element block: the ragged block reads zeros."""
    x, w = rnd(5, K, seed=K), rnd(300, K, scale=0.02, seed=K + 1)
    with torch.inference_mode():
        got = thin_linear(x, w)
        ref = F.linear(x, w)
    assert float((got - ref).abs().max()) <= tol(ref)


@pytest.mark.parametrize("scale", [1e-6, 1e-3, 1.0, 1e2, 1e4])
def test_fp32_magnitudes_and_bias(scale):
    x, w = rnd(4, 2048, scale=scale, seed=7), rnd(1024, 2048, scale=0.02, seed=8)
    b = rnd(1024, scale=scale, seed=9)
    with torch.inference_mode():
        got = thin_linear(x, w, b)
        ref = F.linear(x, w, b)
    assert float((got - ref).abs().max()) <= tol(ref)


def test_fp32_silu_mul_epilogue():
    x = rnd(16, 4096, seed=10)
    wg, wu = rnd(1536, 4096, scale=0.02, seed=11), rnd(1536, 4096, scale=0.02, seed=12)
    with torch.inference_mode():
        got = thin_linear_silu_mul(x, wg, wu)
        ref = F.silu(F.linear(x, wg)) * F.linear(x, wu)
    assert float((got - ref).abs().max()) <= tol(ref)


def test_fp32_deterministic_and_zeros():
    x, w = rnd(32, 4096, seed=13), rnd(4096, 4096, scale=0.02, seed=14)
    with torch.inference_mode():
        a, b = thin_linear(x, w), thin_linear(x, w)
        z = thin_linear(torch.zeros_like(x), w)
    assert torch.equal(a, b)
    assert torch.all(z == 0)


def test_fp32_strided_weight_view():
    big = rnd(4096, 2048 + 32, scale=0.02, seed=15)
    w = big[:, :2048]                     # row stride 2080 fp32 = 8320 bytes (16-byte multiple)
    x = rnd(12, 2048, seed=16)
    with torch.inference_mode():
        got = thin_linear(x, w)
        ref = F.linear(x, w)
    assert float((got - ref).abs().max()) <= tol(ref)


def test_no_device_errors_recorded():
    assert _lib.device_error(torch.device(DEV, torch.cuda.current_device())) == 0
