"""simsd_thin_linear_noalloc: the thin linear for callers that cannot allocate.

Some callers of this library have no way to allocate device memory at call time
(a plugin host that only lends out the call's tensors, code running inside an
allocator callback, a foreign-language binding with no CUDA allocator).  For
them the library offers one entry point whose scratch is a fixed array inside
the library itself.  This test drives it through the C ABI, with inputs and
outputs that the test allocates, and checks it against the regular
workspace-based entry point on two calls in a row.

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

from kernels import _lib
from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul

pytestmark = pytest.mark.gpu
DEV = "cuda"


def tol(ref):
    if ref.dtype == torch.float32:
        return 1e-5 * max(1.0, float(ref.abs().max()))
    return 2 ** -7 * float(ref.abs().max()) + 1e-3


def rnd(*shape, dtype=torch.bfloat16, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV, dtype=torch.float32) * scale).to(dtype)


def noalloc(x, w, w_up=None, bias=None):
    """Call the entry point; y is allocated here, by the caller, not by the library."""
    M, K = x.shape
    N = w.shape[0]
    y = torch.empty(M, N, device=x.device, dtype=x.dtype)
    rc = _lib.lib().simsd_thin_linear_noalloc(
        x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), w.stride(0), w.stride(1),
        w_up.data_ptr() if w_up is not None else None, bias.data_ptr() if bias is not None else None,
        y.data_ptr(), y.stride(0), M, N, K, _lib.dtype_code(x.dtype),
        _lib.EPI_SILU_MUL if w_up is not None else _lib.EPI_NONE,
        torch.cuda.current_stream().cuda_stream)
    return rc, y


def noalloc_error():
    """The static array's error word (read and, if set, cleared by the library)."""
    v = ctypes.c_int(-1)
    rc = _lib.lib().simsd_thin_linear_noalloc_error(torch.cuda.current_stream().cuda_stream, ctypes.byref(v))
    assert rc == _lib.SIMSD_OK
    return v.value


@pytest.mark.parametrize("inkernel", [False, True], ids=["fixup-kernel", "in-kernel-reduce"])
@pytest.mark.parametrize("M,N,K", [(4, 2048, 2048), (16, 6144, 4096), (32, 4096, 12288), (1, 300, 72)])
def test_noalloc_matches_workspace_entry_point_twice(M, N, K, inkernel):
    """Two calls in a row against the workspace entry point, with split tiles
    summed by the separate kernel or by their last contributor (the only mode
    that uses the array's per-tile counters, which every launch leaves zero)."""
    x, w = rnd(M, K, seed=M), rnd(N, K, scale=0.02, seed=N + K)
    prev = _lib.set_inkernel_reduce(inkernel)
    try:
        with torch.inference_mode():
            ref = thin_linear(x, w)
            for _ in range(2):
                rc, y = noalloc(x, w)
                torch.cuda.synchronize()
                assert rc == _lib.SIMSD_OK
                assert float((y.float() - ref.float()).abs().max()) <= tol(ref)
                assert float((y.float() - F.linear(x, w).float()).abs().max()) <= tol(ref)
    finally:
        _lib.set_inkernel_reduce(prev)
    assert noalloc_error() == 0


def test_noalloc_strided_activations_twice():
    """A bf16 activation view with a padded row stride (the tensor-core path) and
    a transposed one (the CUDA-core path)."""
    big = rnd(8, 4096 + 64, seed=12)
    x = big[:, :4096]
    xt = rnd(2048, 8, seed=13).t()              # [8, 2048], column-major
    w = rnd(3072, 4096, scale=0.02, seed=14)
    w2 = rnd(1024, 2048, scale=0.02, seed=15)
    with torch.inference_mode():
        ref, ref2 = F.linear(x, w), F.linear(xt, w2)
        for _ in range(2):
            rc, y = noalloc(x, w)
            rc2, y2 = noalloc(xt, w2)
            torch.cuda.synchronize()
            assert rc == _lib.SIMSD_OK and rc2 == _lib.SIMSD_OK
            assert float((y.float() - ref.float()).abs().max()) <= tol(ref)
            assert float((y2.float() - ref2.float()).abs().max()) <= tol(ref2)
    assert noalloc_error() == 0


def test_noalloc_silu_mul_and_fp32_twice():
    x = rnd(8, 4096, seed=3)
    wg, wu = rnd(1536, 4096, scale=0.02, seed=4), rnd(1536, 4096, scale=0.02, seed=5)
    xf, wf = rnd(4, 512, dtype=torch.float32, seed=6), rnd(256, 512, dtype=torch.float32, scale=0.02, seed=7)
    with torch.inference_mode():
        ref = thin_linear_silu_mul(x, wg, wu)
        reff = thin_linear(xf, wf)
        for _ in range(2):
            rc, y = noalloc(x, wg, w_up=wu)
            rcf, yf = noalloc(xf, wf)
            torch.cuda.synchronize()
            assert rc == _lib.SIMSD_OK and rcf == _lib.SIMSD_OK
            assert float((y.float() - ref.float()).abs().max()) <= tol(ref)
            assert float((yf - reff).abs().max()) <= tol(reff)
    assert noalloc_error() == 0


def test_noalloc_rejects_shapes_beyond_its_scratch():
    """M = 64, K = N = 4096 runs one CTA per SM, each with two 64 x 128 fp32
    partial slots (64 KiB); the array holds 8 MiB less a 64 KiB header, so the
    call fits on a GPU with at most 127 SMs and is refused above that (a
    148-SM B200 refuses it)."""
    x, w = rnd(64, 4096, seed=8), rnd(4096, 4096, scale=0.02, seed=9)
    sms = _lib.lib().simsd_device_sm_count()
    fits = sms * 2 * 64 * 128 * 4 <= (8 << 20) - (64 << 10)
    with torch.inference_mode():
        rc, y = noalloc(x, w)
        torch.cuda.synchronize()
    if fits:
        assert rc == _lib.SIMSD_OK
        assert float((y.float() - F.linear(x, w).float()).abs().max()) <= tol(y)
    else:
        assert rc == _lib.SIMSD_ERR_SCRATCH_LIMIT
        assert b"static" in _lib.lib().simsd_status_string(rc)
    assert noalloc_error() == 0
