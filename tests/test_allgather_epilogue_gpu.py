"""The fused all-gather's store path on one GPU.

simsd_thin_linear_allgather stores every output element of this rank's
columns into every rank's y at col_offset.  Here the "ranks" are two buffers
on the same GPU, so the epilogue's multi-target stores (packed 4- and 8-byte
pieces where the columns allow, 2-byte ones where an odd column offset does
not) run without a second process; the outputs must be the single-GPU thin
linear's bit for bit, and nothing outside the rank's columns may be written.
No sync point is needed: the launch is complete on the stream."""
from __future__ import annotations

import ctypes

import pytest
import torch

from kernels import _lib
from kernels.thin_linear_fused import thin_linear, thin_linear_silu_mul

pytestmark = pytest.mark.gpu
DEV = "cuda"


def rnd(*shape, scale=1.0, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    return (torch.randn(*shape, generator=g, device=DEV) * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K,silu,col_offset", [
    (16, 2048, 4096, False, 2048),     # 8-byte pieces
    (64, 1536, 4096, True, 1536),      # SiLU*mul, 64 activation rows
    (32, 3072, 4096, False, 6),        # 4-byte pieces (even offset, not a multiple of 4)
    (5, 1000, 4096, False, 3),         # odd offset: 2-byte stores; ragged last tile
    (40, 640, 12288, False, 640),      # deep K, larger clusters
    (1, 384, 1024, True, 384),
])
def test_allgather_stores_into_every_target(M, N, K, silu, col_offset):
    x = rnd(M, K, seed=M)
    w = rnd(N, K, scale=0.02, seed=N)
    w_up = rnd(N, K, scale=0.02, seed=N + 1) if silu else None
    world, rank = 2, 0
    ldy = col_offset + N + 8
    ys = [torch.full((M, ldy), float("nan"), device=DEV, dtype=torch.bfloat16) for _ in range(world)]
    peers = (ctypes.c_void_p * world)(*[y.data_ptr() for y in ys])
    ws = _lib.workspace(torch.device(DEV, torch.cuda.current_device()), _lib.lib().simsd_workspace_header_bytes())
    with torch.inference_mode():
        ref = thin_linear_silu_mul(x, w, w_up) if silu else thin_linear(x, w)
        rc = _lib.lib().simsd_thin_linear_allgather(
            x.data_ptr(), x.stride(0), x.stride(1), w.data_ptr(), w.stride(0), w.stride(1),
            w_up.data_ptr() if silu else None, None, peers, ldy, col_offset, M, N, K, _lib.SIMSD_BF16,
            _lib.EPI_SILU_MUL if silu else _lib.EPI_NONE, rank, world, 0, ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream().cuda_stream)
        torch.cuda.synchronize()
    assert rc == _lib.SIMSD_OK
    for y in ys:
        assert torch.equal(y[:, col_offset:col_offset + N], ref)
        assert bool(torch.isnan(y[:, :col_offset].float()).all())
        assert bool(torch.isnan(y[:, col_offset + N:].float()).all())
    assert _lib.device_error() == 0
