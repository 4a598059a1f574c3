"""libsimsd_b200.so loads without a GPU, exports every symbol the header declares,
and rejects bad arguments before touching a device."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
HEADER = REPO / "include" / "simsd_b200.h"


def header_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(simsd_\w+)\s*\(", text))


@pytest.fixture(scope="module")
def L():
    from kernels import _lib
    return _lib.lib()


def test_library_exports_every_declared_symbol(L):
    from kernels import _lib
    names = header_functions()
    assert len(names) >= 12
    for n in names:
        assert hasattr(L, n), f"{n} not exported"
    assert names == set(_lib.SIGNATURES), "ctypes signatures must cover exactly the header"


def test_static_queries(L):
    assert b"sm_100a" in L.simsd_version()
    assert L.simsd_workspace_header_bytes() == 256 * 1024
    assert L.simsd_status_string(0) == b"ok"
    assert L.simsd_status_string(-3).startswith(b"workspace")
    # workspace sizes are pure arithmetic
    small = L.simsd_thin_linear_workspace_size(4, 2048, 2048, 0, 0, 0)
    big = L.simsd_thin_linear_workspace_size(64, 2048, 2048, 0, 0, 0)
    assert 256 * 1024 < small < big
    assert L.simsd_moe_workspace_size(1024, 8, 256, 2048, 512, 0) > 2 * 8192 * 2048 * 2 + 8192 * 512 * 2


def test_argument_validation_happens_before_device_work(L):
    from kernels import _lib
    buf = ctypes.create_string_buffer(16)
    p = ctypes.cast(buf, ctypes.c_void_p).value
    # bad shape
    assert L.simsd_thin_linear(p, 1, 1, p, 1, 1, None, None, p, 1, 0, 1, 1, 0, 0, 0, 0, p, 1 << 20, None) \
        == _lib.SIMSD_ERR_SHAPE
    # bad dtype
    assert L.simsd_thin_linear(p, 1, 1, p, 1, 1, None, None, p, 1, 1, 1, 1, 7, 0, 0, 0, p, 1 << 20, None) \
        == _lib.SIMSD_ERR_DTYPE
    # SiLU-mul without the up weight
    assert L.simsd_thin_linear(p, 1, 1, p, 1, 1, None, None, p, 1, 1, 1, 1, 0, 1, 0, 0, p, 1 << 20, None) \
        == _lib.SIMSD_ERR_UNSUPPORTED
    # missing workspace
    assert L.simsd_thin_linear(p, 1, 1, p, 1, 1, None, None, p, 1, 1, 1, 1, 0, 0, 0, 0, None, 0, None) \
        == _lib.SIMSD_ERR_WORKSPACE
    # router: k > E, E too large
    assert L.simsd_moe_route(p, 1, 0, p, 1, 0, None, 1, 8, 4, 5, 1, 1.0, p, p, None, None) \
        == _lib.SIMSD_ERR_SHAPE
    assert L.simsd_moe_route(p, 1, 0, p, 1, 0, None, 1, 8, 2048, 2, 1, 1.0, p, p, None, None) \
        == _lib.SIMSD_ERR_SHAPE
    # align: padded layout half-specified
    assert L.simsd_moe_align(p, 4, 8, p, p, p, p, 16, 4, p, None, p, None) == _lib.SIMSD_ERR_SHAPE
    # dispatch: bad dtype, E too large
    assert L.simsd_moe_dispatch(p, 1, p, p, p, p, 1, 1, p, 1, 1, p, 1, None, 0, 1, 1, 4, 8, 8, 9,
                                p, 1 << 20, None) == _lib.SIMSD_ERR_DTYPE
    assert L.simsd_moe_dispatch(p, 1, p, p, p, p, 1, 1, p, 1, 1, p, 1, None, 0, 1, 1, 4096, 8, 8, 0,
                                p, 1 << 20, None) == _lib.SIMSD_ERR_SHAPE


def test_launch_flags_round_trip():
    """Every documented launch flag is kept by simsd_set_launch_flags (no GPU needed)."""
    from kernels import _lib
    L = _lib.lib()
    prev = L.simsd_get_launch_flags()
    try:
        for bit in (_lib.LAUNCH_PDL, _lib.LAUNCH_INKERNEL_REDUCE, _lib.LAUNCH_GROUPED_FIXUP,
                    _lib.LAUNCH_MOE_SIZE_CLASSES):
            L.simsd_set_launch_flags(bit)
            assert L.simsd_get_launch_flags() == bit
        with _lib.moe_size_classes(True):
            assert L.simsd_get_launch_flags() & _lib.LAUNCH_MOE_SIZE_CLASSES
    finally:
        L.simsd_set_launch_flags(prev)
