"""On-disk pre-packed stacked expert weights for the fused MoE dispatch.

The reference stacks each MoE layer's per-expert gate/up/down Linears into
[E, I, H] / [E, I, H] / [E, H, I] tensors at install time, in memory, every time
a model is loaded (`stack_expert_weights`, kernels/moe_dispatch_fused.py:195-217,
called from kernels/fused_toggle.py:151-198).  This module persists that layout
once, one file per MoE layer, so a later install reads the three stacked
tensors straight into device memory in the order the grouped GEMMs stream them
(no per-expert gathers, no host-side stacking copy, and the per-expert modules
need not be materialised at all).

File layout (little-endian):
  8 bytes   magic b"SIMSDEXP"
  8 bytes   header length n (uint64)
  n bytes   UTF-8 JSON header: {"version": 1, "E", "I", "H", "dtype",
            "arrays": [{"name", "shape", "offset", "nbytes", "crc32"}, ...]}
  data      each array's raw bytes (row-major, the dtype's bit patterns),
            starting at a 4096-byte aligned offset from the file start
Arrays: w_gate [E, I, H], w_up [E, I, H], w_down [E, H, I].  bf16/fp16/fp32.
`load_packed` checks magic, version, shapes, sizes and (by default) every
array's CRC-32, and raises ValueError on any mismatch.
"""
from __future__ import annotations

import json
import os
import zlib
from pathlib import Path

import numpy as np
import torch

MAGIC = b"SIMSDEXP"
VERSION = 1
ALIGN = 4096
NAMES = ("w_gate", "w_up", "w_down")
_DTYPES = {"bfloat16": torch.bfloat16, "float16": torch.float16, "float32": torch.float32}
_RAW = {torch.bfloat16: (torch.int16, np.int16), torch.float16: (torch.float16, np.float16),
        torch.float32: (torch.float32, np.float32)}


def _raw_numpy(t: torch.Tensor) -> np.ndarray:
    """The tensor's bit patterns as a contiguous CPU numpy array."""
    view_t, _ = _RAW[t.dtype]
    return t.detach().to("cpu").contiguous().view(view_t).numpy()


def pack_stacked(path, w_gate: torch.Tensor, w_up: torch.Tensor, w_down: torch.Tensor) -> Path:
    """Write already-stacked expert weights to `path` (atomically: a temporary
    file renamed into place)."""
    if w_gate.ndim != 3 or w_up.shape != w_gate.shape:
        raise ValueError("w_gate / w_up must be [E, I, H] and alike")
    E, I, H = w_gate.shape
    if tuple(w_down.shape) != (E, H, I):
        raise ValueError(f"w_down must be [{E}, {H}, {I}], got {tuple(w_down.shape)}")
    if not (w_gate.dtype == w_up.dtype == w_down.dtype) or w_gate.dtype not in _RAW:
        raise TypeError("the three stacks must share a dtype: bfloat16, float16 or float32")
    dtype_name = str(w_gate.dtype).removeprefix("torch.")
    raws = [_raw_numpy(t) for t in (w_gate, w_up, w_down)]
    arrays, off = [], 0
    for name, raw in zip(NAMES, raws):
        arrays.append({"name": name, "shape": list(raw.shape), "offset": 0, "nbytes": int(raw.nbytes),
                       "crc32": zlib.crc32(raw.tobytes()) & 0xFFFFFFFF})
    # offsets depend on the header length, which depends on the offsets' digits:
    # fix the header at a generous padded size first
    hdr_len = 4096
    off = ((16 + hdr_len + ALIGN - 1) // ALIGN) * ALIGN
    for a in arrays:
        a["offset"] = off
        off = ((off + a["nbytes"] + ALIGN - 1) // ALIGN) * ALIGN
    header = json.dumps({"version": VERSION, "E": E, "I": I, "H": H, "dtype": dtype_name,
                         "arrays": arrays}).encode()
    if len(header) > hdr_len:
        raise ValueError("expert pack header too large")
    header = header + b" " * (hdr_len - len(header))
    path = Path(path)
    tmp = path.with_name(path.name + f".tmp{os.getpid()}")
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(np.uint64(hdr_len).tobytes())
        f.write(header)
        for a, raw in zip(arrays, raws):
            f.seek(a["offset"])
            f.write(raw.tobytes())
        f.truncate(off)
    os.replace(tmp, path)
    return path


def pack_experts(path, experts) -> Path:
    """Stack a layer's per-expert modules (attributes gate_proj / up_proj /
    down_proj) and write them to `path`; the modules are left untouched."""
    from .moe_dispatch_fused import stack_expert_weights
    return pack_stacked(path, *stack_expert_weights(experts, free_originals=False))


def read_header(path) -> dict:
    with open(path, "rb") as f:
        magic = f.read(8)
        if magic != MAGIC:
            raise ValueError(f"{path}: not a simsd expert pack")
        n = int(np.frombuffer(f.read(8), dtype=np.uint64)[0])
        hdr = json.loads(f.read(n).decode())
    if hdr.get("version") != VERSION:
        raise ValueError(f"{path}: unsupported expert pack version {hdr.get('version')}")
    E, I, H = hdr["E"], hdr["I"], hdr["H"]
    want = {"w_gate": [E, I, H], "w_up": [E, I, H], "w_down": [E, H, I]}
    if hdr.get("dtype") not in _DTYPES or [a["name"] for a in hdr["arrays"]] != list(NAMES):
        raise ValueError(f"{path}: malformed expert pack header")
    esz = torch.empty((), dtype=_DTYPES[hdr["dtype"]]).element_size()
    size = os.path.getsize(path)
    for a in hdr["arrays"]:
        if a["shape"] != want[a["name"]] or a["nbytes"] != int(np.prod(a["shape"])) * esz \
                or a["offset"] % ALIGN or a["offset"] + a["nbytes"] > size:
            raise ValueError(f"{path}: array {a['name']} does not match the header")
    return hdr


def load_packed(path, device="cuda", verify: bool = True):
    """(w_gate, w_up, w_down) from a pack, on `device`: each array is mapped
    read-only from the file and copied to the device in one transfer."""
    hdr = read_header(path)
    dtype = _DTYPES[hdr["dtype"]]
    view_t, np_t = _RAW[dtype]
    mm = np.memmap(path, dtype=np.uint8, mode="r")
    out = []
    for a in hdr["arrays"]:
        raw = mm[a["offset"]: a["offset"] + a["nbytes"]]
        if verify and (zlib.crc32(raw) & 0xFFFFFFFF) != a["crc32"]:
            raise ValueError(f"{path}: checksum mismatch in {a['name']}")
        host = torch.from_numpy(np.asarray(raw).view(np_t).reshape(a["shape"]).copy()).view(dtype)
        out.append(host.to(device))
    del mm
    return tuple(out)
