"""numpy/ctypes front end of the CPU oracle (oracle/simsd_oracle.c).

TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's CPU
baseline may import this module; the product never does.  Each function
restates a reference algorithm (file:line given in simsd_oracle.c) on numpy
arrays; bf16 values travel as uint16 bit patterns.
"""
from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB = HERE / "liboracle.so"
DT_BF16, DT_F16, DT_F32 = 0, 1, 2

_lib = None


def build(force: bool = False) -> Path:
    src = HERE / "simsd_oracle.c"
    if force or not LIB.exists() or LIB.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(HERE), "-B" if force else "liboracle.so"],
                       check=True, capture_output=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(str(LIB))
        P, I, L64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        L.oracle_thin_linear.argtypes = [P, L64, L64, P, L64, L64, P, I, I, I, I, P, P]
        L.oracle_thin_linear_silu_mul.argtypes = [P, L64, P, P, L64, I, I, I, I, P, P]
        L.oracle_route.argtypes = [P, L64, I, P, L64, I, P, I, I, I, I, I, F, P, P, P]
        L.oracle_align.argtypes = [P, I, I, P, P, P, P, I, I, P, P]
        L.oracle_align.restype = I
        L.oracle_moe_dispatch.argtypes = [P, P, P, P, P, P, P, I, I, I, I, I, I, I, P, P]
        _lib = L
    return _lib


# ------------------------------------------------------------------ bf16 helpers
def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (uint16)."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def _dt(a: np.ndarray) -> int:
    if a.dtype == np.uint16:
        return DT_BF16
    if a.dtype == np.float16:
        return DT_F16
    if a.dtype == np.float32:
        return DT_F32
    raise TypeError(f"oracle arrays are bf16 bits (uint16), float16 or float32, got {a.dtype}")


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


# ------------------------------------------------------------------ thin linear
def thin_linear(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None):
    """(acc fp32 [M,N], y [M,N] in x's dtype) of y = x w^T (+ bias), fp32 accumulate."""
    x = np.ascontiguousarray(x)
    w = np.ascontiguousarray(w)
    dt = _dt(x)
    M, K = x.shape
    N = w.shape[0]
    acc = np.empty((M, N), np.float32)
    y = np.empty((M, N), x.dtype)
    b = None if bias is None else np.ascontiguousarray(bias)
    lib().oracle_thin_linear(_p(x), K, 1, _p(w), K, 1, _p(b), M, N, K, dt, _p(acc), _p(y))
    return acc, y


def thin_linear_silu_mul(x: np.ndarray, wg: np.ndarray, wu: np.ndarray):
    """(acc fp32 [M,I], y [M,I]) of silu(x wg^T) * (x wu^T), products in fp32."""
    x, wg, wu = (np.ascontiguousarray(a) for a in (x, wg, wu))
    dt = _dt(x)
    M, K = x.shape
    I = wg.shape[0]
    acc = np.empty((M, I), np.float32)
    y = np.empty((M, I), x.dtype)
    lib().oracle_thin_linear_silu_mul(_p(x), K, _p(wg), _p(wu), K, M, I, K, dt, _p(acc), _p(y))
    return acc, y


# ------------------------------------------------------------------ router
def route(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None, k: int, renorm: bool = True,
          scale: float = 1.0):
    """(ids int64 [T,k], weights fp32 [T,k], logits fp32 [T,E]) with the fixed router arithmetic."""
    x, w = np.ascontiguousarray(x), np.ascontiguousarray(w)
    T, H = x.shape
    E = w.shape[0]
    ids = np.empty((T, k), np.int64)
    wts = np.empty((T, k), np.float32)
    logits = np.empty((T, E), np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    lib().oracle_route(_p(x), H, _dt(x), _p(w), H, _dt(w), _p(b), T, H, E, k, int(renorm),
                       ctypes.c_float(scale), _p(ids), _p(wts), _p(logits))
    return ids, wts, logits


# ------------------------------------------------------------------ align
def align(ids: np.ndarray, E: int, block_m: int = 16, num_tiles: int | None = None):
    flat = np.ascontiguousarray(ids.reshape(-1), dtype=np.int64)
    S = flat.size
    if num_tiles is None:
        num_tiles = min(E, S) + (S + block_m - 1) // block_m
    out = {
        "counts": np.empty(E, np.int32), "offsets": np.empty(E + 1, np.int32),
        "sorted_slots": np.empty(S, np.int32), "slot_to_row": np.empty(S, np.int32),
        "slots": np.empty(num_tiles * block_m, np.int32), "tile_expert": np.empty(num_tiles, np.int32),
    }
    rc = lib().oracle_align(_p(flat), S, E, _p(out["counts"]), _p(out["offsets"]),
                            _p(out["sorted_slots"]), _p(out["slot_to_row"]), block_m, num_tiles,
                            _p(out["slots"]), _p(out["tile_expert"]))
    out["status"] = rc
    return out


# ------------------------------------------------------------------ MoE dispatch
def moe_dispatch(x, ids, w, wg, wu, wd, add=None, mode: int = 0):
    """(acc fp32 [T,H], out [T,H]); mode 0 = stock moe_infer rounding, 1 = fused numerics."""
    x, wg, wu, wd = (np.ascontiguousarray(a) for a in (x, wg, wu, wd))
    ids = np.ascontiguousarray(ids, dtype=np.int64)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, H = x.shape
    k = ids.shape[1]
    E, I, _ = wg.shape
    acc = np.empty((T, H), np.float32)
    out = np.empty((T, H), x.dtype)
    a = None if add is None else np.ascontiguousarray(add)
    lib().oracle_moe_dispatch(_p(x), _p(ids), _p(w), _p(wg), _p(wu), _p(wd), _p(a), T, k, E, H, I,
                              _dt(x), mode, _p(acc), _p(out))
    return acc, out


def _to_f32(a: np.ndarray) -> np.ndarray:
    if a.dtype == np.uint16:
        return bf16_bits_to_f32(a)
    return np.ascontiguousarray(a, dtype=np.float32)


def _round_to(a: np.ndarray, dt: int) -> np.ndarray:
    """fp32 values rounded to the activation type (kept as fp32 values)."""
    if dt == DT_BF16:
        return bf16_bits_to_f32(f32_to_bf16_bits(a))
    if dt == DT_F16:
        return a.astype(np.float16).astype(np.float32)
    return a.astype(np.float32)


def _from_f32(a: np.ndarray, dt: int) -> np.ndarray:
    if dt == DT_BF16:
        return f32_to_bf16_bits(a)
    if dt == DT_F16:
        return a.astype(np.float16)
    return a.astype(np.float32)


def _silu(g: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def moe_dispatch_grouped(x, ids, w, wg, wu, wd, add=None, mode: int = 0):
    """The arithmetic of `moe_dispatch` (same rounding points as modes 0 / 1 of
    the C oracle) with the products grouped by expert and formed by numpy's
    fp32 matrix products, for the layer sizes the C loop is too slow for
    (1.4 TFLOP at T = 4096).  Only the summation order
    of each dot product differs from the C oracle; tests/test_oracle_golden.py
    pins the two to each other.  Returns (acc fp32 [T,H], out [T,H])."""
    dt = _dt(np.asarray(x))
    X = _to_f32(np.asarray(x))
    ids = np.asarray(ids, dtype=np.int64)
    w = np.asarray(w, dtype=np.float32)
    T, k = ids.shape
    E = wg.shape[0]
    H = X.shape[1]
    flat = ids.reshape(-1)
    Y = np.zeros((T * k, H), np.float32)
    for e in np.unique(flat):
        if e < 0 or e >= E:
            continue
        slots = np.nonzero(flat == e)[0]
        xe = X[slots // k]
        g = xe @ _to_f32(wg[e]).T
        u = xe @ _to_f32(wu[e]).T
        if mode == 0:
            g, u = _round_to(g, dt), _round_to(u, dt)
            h = _round_to(_round_to(_silu(g), dt) * u, dt)
        else:
            h = _round_to(_silu(g) * u, dt)
        Y[slots] = _round_to(h @ _to_f32(wd[e]).T, dt)
    acc = np.zeros((T, H), np.float32)
    Yt = Y.reshape(T, k, H)
    for j in range(k):
        valid = ((ids[:, j] >= 0) & (ids[:, j] < E))[:, None]
        acc = np.where(valid, acc + Yt[:, j] * w[:, j:j + 1], acc).astype(np.float32)
    v = acc
    if add is not None:
        v = _round_to(acc, dt) + _to_f32(np.asarray(add))
    return acc, _from_f32(v, dt)


def dense_swiglu(x, wg, wu, wd, mode: int = 1):
    """down(silu(gate(x)) * up(x)) for one dense (shared) expert [I,H],[I,H],[H,I],
    rounded like moe_dispatch_grouped's experts; returns it in x's type."""
    dt = _dt(np.asarray(x))
    ids = np.zeros((np.asarray(x).shape[0], 1), np.int64)
    ones = np.ones(ids.shape, np.float32)
    _, out = moe_dispatch_grouped(x, ids, ones, np.asarray(wg)[None], np.asarray(wu)[None],
                                  np.asarray(wd)[None], mode=mode)
    return out


def ep_plan(ids: np.ndarray, E: int, world: int, cap: int):
    """Per-peer buckets of slots for the expert-parallel MoE layer (numpy).

    The reference runs its MoE layer on one GPU and has no such step; this is
    the contract of simsd_moe_ep_plan, restated for the checks: expert e lives
    on rank e // (E // world) as local expert e % (E // world); each peer's
    slots, in slot order (the stable order moe_infer's argsort gives within an
    expert, kernels/workspace/moe_dispatch/build_oracle.py:34-67), fill its
    bucket from position 0; slots past `cap` or with ids outside [0, E) are not
    sent (slot_pos -1).
    """
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    epr = E // world
    send_slot = np.full(world * cap, -1, np.int32)
    send_expert = np.full(world * cap, -1, np.int32)
    slot_pos = np.full(flat.size, -1, np.int32)
    counts = np.zeros(world, np.int32)
    for s, e in enumerate(flat):
        if e < 0 or e >= E:
            continue
        peer = int(e) // epr
        pos = counts[peer]
        counts[peer] += 1
        if pos < cap:
            send_slot[peer * cap + pos] = s
            send_expert[peer * cap + pos] = int(e) - peer * epr
            slot_pos[s] = peer * cap + pos
    return {"send_slot": send_slot, "send_expert": send_expert, "slot_pos": slot_pos, "counts": counts}
