"""Layer ops of the verify forward around its linears, on libsimsd_b200.

* `rmsnorm(x, weight, eps, residual=None)` — the fp32 RMSNorm the SDAR runners
  install (sdar/run_native_tp2.py:34-51), optionally fused with the residual add
  before it: returns y, or (h, y) with h = x + residual.
* `qk_norm_rope(qkv, ...)` — the attention front end (sdar/modeling_sdar.py
  :197-302): per-head q/k RMSNorm, rotary embedding, and the K/V write into a
  static cache, from the merged q/k/v projection output.

Forward-only; CUDA tensors only (no CPU fallback).
"""
from __future__ import annotations

import torch

from . import _lib


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    if x.dtype not in (torch.bfloat16, torch.float16) or weight.dtype != x.dtype:
        raise TypeError(f"rmsnorm takes bf16/fp16 x and weight of the same type, got {x.dtype}/{weight.dtype}")
    n = x.shape[-1]
    if weight.shape != (n,):
        raise ValueError(f"weight must be [{n}]")
    if residual is not None and residual.shape != x.shape:
        raise ValueError("residual must have x's shape")
    dev = _lib.require_cuda(x, weight, residual)
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    rows = x2.shape[0]
    y = torch.empty((rows, n), dtype=x.dtype, device=dev)
    h = None
    r2 = None
    if residual is not None:
        r2 = residual.reshape(-1, n)
        if r2.stride(-1) != 1:
            r2 = r2.contiguous()
        h = torch.empty((rows, n), dtype=x.dtype, device=dev)
    w = weight.contiguous()
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_rmsnorm(
            x2.data_ptr(), x2.stride(0), r2.data_ptr() if r2 is not None else None, r2.stride(0) if r2 is not None else 0,
            h.data_ptr() if h is not None else None, n, w.data_ptr(), y.data_ptr(), n, rows, n, float(eps),
            _lib.dtype_code(x.dtype), _lib.stream_ptr(dev))
    _lib.check(rc, "rmsnorm")
    y = y.view(x.shape)
    return y if residual is None else (h.view(x.shape), y)


def qk_norm_rope(qkv: torch.Tensor, heads: int, kv_heads: int, q_weight: torch.Tensor, k_weight: torch.Tensor,
                 cos: torch.Tensor, sin: torch.Tensor, eps: float, k_cache: torch.Tensor, v_cache: torch.Tensor,
                 pos: int) -> torch.Tensor:
    """qkv [L, (heads + 2 kv_heads) * 128] -> q [heads, L, 128]; writes the
    rotated, normed k and the v of the L tokens at cache rows pos .. pos + L - 1
    of k_cache / v_cache [kv_heads, cap, 128] (contiguous)."""
    D = 128
    L = qkv.shape[0]
    if qkv.ndim != 2 or qkv.shape[1] != (heads + 2 * kv_heads) * D or qkv.stride(1) != 1:
        raise ValueError(f"qkv must be [L, {(heads + 2 * kv_heads) * D}] with unit column stride")
    for t in (q_weight, k_weight, cos, sin, k_cache, v_cache):
        if t.dtype != qkv.dtype:
            raise TypeError("qk_norm_rope: every tensor must have qkv's dtype")
    if cos.shape != (L, D) or sin.shape != (L, D) or not cos.is_contiguous() or not sin.is_contiguous():
        raise ValueError(f"cos/sin must be contiguous [{L}, {D}]")
    if k_cache.shape != v_cache.shape or k_cache.shape[0] != kv_heads or k_cache.shape[2] != D \
            or not k_cache.is_contiguous() or not v_cache.is_contiguous():
        raise ValueError(f"caches must be contiguous [{kv_heads}, cap, {D}]")
    dev = _lib.require_cuda(qkv, q_weight, k_weight, cos, sin, k_cache, v_cache)
    q = torch.empty((heads, L, D), dtype=qkv.dtype, device=dev)
    with _lib.device_guard(dev):
        rc = _lib.lib().simsd_qk_norm_rope(
            qkv.data_ptr(), qkv.stride(0), L, heads, kv_heads, D, q_weight.contiguous().data_ptr(),
            k_weight.contiguous().data_ptr(), cos.data_ptr(), sin.data_ptr(), float(eps), q.data_ptr(),
            k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[1], int(pos), _lib.dtype_code(qkv.dtype),
            _lib.stream_ptr(dev))
    _lib.check(rc, "qk_norm_rope")
    return q


def verify_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, Lk: int, mask: torch.Tensor,
                     scale: float) -> torch.Tensor:
    """GQA attention of q [Hq, L, 128] over keys [0, Lk) of k_cache / v_cache
    [Hk, cap, 128] under mask [L, >= Lk] (bool, True = attend) -> o [L, Hq * 128],
    the layout the output projection reads.  bf16, contiguous operands."""
    Hq, L, D = q.shape
    Hk = k_cache.shape[0]
    if q.dtype != torch.bfloat16 or k_cache.dtype != q.dtype or v_cache.dtype != q.dtype:
        raise TypeError("verify_attention takes bf16 q / k_cache / v_cache")
    if D != 128 or k_cache.shape != v_cache.shape or k_cache.shape[2] != 128 or Hq % Hk != 0:
        raise ValueError("head_dim 128, Hq a multiple of Hk, k_cache and v_cache alike")
    if mask.dtype != torch.bool or mask.ndim != 2 or mask.shape[0] != L or mask.shape[1] < Lk or mask.stride(1) != 1:
        raise ValueError(f"mask must be a bool [{L}, >= {Lk}] with unit column stride")
    if not (q.is_contiguous() and k_cache.is_contiguous() and v_cache.is_contiguous()):
        raise ValueError("q, k_cache and v_cache must be contiguous")
    dev = _lib.require_cuda(q, k_cache, v_cache, mask)
    o = torch.empty((L, Hq * D), dtype=q.dtype, device=dev)
    L_ = _lib.lib()
    with _lib.device_guard(dev):
        ws = _lib.workspace(dev, L_.simsd_verify_attention_workspace_size(Hq, Hk, L, Lk))
        rc = L_.simsd_verify_attention(q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[1], Hq, Hk,
                                       L, Lk, mask.data_ptr(), mask.stride(0), float(scale), o.data_ptr(),
                                       _lib.dtype_code(q.dtype), ws.data_ptr(), ws.numel(), _lib.stream_ptr(dev))
    _lib.check(rc, "verify_attention")
    return o
