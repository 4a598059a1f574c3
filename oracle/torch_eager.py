"""Torch eager restatement of the reference's CPU path for the hot path.

TEST INFRASTRUCTURE / BASELINE ONLY: used by tests/ and by bench.py's CPU
baseline leg (`cpu_baseline`, `--impl reference`), never by the product.

* `linear` / `silu_mul`: the ground truth of kernels/thin_linear_fused.py
  (`F.linear`, kernels/workspace/thin_linear/CONTRACT.md) and SDARMLP's
  `act_fn(gate_proj(x)) * up_proj(x)` (sdar/modeling_sdar.py:113-119).
* `moe_infer`: the stock LLaDA2 `moe_infer` as the reference transcribes it
  (kernels/workspace/moe_dispatch/build_oracle.py:34-67): slots sorted by
  expert, one F.linear chain per active expert, outputs scattered back, then the
  fp32 weighted sum over k cast to x.dtype.
* `route`: sigmoid scores, top-k on score + bias, the chosen scores renormalised
  (+1e-20) and scaled (build_oracle.py:71-90 with the selection bias).
"""
from __future__ import annotations

import torch
import torch.nn.functional as F


def linear(x, w, bias=None):
    return F.linear(x, w, bias)


def silu_mul(x, w_gate, w_up):
    return F.silu(F.linear(x, w_gate)) * F.linear(x, w_up)


def moe_infer(x, topk_ids, topk_weight, w_gate, w_up, w_down):
    T, k = topk_ids.shape
    E = w_gate.shape[0]
    flat = topk_ids.reshape(-1)
    order = torch.argsort(flat, stable=True)
    counts = torch.bincount(flat, minlength=E).tolist()   # the stock path's host sync
    rows = x[order // k]
    outs = []
    start = 0
    for e, n in enumerate(counts):
        if n == 0:
            continue
        h = rows[start:start + n]
        outs.append(F.linear(F.silu(F.linear(h, w_gate[e])) * F.linear(h, w_up[e]), w_down[e]))
        start += n
    y = torch.cat(outs) if outs else rows.new_empty(0, x.shape[1])
    back = torch.empty_like(y)
    back[order] = y
    return (back.view(T, k, -1).to(topk_weight.dtype) * topk_weight.unsqueeze(-1)).sum(1).to(x.dtype)


def route(x, w_router, bias, k, renorm=True, scale=1.0):
    s = torch.sigmoid(F.linear(x.float(), w_router.float()))
    choice = s + bias if bias is not None else s
    ids = choice.topk(k, dim=-1).indices
    w = s.gather(1, ids)
    if renorm and k > 1:
        w = w / (w.sum(-1, keepdim=True) + 1e-20)
    return ids, (w * scale).float()


def moe_layer(x, w_router, bias, k, w_gate, w_up, w_down, shared=None, scale=1.0):
    ids, w = route(x, w_router, bias, k, scale=scale)
    out = moe_infer(x, ids, w, w_gate, w_up, w_down)
    if shared is not None:
        sg, su, sd = shared
        out = out + F.linear(silu_mul(x, sg, su), sd)
    return out


def thin_sweep_step(weights, xs, shapes, ms):
    """One step of the SDAR-8B thin-M sweep on the CPU (bench's CPU baseline)."""
    out = []
    for M in ms:
        for name, K, N, silu in shapes:
            x = xs[M][K]
            if silu:
                gu = F.linear(x, weights[name])
                out.append(F.silu(gu[:, : N // 2]) * gu[:, N // 2:])
            else:
                out.append(F.linear(x, weights[name]))
    return out
