"""The SDAR verify forward with its linears split across GPUs (BASELINE
"linears sharded at 1/2/4/8 GPUs").

Every linear of the target - the merged q/k/v, o_proj, the fused gate/up,
down_proj and lm_head - is split by output column over the ranks of a node
(rank r holds rows [r N/g, (r+1) N/g) of the weight; gate and up at the same
rows, so SiLU(gate) * up stays local), and its output is all-gathered by the
GEMM itself (`FusedAllGather`: NVLink peer stores + device counters, a bounded
wait before each reader).  Embedding, RMSNorms, q/k norm + rotary + cache
write and the verify attention are replicated on every rank, over a replicated
static KV cache.  The reference runs its target tensor-parallel through
transformers' `tp_plan="auto"` (main_table/run_native_tp2_cache.py:90-127): q/k/v
and gate/up column-wise as here, o/down row-wise with an all-reduce, lm_head
column-wise with the logits replicated ("colwise_rep", sdar/modeling_sdar.py:743).
Column-splitting o and down as well keeps every output element's K reduction
on one GPU: with each split pinned to the single-GPU K split (`plan_n`), the
sharded forward computes the single-GPU fused forward's hidden states and
greedy tokens bit for bit, which a row-wise all-reduce (a different summation
order) could not.

Collective: every rank builds it from the same model (same seed) and makes the
same calls in the same order.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from .layer_ops import qk_norm_rope, rmsnorm, verify_attention
from .parallel import FusedAllGather, column_shard
from .sdar_verify import SDARVerifyModel, VerifyHarness, rope_cos_sin


class ShardedVerify:
    """Column-parallel verify forward over the window of a `VerifyHarness`."""

    def __init__(self, model: SDARVerifyModel, group=None):
        self.model = model
        self.s = model.s
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.ag = FusedAllGather(group)
        r, g = self.rank, self.world
        self.layers = []
        with torch.no_grad():
            for layer in model.layers:
                a, m = layer.self_attn, layer.mlp
                qkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight])
                self.layers.append({
                    "qkv": column_shard(qkv, r, g),
                    "o": column_shard(a.o_proj.weight, r, g),
                    "gate": column_shard(m.gate_proj.weight, r, g),
                    "up": column_shard(m.up_proj.weight, r, g),
                    "down": column_shard(m.down_proj.weight, r, g),
                })
                del qkv
            self.lm_head = column_shard(model.lm_head.weight, r, g)
        s = self.s
        self.n_qkv = (s.heads + 2 * s.kv_heads) * s.head_dim
        self.n_o = s.hidden
        self.n_mlp = s.intermediate

    def window_hidden(self, h: VerifyHarness) -> torch.Tensor:
        """The final-norm hidden states [1, L, H] of the window (the lm_head
        input), as SDARVerifyModel.hidden(fused=True) computes them."""
        m, s, ag = self.model, self.s, self.ag
        ids, positions, mask, pos = h.win_ids, h.win_pos, h.window_mask, h.P
        x0 = m.embed_tokens(ids)
        L, H = x0.shape[1], x0.shape[2]
        cos, sin = rope_cos_sin(positions, s.head_dim, s.rope_theta, x0.dtype)
        x = rmsnorm(x0, m.layers[0].input_layernorm.weight, m.layers[0].input_layernorm.eps)
        res = x0
        n = len(m.layers)
        for i, (layer, w) in enumerate(zip(m.layers, self.layers)):
            a = layer.self_attn
            kc, vc = h.caches[i]
            qkv = ag.linear(x.reshape(L, H), w["qkv"], plan_n=self.n_qkv)
            q = qk_norm_rope(qkv, s.heads, s.kv_heads, a.q_norm.weight, a.k_norm.weight, cos, sin, a.q_norm.eps,
                             kc[0], vc[0], pos)
            o = verify_attention(q, kc[0], vc[0], pos + L, mask[0, 0], s.head_dim ** -0.5)
            att = ag.linear(o.view(L, -1), w["o"], plan_n=self.n_o).view(1, L, H)
            pn = layer.post_attention_layernorm
            res, x = rmsnorm(att, pn.weight, pn.eps, residual=res)
            mid = ag.linear(x.reshape(L, H), w["gate"], w["up"], plan_n=self.n_mlp)
            mlp = ag.linear(mid, w["down"], plan_n=self.n_o).view(1, L, H)
            nn_ = m.layers[i + 1].input_layernorm if i + 1 < n else m.norm
            res, x = rmsnorm(mlp, nn_.weight, nn_.eps, residual=res)
        return x

    def window_logits(self, h: VerifyHarness) -> torch.Tensor:
        """[L, vocab] logits: the column-split lm_head, gathered."""
        x = self.window_hidden(h)[0]
        return self.ag.linear(x, self.lm_head, plan_n=self.s.vocab)

    def window_argmax(self, h: VerifyHarness) -> torch.Tensor:
        """The greedy target token of every window row, [L] int64 (ties to the
        lowest id, as torch.argmax and the single-GPU fused head)."""
        return self.window_logits(h).argmax(-1)

    def close(self) -> None:
        self.ag.close()
