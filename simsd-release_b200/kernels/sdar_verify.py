"""Synthetic SDAR-shaped target for the multi-block verify.

The caller side of the thin-M linear: a random-init decoder with SDAR's
architecture (sdar/modeling_sdar.py — SDARMLP :99-119, rotary :129-153 and
:398-435, SDARAttention :197-302 with q/k RMSNorm over head_dim and GQA,
SDARDecoderLayer :324-367, model :520-563, lm_head :842) and the stock fp32
RMSNorm that the runners install (sdar/run_native_tp2.py:34-51), plus the
verify-time pieces that feed it:

* `build_verify_sequence_multi` — the multi-draft-block layout of
  speculative_decoding/verify.py:350-418 ([prompt | acc data | D_k data, D_k mask]);
* `multi_block_causal_mask` — the visibility rules of
  sdar/new_attn_multi_block.py:22-186;
* `greedy_match_verify` — speculative_decoding/mrs.py:111-145;
* `VerifyHarness` — prefill of a prompt into a KV prefix, then the K-block verify
  forward over the 2·bl·K query rows (verify.py:421-547 with a cached prefix),
  capturable in a CUDA graph.

Its linears are plain `nn.Linear` modules named like SDAR's, so
`fused_toggle.apply_to_model` swaps them exactly as it does in the real model;
attention stays on torch SDPA.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn as nn
import torch.nn.functional as F

MASK_TOKEN_ID = 151669   # speculative_decoding/verify.py:9


@dataclass
class SDARShape:
    hidden: int = 4096
    layers: int = 36
    heads: int = 32
    kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 12288
    vocab: int = 151936
    rope_theta: float = 1e6
    eps: float = 1e-6

    @property
    def linear_params(self) -> int:
        h, d = self.hidden, self.head_dim
        per = h * (self.heads * d) + 2 * h * (self.kv_heads * d) + (self.heads * d) * h + 3 * h * self.intermediate
        return per * self.layers


SDAR_8B = SDARShape()


class RMSNorm(nn.Module):
    """fp32 mean-square normalisation, weight applied in the input dtype."""

    def __init__(self, n: int, eps: float):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(n))
        self.eps = eps

    def forward(self, x):
        dt = x.dtype
        x32 = x.to(torch.float32)
        x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + self.eps)
        return self.weight * x32.to(dt)


def rope_cos_sin(positions: torch.Tensor, head_dim: int, theta: float, dtype):
    """cos/sin [L, head_dim] of the default rotary embedding, computed in fp32."""
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=positions.device, dtype=torch.float32) / head_dim))
    freqs = positions.to(torch.float32)[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def _rotate_half(x):
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


class Attention(nn.Module):
    def __init__(self, s: SDARShape):
        super().__init__()
        self.s = s
        self.q_proj = nn.Linear(s.hidden, s.heads * s.head_dim, bias=False)
        self.k_proj = nn.Linear(s.hidden, s.kv_heads * s.head_dim, bias=False)
        self.v_proj = nn.Linear(s.hidden, s.kv_heads * s.head_dim, bias=False)
        self.o_proj = nn.Linear(s.heads * s.head_dim, s.hidden, bias=False)
        self.q_norm = RMSNorm(s.head_dim, s.eps)
        self.k_norm = RMSNorm(s.head_dim, s.eps)

    def forward(self, h, cos, sin, mask, past=None, cache=None, pos=0):
        """past: prefix (k, v) to concatenate; cache: static (k_cache, v_cache)
        [1, Hk, cap, D] whose rows [pos, pos + L) take this call's k/v and whose
        rows [0, pos + L) are attended (the reference's static block cache)."""
        B, L, _ = h.shape
        s = self.s
        q = self.q_norm(self.q_proj(h).view(B, L, s.heads, s.head_dim)).transpose(1, 2)
        k = self.k_norm(self.k_proj(h).view(B, L, s.kv_heads, s.head_dim)).transpose(1, 2)
        v = self.v_proj(h).view(B, L, s.kv_heads, s.head_dim).transpose(1, 2)
        c, si = cos[None, None], sin[None, None]
        q = q * c + _rotate_half(q) * si
        k = k * c + _rotate_half(k) * si
        if cache is not None:
            cache[0][:, :, pos:pos + L].copy_(k)
            cache[1][:, :, pos:pos + L].copy_(v)
            k, v = cache[0][:, :, :pos + L], cache[1][:, :, :pos + L]
        elif past is not None:
            k = torch.cat([past[0], k], dim=2)
            v = torch.cat([past[1], v], dim=2)
        o = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, scale=s.head_dim ** -0.5, enable_gqa=True)
        o = o.transpose(1, 2).reshape(B, L, -1)
        return self.o_proj(o), (k, v)

    def forward_fused(self, x, cos, sin, mask, cache, pos):
        """The same with libsimsd_b200's layer ops: one merged q/k/v launch, then
        q/k RMSNorm + rotary + the cache write in one kernel, then GQA attention
        straight over the static cache (B = 1)."""
        from .layer_ops import qk_norm_rope, verify_attention
        from .thin_linear_fused import thin_linear_cat
        _, L, H = x.shape
        s = self.s
        qkv = thin_linear_cat(x.reshape(L, H), [self.q_proj.weight, self.k_proj.weight, self.v_proj.weight],
                              whole=True)
        q = qk_norm_rope(qkv, s.heads, s.kv_heads, self.q_norm.weight, self.k_norm.weight, cos, sin, self.q_norm.eps,
                         cache[0][0], cache[1][0], pos)
        o = verify_attention(q, cache[0][0], cache[1][0], pos + L, mask[0, 0], s.head_dim ** -0.5)
        return self.o_proj(o.view(1, L, -1))


class MLP(nn.Module):
    def __init__(self, s: SDARShape):
        super().__init__()
        self.gate_proj = nn.Linear(s.hidden, s.intermediate, bias=False)
        self.up_proj = nn.Linear(s.hidden, s.intermediate, bias=False)
        self.down_proj = nn.Linear(s.intermediate, s.hidden, bias=False)
        self.act_fn = nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


class DecoderLayer(nn.Module):
    def __init__(self, s: SDARShape):
        super().__init__()
        self.self_attn = Attention(s)
        self.mlp = MLP(s)
        self.input_layernorm = RMSNorm(s.hidden, s.eps)
        self.post_attention_layernorm = RMSNorm(s.hidden, s.eps)

    def forward(self, h, cos, sin, mask, past=None, cache=None, pos=0):
        a, kv = self.self_attn(self.input_layernorm(h), cos, sin, mask, past, cache, pos)
        h = h + a
        h = h + self.mlp(self.post_attention_layernorm(h))
        return h, kv


class SDARVerifyModel(nn.Module):
    def __init__(self, s: SDARShape = SDAR_8B):
        super().__init__()
        self.s = s
        self.embed_tokens = nn.Embedding(s.vocab, s.hidden)
        self.layers = nn.ModuleList(DecoderLayer(s) for _ in range(s.layers))
        self.norm = RMSNorm(s.hidden, s.eps)
        self.lm_head = nn.Linear(s.hidden, s.vocab, bias=False)

    @classmethod
    def random_init(cls, s: SDARShape = SDAR_8B, device="cuda", dtype=torch.bfloat16, seed: int = 0):
        """All matrices ~N(0, 0.02) (seeded, generated on `device`), norms = 1."""
        with torch.device("meta"):
            m = cls(s)
        m = m.to_empty(device=device).to(dtype)
        g = torch.Generator(device=device).manual_seed(seed)
        with torch.no_grad():
            for name, p in m.named_parameters():
                if name.endswith("norm.weight"):
                    p.fill_(1.0)
                else:
                    p.copy_(torch.randn(p.shape, generator=g, device=device, dtype=torch.float32).mul_(0.02))
        return m.eval()

    def hidden(self, ids, positions, mask, past=None, caches=None, pos=0, fused=False):
        """The final-norm hidden states [1, L, H] (the lm_head input) and the KV.

        caches: per-layer static (k_cache, v_cache) written at rows [pos, pos+L).
        fused (with caches): libsimsd_b200's layer ops — RMSNorms fused with the
        residual add before them, the merged q/k/v launch and the q/k norm +
        rotary + cache-write kernel — in place of the torch expressions.
        """
        h = self.embed_tokens(ids)
        cos, sin = rope_cos_sin(positions, self.s.head_dim, self.s.rope_theta, h.dtype)
        if fused and caches is not None:
            from .layer_ops import rmsnorm
            n = len(self.layers)
            x = rmsnorm(h, self.layers[0].input_layernorm.weight, self.layers[0].input_layernorm.eps)
            for i, layer in enumerate(self.layers):
                a = layer.self_attn.forward_fused(x, cos, sin, mask, caches[i], pos)
                pn = layer.post_attention_layernorm
                h, x = rmsnorm(a, pn.weight, pn.eps, residual=h)
                m = layer.mlp(x)
                nn_ = self.layers[i + 1].input_layernorm if i + 1 < n else self.norm
                h, x = rmsnorm(m, nn_.weight, nn_.eps, residual=h)
            return x, None
        kvs = []
        for i, layer in enumerate(self.layers):
            h, kv = layer(h, cos, sin, mask, None if past is None else past[i],
                          None if caches is None else caches[i], pos)
            kvs.append(kv)
        return self.norm(h), kvs

    def forward(self, ids, positions, mask, past=None):
        """ids [1, L]; positions [L]; mask [1, 1, L, L_past + L] bool; past: list of (k, v)."""
        h, kvs = self.hidden(ids, positions, mask, past)
        return self.lm_head(h), kvs


# ------------------------------------------------------------------ verify sequence
def build_verify_sequence_multi(prompt_ids, accepted_blocks, draft_blocks, step_maps, block_length, block_size,
                                mask_token_id=MASK_TOKEN_ID, share_mask_position=True):
    """(input_ids, token_labels, block_ids, positions) of the K-draft-block verify layout."""
    n = len(prompt_ids)
    ids, labels, blocks, pos = list(prompt_ids), [0] * n, [-1] * n, list(range(n))
    cur = n
    for b, toks in enumerate(accepted_blocks):
        ids += list(toks)
        labels += [1] * len(toks)
        blocks += [b] * len(toks)
        pos += list(range(cur, cur + len(toks)))
        cur += len(toks)
    M = len(accepted_blocks)
    for k, (draft, smap) in enumerate(zip(draft_blocks, step_maps)):
        data_pos = list(range(cur, cur + block_length))
        cur += block_length
        ids += list(draft)
        labels += [st + 1 if st >= 0 else block_size + 1 for st in smap]
        blocks += [M + k] * block_length
        pos += data_pos
        if share_mask_position:
            mask_pos = data_pos
        else:
            mask_pos = list(range(cur, cur + block_length))
            cur += block_length
        ids += [mask_token_id] * block_length
        labels += [block_size + 1] * block_length
        blocks += [M + k] * block_length
        pos += mask_pos
    return ids, labels, blocks, pos


def multi_block_causal_mask(token_labels: torch.Tensor, block_ids: torch.Tensor, block_size: int) -> torch.Tensor:
    """[L, L] bool visibility (True = key visible to query) for one sequence.

    prompt: block-causal over prompt blocks of `block_size`; data/mask tokens
    see the whole prompt; inside a block, data(t) sees data(<= t) and
    mask(> t), mask(t) sees data(< t) and mask(>= t), where a mask token's t is
    the step of the data token with the same rank in its block; a later block
    sees earlier blocks' data only; padding sees and is seen by nothing.
    """
    lab, blk = token_labels.tolist(), block_ids.tolist()
    L = len(lab)
    typ = [0 if l == 0 else (1 if 1 <= l <= block_size else (2 if l == block_size + 1 else -1)) for l in lab]
    t = [0.0 if ty == 0 else (float(l) if ty >= 1 else math.inf) for ty, l in zip(typ, lab)]
    # mask tokens take the step of the same-rank data token of their block
    data_by_blk, mask_by_blk = {}, {}
    for i, (ty, b) in enumerate(zip(typ, blk)):
        if b >= 0 and ty == 1:
            data_by_blk.setdefault(b, []).append(i)
        if b >= 0 and ty == 2:
            mask_by_blk.setdefault(b, []).append(i)
    for b, ms in mask_by_blk.items():
        ds = data_by_blk.get(b, [])
        for r, i in enumerate(ms):
            if r < len(ds):
                t[i] = t[ds[r]]
    dev = token_labels.device
    typ_t = torch.tensor(typ, device=dev)
    t_t = torch.tensor(t, device=dev)
    b_t = torch.tensor(blk, device=dev)
    is_p, is_d, is_m, is_pad = typ_t == 0, typ_t == 1, typ_t == 2, typ_t == -1
    pblk = (torch.cumsum(is_p.long(), 0) - 1) // block_size
    qi, kj = (slice(None), None), (None, slice(None))
    rule_prompt = is_p[qi] & is_p[kj] & (pblk[kj] <= pblk[qi])
    rule_see_prompt = (~is_p)[qi] & (~is_pad)[qi] & is_p[kj]
    same = (b_t[qi] == b_t[kj]) & (b_t[qi] >= 0)
    ti, tj = t_t[qi], t_t[kj]
    dd = same & is_d[qi] & is_d[kj] & (tj <= ti)
    dm = same & is_d[qi] & is_m[kj] & (tj > ti)
    md = same & is_m[qi] & is_d[kj] & (tj < ti)
    mm = same & is_m[qi] & is_m[kj] & (tj >= ti)
    cross = (b_t[qi] > b_t[kj]) & (b_t[kj] >= 0) & is_d[kj]
    vis = rule_prompt | rule_see_prompt | dd | dm | md | mm | cross
    return vis & (~is_pad)[qi] & (~is_pad)[kj]


def greedy_match_verify(draft_ids, target_argmax):
    """(accepted_ids, n_accepted, bonus): accept while draft == target argmax."""
    for pos, (d, a) in enumerate(zip(draft_ids, target_argmax)):
        if d != a:
            return list(draft_ids[:pos]) + [a], pos, a
    return list(draft_ids), len(draft_ids), None


# ------------------------------------------------------------------ harness
class VerifyHarness:
    """Prefill a prompt once, then run the K-block verify forward over the window.

    `window_logits()` is the timed op: 2·bl·K query rows through every layer
    against the cached prefix, returning [2·bl·K, vocab] logits.
    """

    def __init__(self, model: SDARVerifyModel, prompt_ids, draft_blocks, step_maps, block_length: int,
                 block_size: int | None = None):
        self.model = model
        self.bl = block_length
        self.bs = block_size or block_length
        self.K = len(draft_blocks)
        dev = next(model.parameters()).device
        ids, labels, blocks, pos = build_verify_sequence_multi(prompt_ids, [], draft_blocks, step_maps,
                                                               block_length, self.bs)
        self.P = len(prompt_ids)
        full = multi_block_causal_mask(torch.tensor(labels, device=dev), torch.tensor(blocks, device=dev), self.bs)
        self.ids = torch.tensor(ids, device=dev)[None]
        self.pos = torch.tensor(pos, device=dev)
        self.prefix_mask = full[: self.P, : self.P][None, None].contiguous()
        self.window_mask = full[self.P:, :][None, None].contiguous()
        with torch.inference_mode():
            _, self.past = model(self.ids[:, : self.P], self.pos[: self.P], self.prefix_mask)
        self.win_ids = self.ids[:, self.P:].clone()
        self.win_pos = self.pos[self.P:].clone()
        # static per-layer KV caches (the reference's static block cache): the
        # prefix rows once, the window rows rewritten by every verify forward
        cap = self.P + self.win_ids.shape[1]
        self.caches = []
        for k, v in self.past:
            kc = torch.zeros((1, k.shape[1], cap, k.shape[3]), dtype=k.dtype, device=dev)
            vc = torch.zeros_like(kc)
            kc[:, :, : self.P].copy_(k)
            vc[:, :, : self.P].copy_(v)
            self.caches.append((kc, vc))
        self.past = None
        self.fused = False      # True: libsimsd_b200's layer ops around the linears

    def set_drafts(self, draft_blocks, step_maps):
        """Replace the window's draft tokens / step maps in place (graph-safe)."""
        _, labels, blocks, _ = build_verify_sequence_multi([0] * self.P, [], draft_blocks, step_maps, self.bl, self.bs)
        dev = self.win_ids.device
        full = multi_block_causal_mask(torch.tensor(labels, device=dev), torch.tensor(blocks, device=dev), self.bs)
        w = []
        for d in draft_blocks:
            w += list(d) + [MASK_TOKEN_ID] * self.bl
        self.win_ids.copy_(torch.tensor(w, device=dev)[None])
        self.window_mask.copy_(full[self.P:, :][None, None])

    def window_hidden(self):
        h, _ = self.model.hidden(self.win_ids, self.win_pos, self.window_mask, caches=self.caches, pos=self.P,
                                 fused=self.fused)
        return h

    def window_logits(self):
        return self.model.lm_head(self.window_hidden())[0]

    def window_argmax(self):
        """The greedy target token of every window row, [L] int64, with the fused
        lm_head + argmax (no [L, vocab] logits)."""
        from .thin_linear_fused import thin_linear_argmax
        return thin_linear_argmax(self.window_hidden()[0], self.model.lm_head.weight)

    def window_argmax_via_logits(self):
        """The same from the logits, as the reference does (lm_head, then argmax)."""
        return self.window_logits().float().argmax(-1)

    def accept_ids(self, target_ids, draft_blocks):
        """accept() from per-row greedy targets [L] instead of logits."""
        out = []
        for k in range(self.K):
            arg = target_ids[self.mask_rows(k)].tolist()
            acc, n, bonus = greedy_match_verify(list(draft_blocks[k]), arg)
            out.append((acc, n, bonus))
            if bonus is not None:
                break
        return out

    def mask_rows(self, k: int) -> slice:
        start = k * 2 * self.bl + self.bl
        return slice(start, start + self.bl)

    def accept(self, logits, draft_blocks):
        """Greedy acceptance over the K blocks in order, stopping at the first reject."""
        out = []
        for k in range(self.K):
            arg = logits[self.mask_rows(k)].float().argmax(-1).tolist()
            acc, n, bonus = greedy_match_verify(list(draft_blocks[k]), arg)
            out.append((acc, n, bonus))
            if bonus is not None:
                break
        return out
