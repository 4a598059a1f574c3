"""The verify-side restatements (kernels/sdar_verify.py) against the reference's
own outputs recorded in tests/golden/sdar_verify.npz: the SDAR decoder's logits
(sdar/modeling_sdar.py with patch_stock_rms_norm, tiny fp32 config), the
multi-block verify layout (speculative_decoding/verify.py:350-418), the mask
(sdar/new_attn_multi_block.py:22-186) and greedy acceptance (mrs.py:111-145)."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import torch

from kernels.sdar_verify import (SDARShape, SDARVerifyModel, build_verify_sequence_multi, greedy_match_verify,
                                 multi_block_causal_mask)

Z = np.load(Path(__file__).resolve().parent / "golden" / "sdar_verify.npz")
TINY = SDARShape(hidden=64, layers=2, heads=4, kv_heads=2, head_dim=16, intermediate=128, vocab=256, rope_theta=1e6)


def test_verify_sequence_layout_matches_reference():
    ids, labels, blocks, pos = build_verify_sequence_multi(list(range(10, 30)), [[40, 41, 42, 43]],
                                                           [[5, 6, 7, 8], [9, 10, 11, 12]],
                                                           [[0, 2, 1, 3], [3, 1, 0, 2]], 4, 4, mask_token_id=255)
    assert ids == Z["ids"].tolist() and labels == Z["labels"].tolist()
    assert blocks == Z["blocks"].tolist() and pos == Z["pos"].tolist()


def test_multi_block_mask_matches_reference():
    m = multi_block_causal_mask(torch.from_numpy(Z["labels"]), torch.from_numpy(Z["blocks"]), 4)
    assert torch.equal(m, torch.from_numpy(Z["mask"]))


def test_decoder_logits_match_reference_bit_for_bit():
    model = SDARVerifyModel(TINY).eval()
    sd = {k[2:]: torch.from_numpy(Z[k]) for k in Z.files if k.startswith("w.")}
    model.load_state_dict(sd, strict=True)
    mask = torch.from_numpy(Z["mask"])[None, None]
    with torch.no_grad():
        logits, _ = model(torch.from_numpy(Z["ids"])[None], torch.from_numpy(Z["pos"]), mask)
    assert torch.equal(logits[0], torch.from_numpy(Z["logits"]))


def test_prefix_cache_matches_full_forward():
    """Prefill + window over a cached prefix gives the full forward's window logits."""
    model = SDARVerifyModel(TINY).eval()
    model.load_state_dict({k[2:]: torch.from_numpy(Z[k]) for k in Z.files if k.startswith("w.")})
    mask = torch.from_numpy(Z["mask"])
    ids, pos = torch.from_numpy(Z["ids"])[None], torch.from_numpy(Z["pos"])
    P = 24                                     # prompt + accepted block
    with torch.no_grad():
        full, _ = model(ids, pos, mask[None, None])
        _, past = model(ids[:, :P], pos[:P], mask[:P, :P][None, None])
        win, _ = model(ids[:, P:], pos[P:], mask[P:, :][None, None], past)
    torch.testing.assert_close(win[0], full[0, P:], rtol=1e-5, atol=1e-6)


def test_greedy_match_matches_reference():
    for name in ("hit", "miss2"):
        draft = Z[f"greedy.{name}.draft"].tolist()
        logits = torch.from_numpy(Z["logits"])[-4:]
        acc, n, bonus = greedy_match_verify(draft, logits.argmax(-1).tolist())
        assert acc == Z[f"greedy.{name}.accepted"].tolist()
        assert n == int(Z[f"greedy.{name}.n"])
        assert (-1 if bonus is None else bonus) == int(Z[f"greedy.{name}.bonus"])
