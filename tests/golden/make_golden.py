#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run where a checkout of the reference exists, naming it with the required
SIMSD_REFERENCE environment variable; the GPU box never runs this.

    SIMSD_REFERENCE=<path to the SimSD-release checkout> python tests/golden/make_golden.py

Writes (inputs and the reference's outputs, bf16 as uint16 bit patterns):
  align.npz          kernels/moe_dispatch_fused.py:93-132 `_align` (and :135 `_num_tiles`)
                     on ids from kernels/workspace/moe_dispatch/build_oracle.py:71-90 `_routing`
  moe_dispatch.npz   build_oracle.py:34-67 `reference_moe_dispatch` (the stock moe_infer
                     transcription) on inputs made by build_oracle.py:93-112 `_case`
  thin_linear.npz    torch.nn.functional.linear, the reference's ground truth for
                     kernels/thin_linear_fused.py (CONTRACT: "reference = F.linear"),
                     on the odd/degenerate shapes of thin_linear_fused_test.py:57-62
                     (scaled down) and the magnitude / zero / bias cases of :74-109
  router.npz         the router restatement sigmoid(x.float() @ Wr.float().T), top-k of
                     score + bias, gathered scores renormalised (+1e-20) x scale, in torch
  sdar_verify.npz    a tiny fp32 SDARForCausalLM (sdar/modeling_sdar.py, imported with the
                     shims transformers 5.x needs) with patch_stock_rms_norm, its logits on a
                     K=2 verify sequence from speculative_decoding/verify.py:350-418
                     build_verify_sequence_multi, the mask of
                     sdar/new_attn_multi_block.py:22-186, and mrs.py:111-145
                     greedy_match_verify results
  manifest.json      provenance of every case
"""
from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

if not os.environ.get("SIMSD_REFERENCE"):
    sys.exit("make_golden.py: set SIMSD_REFERENCE to the reference checkout (SimSD-release)")
REF = Path(os.environ["SIMSD_REFERENCE"]).resolve()
OUT = Path(__file__).resolve().parent
sys.path.insert(0, str(REF))

from kernels.moe_dispatch_fused import _align, _num_tiles  # noqa: E402  (the reference's)
from kernels.workspace.moe_dispatch.build_oracle import (  # noqa: E402
    _case, _routing, reference_moe_dispatch)


def bits(t: torch.Tensor) -> np.ndarray:
    """bf16 -> uint16 bit patterns; other dtypes -> numpy as is."""
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def load_reference_sdar():
    """Import the reference's sdar/modeling_sdar.py under transformers 5.x.

    The file targets transformers 4.52 and a configuration module that is not in
    the checkout, so five names are supplied before it is executed: a
    SDARConfig (Qwen3Config subclass), SlidingWindowCache, LossKwargs, the
    'default' RoPE init and a stand-in for flash-attn's Triton RMSNorm (the
    runners replace RMSNorm.forward with patch_stock_rms_norm anyway).
    """
    import importlib.util
    import types
    from typing import TypedDict

    import transformers.cache_utils as cu
    import transformers.utils as tu
    from transformers import Qwen3Config
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    if not hasattr(cu, "SlidingWindowCache"):
        cu.SlidingWindowCache = type("SlidingWindowCache", (), {})
    if not hasattr(tu, "LossKwargs"):
        tu.LossKwargs = TypedDict("LossKwargs", {}, total=False)
    if "default" not in ROPE_INIT_FUNCTIONS:
        def _default(config, device=None, **kw):
            rp = getattr(config, "rope_parameters", None) or {}
            base = rp.get("rope_theta", getattr(config, "rope_theta", 10000.0))
            dim = getattr(config, "head_dim", config.hidden_size // config.num_attention_heads)
            inv = 1.0 / (base ** (torch.arange(0, dim, 2, dtype=torch.int64).to(device=device, dtype=torch.float) / dim))
            return inv, 1.0
        ROPE_INIT_FUNCTIONS["default"] = _default
    ln = types.ModuleType("flash_attn.ops.triton.layer_norm")
    ln.rms_norm_fn = lambda *a, **k: None
    for name in ("flash_attn.ops", "flash_attn.ops.triton"):
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["flash_attn.ops.triton.layer_norm"] = ln
    pkg = types.ModuleType("sdar_ref")
    pkg.__path__ = [str(REF / "sdar")]
    sys.modules["sdar_ref"] = pkg
    cfgmod = types.ModuleType("sdar_ref.configuration_sdar")
    SDARConfig = type("SDARConfig", (Qwen3Config,), {"model_type": "sdar"})
    cfgmod.SDARConfig = SDARConfig
    sys.modules["sdar_ref.configuration_sdar"] = cfgmod
    spec = importlib.util.spec_from_file_location("sdar_ref.modeling_sdar", REF / "sdar" / "modeling_sdar.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["sdar_ref.modeling_sdar"] = mod
    spec.loader.exec_module(mod)
    mod.liger_kernel_is_available = False
    return mod, SDARConfig


def main():
    manifest = {"reference": str(REF), "torch": torch.__version__, "cases": {}}

    # ---------------------------------------------------------------- align
    arrs = {}
    cases = [("uniform_T32_E256_k8", 32, 8, 256, None, 4), ("skew_T64_E256_k8", 64, 8, 256, 0.2, 2),
             ("tiny_T4_E8_k2", 4, 2, 8, None, 6), ("odd_T7_E13_k3", 7, 3, 13, None, 7),
             ("single_T1_E256_k8", 1, 8, 256, 0.05, 5), ("k1_T16_E32", 16, 1, 32, None, 8),
             ("big_T1024_E256_k8", 1024, 8, 256, 0.5, 21), ("skew_T256_E256_k8", 256, 8, 256, 0.05, 22)]
    for name, T, k, E, conc, seed in cases:
        g = torch.Generator().manual_seed(seed)
        ids, _ = _routing(T, k, E, "cpu", concentration=conc, generator=g)
        M = T * k
        nt = _num_tiles(M, E)
        slots, tile_expert = _align(ids, E, nt)
        arrs[f"{name}.ids"] = ids.numpy()
        arrs[f"{name}.E"] = np.array(E)
        arrs[f"{name}.num_tiles"] = np.array(nt)
        arrs[f"{name}.slots"] = slots.numpy()
        arrs[f"{name}.tile_expert"] = tile_expert.numpy()
        manifest["cases"][f"align/{name}"] = {"T": T, "k": k, "E": E, "concentration": conc, "seed": seed,
                                              "src": "kernels/moe_dispatch_fused.py:93-132 _align"}
    # all tokens to one expert (k = 1), as build_oracle.py:143-155 constructs it
    ids = torch.zeros(32, 1, dtype=torch.long)
    nt = _num_tiles(32, 256)
    slots, tile_expert = _align(ids, 256, nt)
    arrs.update({"all_one_expert.ids": ids.numpy(), "all_one_expert.E": np.array(256),
                 "all_one_expert.num_tiles": np.array(nt), "all_one_expert.slots": slots.numpy(),
                 "all_one_expert.tile_expert": tile_expert.numpy()})
    manifest["cases"]["align/all_one_expert"] = {"T": 32, "k": 1, "E": 256, "src": "_align"}
    np.savez_compressed(OUT / "align.npz", **arrs)

    # ---------------------------------------------------------------- moe_dispatch
    arrs = {}
    moe_cases = [
        # name, T, k, E, H, I, dtype, scale, concentration, seed
        ("tiny_bf16", 4, 2, 8, 64, 32, torch.bfloat16, 1.0, None, 6),
        ("tiny_fp32", 4, 2, 8, 64, 32, torch.float32, 1.0, None, 6),
        ("odd_dims_bf16", 7, 3, 13, 130, 70, torch.bfloat16, 1.0, None, 7),
        ("k1_bf16", 16, 1, 16, 128, 64, torch.bfloat16, 1.0, None, 8),
        ("large_mag_bf16", 16, 4, 16, 128, 64, torch.bfloat16, 100.0, None, 9),
        ("tiny_mag_fp32", 16, 4, 16, 128, 64, torch.float32, 1e-3, None, 10),
        ("tc_shape_bf16", 32, 4, 8, 256, 128, torch.bfloat16, 1.0, 0.5, 12),
        ("tc_shape_fp16", 16, 2, 8, 192, 64, torch.float16, 1.0, None, 13),
    ]
    for name, T, k, E, H, I, dt, scale, conc, seed in moe_cases:
        c = _case(name, "fake", T, k, E, H, I, dt, "cpu", scale=scale, concentration=conc, seed=seed)
        x, ids, w, wg, wu, wd = c["args"]
        for key, t in (("x", x), ("ids", ids), ("w", w), ("wg", wg), ("wu", wu), ("wd", wd),
                       ("ref", c["ref_out"])):
            arrs[f"{name}.{key}"] = bits(t)
        arrs[f"{name}.dtype"] = np.array(str(dt))
        manifest["cases"][f"moe/{name}"] = {**c["meta"], "src": "build_oracle.py:34-67 reference_moe_dispatch"}
    # all tokens on one expert, k = 1
    c = _case("all_one_expert_bf16", "extreme", 32, 1, 16, 128, 64, torch.bfloat16, "cpu", seed=11)
    c["args"][1] = torch.zeros_like(c["args"][1])
    with torch.inference_mode():
        ref = reference_moe_dispatch(*c["args"])
    for key, t in zip(("x", "ids", "w", "wg", "wu", "wd"), c["args"]):
        arrs[f"all_one_expert_bf16.{key}"] = bits(t)
    arrs["all_one_expert_bf16.ref"] = bits(ref)
    arrs["all_one_expert_bf16.dtype"] = np.array("torch.bfloat16")
    manifest["cases"]["moe/all_one_expert_bf16"] = {"T": 32, "k": 1, "E": 16, "H": 128, "I": 64,
                                                   "src": "reference_moe_dispatch"}
    np.savez_compressed(OUT / "moe_dispatch.npz", **arrs)

    # ---------------------------------------------------------------- thin linear
    arrs = {}
    g = torch.Generator().manual_seed(1234)

    def rnd(*shape, dtype=torch.bfloat16, scale=1.0):
        return (torch.randn(*shape, generator=g, dtype=torch.float32) * scale).to(dtype)

    lin = [("odd_127x65", 4, 127, 65, torch.bfloat16, 1.0, False),
           ("odd_1x1", 4, 1, 1, torch.bfloat16, 1.0, False),
           ("odd_2048x1", 4, 2048, 1, torch.bfloat16, 1.0, False),
           ("odd_3x257", 4, 3, 257, torch.bfloat16, 1.0, False),
           ("odd_1021x77", 4, 1021, 77, torch.bfloat16, 1.0, False),
           ("tc_M1_512x384", 1, 512, 384, torch.bfloat16, 1.0, False),
           ("tc_M4_1024x256", 4, 1024, 256, torch.bfloat16, 1.0, False),
           ("tc_M16_2048x256", 16, 2048, 256, torch.bfloat16, 1.0, False),
           ("tc_M64_512x512", 64, 512, 512, torch.bfloat16, 1.0, False),
           ("tc_M33_640x130", 33, 640, 130, torch.bfloat16, 1.0, False),
           ("fp16_M8_512x256", 8, 512, 256, torch.float16, 1.0, False),
           ("fp32_M4_512x256", 4, 512, 256, torch.float32, 1.0, False),
           ("mag1e-3_M4_512x256", 4, 512, 256, torch.bfloat16, 1e-3, False),
           ("mag1e4_M4_512x256", 4, 512, 256, torch.bfloat16, 1e4, False),
           ("bias_M4_512x256", 4, 512, 256, torch.bfloat16, 1.0, True)]
    for name, M, K, N, dt, scale, has_bias in lin:
        x = rnd(M, K, dtype=dt, scale=scale)
        w = rnd(N, K, dtype=dt, scale=0.02)
        b = rnd(N, dtype=dt, scale=0.5) if has_bias else None
        with torch.inference_mode():
            y = F.linear(x, w, b)
        arrs[f"{name}.x"], arrs[f"{name}.w"], arrs[f"{name}.y"] = bits(x), bits(w), bits(y)
        if b is not None:
            arrs[f"{name}.b"] = bits(b)
        arrs[f"{name}.dtype"] = np.array(str(dt))
        manifest["cases"][f"thin_linear/{name}"] = {"M": M, "K": K, "N": N, "dtype": str(dt), "scale": scale,
                                                    "bias": has_bias, "src": "torch.nn.functional.linear"}
    np.savez_compressed(OUT / "thin_linear.npz", **arrs)

    # ---------------------------------------------------------------- router (torch restatement)
    arrs = {}
    for name, T, H, E, k, bias_std, seed in [("cfg3_T64", 64, 2048, 256, 8, 0.1, 3),
                                             ("skew_T32", 32, 1024, 128, 8, 0.5, 5),
                                             ("small_T16", 16, 256, 32, 4, 0.1, 1)]:
        gg = torch.Generator().manual_seed(seed)
        x = torch.randn(T, H, generator=gg).to(torch.bfloat16)
        wr = (torch.randn(E, H, generator=gg) * 0.02).to(torch.bfloat16)
        b = torch.randn(E, generator=gg) * bias_std
        s = torch.sigmoid(x.float() @ wr.float().T)
        ids = (s + b).topk(k, dim=-1).indices
        wts = s.gather(1, ids)
        wts = wts / (wts.sum(-1, keepdim=True) + 1e-20)
        for key, t in (("x", x), ("wr", wr), ("bias", b), ("ids", ids), ("w", wts)):
            arrs[f"{name}.{key}"] = bits(t)
        manifest["cases"][f"router/{name}"] = {"T": T, "H": H, "E": E, "k": k, "bias_std": bias_std,
                                               "src": "torch restatement of the sigmoid+bias top-k router"}
    np.savez_compressed(OUT / "router.npz", **arrs)

    # ---------------------------------------------------------------- SDAR verify (tiny)
    arrs = {}
    mod, SDARConfig = load_reference_sdar()
    from sdar.run_native_tp2 import patch_stock_rms_norm
    from sdar.new_attn_multi_block import create_multi_block_causal_mask
    from speculative_decoding.mrs import greedy_match_verify
    from speculative_decoding.verify import build_verify_sequence_multi
    cfg = SDARConfig(vocab_size=256, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                     num_attention_heads=4, num_key_value_heads=2, head_dim=16, rope_theta=1e6,
                     rms_norm_eps=1e-6, max_position_embeddings=512, attention_bias=False,
                     tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    cfg.fuse_cross_entropy = False
    m = mod.SDARForCausalLM(cfg).eval()
    patch_stock_rms_norm(m)
    torch.manual_seed(0)
    with torch.no_grad():
        for n, p in m.named_parameters():
            if "norm" in n:
                p.fill_(1.0)
            else:
                p.normal_(0, 0.02)
    prompt = list(range(10, 30))
    accepted = [[40, 41, 42, 43]]
    drafts = [[5, 6, 7, 8], [9, 10, 11, 12]]
    smaps = [[0, 2, 1, 3], [3, 1, 0, 2]]
    ids, labels, blocks, _, pos = build_verify_sequence_multi(prompt, accepted, drafts, smaps, 4, 4,
                                                             mask_token_id=255)
    mask = create_multi_block_causal_mask(torch.tensor([labels]), torch.tensor([blocks]), 4,
                                          block_causal_prompt=True)
    with torch.no_grad():
        logits = m(input_ids=torch.tensor([ids]), attention_mask=mask, position_ids=torch.tensor([pos]),
                   use_cache=False).logits[0]
    for k, v in m.state_dict().items():
        arrs[f"w.{k.replace('model.', '', 1)}"] = v.numpy()
    arrs.update({"ids": np.array(ids), "labels": np.array(labels), "blocks": np.array(blocks),
                 "pos": np.array(pos), "mask": mask[0, 0].numpy(), "logits": logits.numpy()})
    probs = torch.softmax(logits[-4:], -1)            # the last draft block's mask window
    for name, d in (("hit", probs.argmax(-1).tolist()), ("miss2", probs.argmax(-1).tolist()[:2] + [0, 0])):
        acc, n, bonus = greedy_match_verify(d, probs, probs, [0, 1, 2, 3])
        arrs[f"greedy.{name}.draft"] = np.array(d)
        arrs[f"greedy.{name}.accepted"] = np.array(acc)
        arrs[f"greedy.{name}.n"] = np.array(n)
        arrs[f"greedy.{name}.bonus"] = np.array(-1 if bonus is None else bonus)
    np.savez_compressed(OUT / "sdar_verify.npz", **arrs)
    manifest["cases"]["sdar_verify/tiny"] = {"layers": 2, "hidden": 64, "heads": "4/2", "head_dim": 16,
                                             "src": "sdar/modeling_sdar.py SDARForCausalLM + patch_stock_rms_norm"}

    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    for p in sorted(OUT.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
