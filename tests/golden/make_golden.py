#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the reference's own code.

Run in a container where the reference checkout exists (default
/root/reference, override with SIMSD_REFERENCE); the GPU box never runs this.

    python tests/golden/make_golden.py

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

REF = Path(os.environ.get("SIMSD_REFERENCE", "/root/reference"))
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

    (OUT / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    for p in sorted(OUT.glob("*.npz")):
        print(f"{p.name}: {p.stat().st_size / 1024:.0f} KiB")


if __name__ == "__main__":
    main()
