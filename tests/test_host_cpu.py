"""Host-side behaviour of the drop-in `kernels` package that needs no GPU:
error conventions (kernels/thin_linear_fused.py:280-295), no CPU fallback,
the dispatch guard and the toggle (kernels/thin_linear_fused_test.py:253-298)."""
from __future__ import annotations

import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from kernels import fused_toggle
from kernels.moe_dispatch_fused import moe_dispatch, moe_route, stack_expert_weights
from kernels.thin_linear_fused import (FUSE_MAX_M, ThinLinear, _tuned_for, pick_config, should_fuse,
                                       thin_linear)


def test_forward_only_error():
    x = torch.randn(4, 64, dtype=torch.bfloat16, requires_grad=True)
    w = torch.randn(32, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="forward-only"):
        thin_linear(x, w)


def test_dtype_and_shape_errors():
    with pytest.raises(TypeError):
        thin_linear(torch.randn(4, 64, dtype=torch.bfloat16), torch.randn(32, 64))
    with pytest.raises(ValueError):
        thin_linear(torch.randn(4, 64), torch.randn(32, 64, 1))
    with pytest.raises(ValueError):
        thin_linear(torch.randn(4, 64), torch.randn(32, 63))
    with pytest.raises(TypeError):
        thin_linear(torch.randn(4, 64), torch.randn(32, 64).double())


def test_no_cpu_fallback():
    with torch.inference_mode(), pytest.raises(RuntimeError, match="CUDA tensors only"):
        thin_linear(torch.randn(4, 64), torch.randn(32, 64))
    x = torch.randn(4, 64)
    with torch.inference_mode(), pytest.raises(RuntimeError, match="CUDA tensors only"):
        moe_dispatch(x, torch.zeros(4, 2, dtype=torch.long), torch.ones(4, 2), torch.randn(4, 16, 64),
                     torch.randn(4, 16, 64), torch.randn(4, 64, 16))
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        moe_route(x, torch.randn(8, 64), None, k=2)


def test_moe_argument_errors():
    x = torch.randn(4, 64)
    with pytest.raises(TypeError):
        moe_dispatch(x, torch.zeros(4, 2, dtype=torch.int32), torch.ones(4, 2), torch.randn(4, 16, 64),
                     torch.randn(4, 16, 64), torch.randn(4, 64, 16))
    with pytest.raises(ValueError):
        moe_dispatch(x, torch.zeros(4, 2, dtype=torch.long), torch.ones(4, 2), torch.randn(4, 16, 64),
                     torch.randn(4, 16, 64), torch.randn(4, 16, 64))
    with pytest.raises(ValueError):
        moe_route(x, torch.randn(8, 64), None, k=9)


def test_dispatch_guard_and_config():
    assert should_fuse(1, 4096, 4096) and should_fuse(FUSE_MAX_M, 4096, 4096)
    assert not should_fuse(FUSE_MAX_M + 1, 4096, 4096) and not should_fuse(96, 2048, 2048)
    assert pick_config(4, 2048, 2048) == (16, 128, 64, 0)
    assert pick_config(64, 2048, 2048)[0] == 64
    assert _tuned_for(4, 2048, 2048) is None


def test_thin_linear_module_falls_back_above_guard_on_cpu():
    lin = nn.Linear(64, 32, bias=True).to(torch.bfloat16)
    mod = ThinLinear(lin)
    x = torch.randn(2, FUSE_MAX_M, 64, dtype=torch.bfloat16)     # M = 128 > guard -> F.linear
    with torch.inference_mode():
        assert torch.equal(mod(x), F.linear(x, lin.weight, lin.bias))


class _Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.q_proj = nn.Linear(512, 512, bias=False)
        self.gate_proj = nn.Linear(512, 1024, bias=False)
        self.other = nn.Linear(512, 8, bias=False)


def test_toggle_swaps_restores_and_is_idempotent():
    m = _Tiny()
    assert fused_toggle.apply_to_model(m, True) == 2
    assert isinstance(m.q_proj, ThinLinear) and isinstance(m.other, nn.Linear)
    assert fused_toggle.apply_to_model(m, True) == 0
    assert fused_toggle.is_applied(m)
    assert fused_toggle.apply_to_model(m, False) == 2
    assert isinstance(m.q_proj, nn.Linear) and not fused_toggle.is_applied(m)
    assert fused_toggle.apply_to_model(m, False) == 0


def test_toggle_aliases_parameters_and_keeps_state_dict():
    m = _Tiny()
    before = {k: v.clone() for k, v in m.state_dict().items()}
    ptr = m.q_proj.weight.data_ptr()
    with fused_toggle.fused_linear(m) as ctx:
        assert ctx.n == 2
        after = m.state_dict()
        assert set(after) == set(before)
        for k in before:
            assert torch.equal(after[k], before[k])
        assert m.q_proj.weight.data_ptr() == ptr
    assert isinstance(m.q_proj, nn.Linear)


class _MLP(nn.Module):
    def __init__(self):
        super().__init__()
        self.gate_proj = nn.Linear(64, 128, bias=False)
        self.up_proj = nn.Linear(64, 128, bias=False)
        self.down_proj = nn.Linear(128, 64, bias=False)
        self.act_fn = nn.SiLU()

    def forward(self, x):
        return self.down_proj(self.act_fn(self.gate_proj(x)) * self.up_proj(x))


def test_gate_up_patch_installs_and_removes():
    m = nn.Sequential(_MLP())
    assert fused_toggle.apply_to_model(m, True, fuse_gate_up=True) == 3
    assert "forward" in m[0].__dict__
    x = torch.randn(FUSE_MAX_M + 1, 64)                 # above the guard: stock math on CPU
    with torch.inference_mode():
        y = m(x)
    fused_toggle.apply_to_model(m, False)
    assert "forward" not in m[0].__dict__
    with torch.inference_mode():
        assert torch.allclose(y, m(x))


class _Attn(nn.Module):
    def __init__(self, bias=False):
        super().__init__()
        self.q_proj = nn.Linear(64, 128, bias=bias)
        self.k_proj = nn.Linear(64, 32, bias=bias)
        self.v_proj = nn.Linear(64, 32, bias=bias)
        self.o_proj = nn.Linear(128, 64, bias=False)

    def forward(self, x):
        return self.q_proj(x), self.k_proj(x), self.v_proj(x)


def test_qkv_merge_installs_aliases_and_restores():
    m = nn.Sequential(_Attn(), _Attn(bias=True))
    before = {k: v for k, v in m.state_dict(keep_vars=True).items()}
    assert fused_toggle.apply_to_model(m, True, fuse_qkv=True) == 8
    merged = [type(getattr(m[0], a)).__name__ for a in ("q_proj", "k_proj", "v_proj")]
    assert merged == ["_QKVPart"] * 3                  # bias-free attention: merged
    assert type(m[1].q_proj).__name__ == "ThinLinear"  # with biases: plain swap
    after = m.state_dict(keep_vars=True)
    assert set(after) == set(before) and all(after[k] is before[k] for k in before)
    x = torch.randn(FUSE_MAX_M + 1, 64)                 # above the guard: stock math on CPU
    with torch.inference_mode():
        q, k, v = m[0](x)
    assert torch.allclose(q, torch.nn.functional.linear(x, m[0].q_proj.weight))
    assert fused_toggle.apply_to_model(m, False) == 8
    assert isinstance(m[0].q_proj, nn.Linear) and not isinstance(m[0].q_proj, fused_toggle.ThinLinear)


class LLaDA2MoeSparseMoeBlock(nn.Module):     # same class name the toggle looks for
    def __init__(self, E=4, H=32, I=16):
        super().__init__()
        self.experts = nn.ModuleList(_Expert(H, I) for _ in range(E))

    def moe_infer(self, x, topk_ids, topk_weight):
        return "stock"


class _Expert(nn.Module):
    def __init__(self, H, I):
        super().__init__()
        self.gate_proj = nn.Linear(H, I, bias=False)
        self.up_proj = nn.Linear(H, I, bias=False)
        self.down_proj = nn.Linear(I, H, bias=False)


def test_moe_toggle_stacks_and_patches_once():
    m = nn.Sequential(LLaDA2MoeSparseMoeBlock(), LLaDA2MoeSparseMoeBlock())
    g0 = torch.stack([e.gate_proj.weight.detach().clone() for e in m[0].experts])
    assert fused_toggle.apply_moe_to_model(m) == 2
    assert fused_toggle.is_moe_applied(m)
    wg, wu, wd = getattr(m[0], "_simsd_fused_moe")
    assert wg.shape == (4, 16, 32) and wd.shape == (4, 32, 16)
    assert torch.equal(wg, g0)
    assert m[0].experts[0].gate_proj.weight.numel() == 0          # originals released
    assert fused_toggle.apply_moe_to_model(m) == 0                # idempotent
    with pytest.raises(NotImplementedError):
        fused_toggle.apply_moe_to_model(m, False)


def test_stack_expert_weights_keeps_originals_on_request():
    blk = LLaDA2MoeSparseMoeBlock(E=3, H=8, I=4)
    wg, wu, wd = stack_expert_weights(blk.experts, free_originals=False)
    assert wg.is_contiguous() and wg.shape == (3, 4, 8) and wd.shape == (3, 8, 4)
    assert blk.experts[2].up_proj.weight.numel() == 32
    assert torch.equal(wu[2], blk.experts[2].up_proj.weight)


# ------------------------------------------------------------------ packed experts on disk
def test_expert_pack_round_trip_and_checks(tmp_path):
    from kernels.expert_pack import load_packed, pack_experts, read_header
    for dtype in (torch.bfloat16, torch.float16, torch.float32):
        blk = LLaDA2MoeSparseMoeBlock(E=5, H=24, I=12).to(dtype)
        ref = stack_expert_weights(blk.experts, free_originals=False)
        path = pack_experts(tmp_path / f"l0_{dtype}.simsd-experts", blk.experts)
        hdr = read_header(path)
        assert (hdr["E"], hdr["I"], hdr["H"]) == (5, 12, 24)
        assert all(a["offset"] % 4096 == 0 for a in hdr["arrays"])
        got = load_packed(path, "cpu")
        for a, b in zip(got, ref):
            assert a.dtype == dtype and torch.equal(a, b)
    # a flipped byte in the data fails the checksum; a wrong magic fails the header
    raw = bytearray(path.read_bytes())
    raw[hdr["arrays"][1]["offset"] + 3] ^= 0x40
    bad = tmp_path / "bad.simsd-experts"
    bad.write_bytes(bytes(raw))
    with pytest.raises(ValueError, match="checksum"):
        load_packed(bad, "cpu")
    bad.write_bytes(b"NOTAPACK" + bytes(raw[8:]))
    with pytest.raises(ValueError, match="not a simsd expert pack"):
        load_packed(bad, "cpu")


def test_moe_toggle_writes_then_reads_packs(tmp_path):
    torch.manual_seed(0)
    m1 = nn.Sequential(LLaDA2MoeSparseMoeBlock(), LLaDA2MoeSparseMoeBlock())
    m2 = nn.Sequential(LLaDA2MoeSparseMoeBlock(), LLaDA2MoeSparseMoeBlock())
    m2.load_state_dict(m1.state_dict())
    assert fused_toggle.apply_moe_to_model(m1, pack_dir=tmp_path) == 2          # stacks and writes
    assert sorted(p.name for p in tmp_path.iterdir()) == ["0.simsd-experts", "1.simsd-experts"]
    assert fused_toggle.apply_moe_to_model(m2, pack_dir=tmp_path) == 2          # reads back
    for b1, b2 in zip(m1, m2):
        for a, b in zip(getattr(b1, "_simsd_fused_moe"), getattr(b2, "_simsd_fused_moe")):
            assert torch.equal(a, b)
    assert m2[1].experts[0].down_proj.weight.numel() == 0                      # originals released
