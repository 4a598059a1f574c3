"""Opt-in switch that routes a model's linears and MoE blocks through libsimsd_b200.

Same entry points and behaviour as the reference's kernels/fused_toggle.py:
  apply_to_model(model, enable=True, targets=DEFAULT_TARGETS, config=None) -> int   (:52-79)
  is_applied(model)                                                             (:82)
  fused_linear(model, enable=True, **kw)   context manager                     (:86-104)
  warmup(model, block_length=4, extra_M=())                                    (:107-133)
  apply_moe_to_model(model, enable=True) -> int                                (:151-198)
  is_moe_applied(model)                                                         (:201)

Leaf `nn.Linear`s whose name is in `targets` become `ThinLinear` modules that
alias the original parameters (no copy; `state_dict()` unchanged).  It is
idempotent, returns the number of modules swapped or restored, and must run
before CUDA-graph capture, which freezes whatever forward is installed.

Two additions:
* `apply_to_model(..., fuse_gate_up=True)` also patches SwiGLU MLP modules
  (attributes gate_proj / up_proj / down_proj and a SiLU `act_fn`, as `SDARMLP`
  in sdar/modeling_sdar.py:99-119) so gate and up run as one kernel reading both
  weights once, with the SiLU*mul applied before the single rounding;
* `apply_to_model(..., fuse_qkv=True)` makes the q_proj / k_proj / v_proj of
  each attention module (bias-free, as SDAR's, sdar/modeling_sdar.py:197-302)
  share one launch: the first of the three called on an input computes all
  three (`thin_linear_cat`, the weights are not copied) and the other two
  return their parts of that output when called on the same input tensor.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from ._lib import reset_workspace
from .thin_linear_fused import ThinLinear, should_fuse, thin_linear_cat, thin_linear_silu_mul

# Projection names swapped by default: every linear of an SDAR/LLaDA2 decoder
# layer.  The vocabulary projection is opt-in (ALL_TARGETS): with ~150 k output
# rows cuBLAS already fills the GPU there.
_LAYER_PROJECTIONS = ("q", "k", "v", "o", "gate", "up", "down")
DEFAULT_TARGETS = tuple(f"{p}_proj" for p in _LAYER_PROJECTIONS)
ALL_TARGETS = (*DEFAULT_TARGETS, "lm_head")

# id(model) -> {dotted path: (owning module, attribute, original nn.Linear)}
_ORIGINALS: dict[int, dict[str, tuple[nn.Module, str, nn.Linear]]] = {}
_MLP_PATCHED: dict[int, list[nn.Module]] = {}


def _linear_slots(root: nn.Module, wanted, prefix: str = ""):
    """Depth-first (path, owner, attribute, linear) for every nn.Linear child
    whose attribute name is in `wanted`; the swap replaces owner.attribute."""
    for attr, child in root.named_children():
        path = f"{prefix}.{attr}" if prefix else attr
        if isinstance(child, nn.Linear):
            if attr in wanted:
                yield path, root, attr, child
        else:
            yield from _linear_slots(child, wanted, path)


def _is_silu(act) -> bool:
    return isinstance(act, nn.SiLU) or getattr(act, "__name__", "") == "silu" or \
        act is torch.nn.functional.silu


def _gate_up_forward(self, x):
    gate, up = self.gate_proj, self.up_proj
    M = x.numel() // x.shape[-1] if x.shape[-1] else 0
    if (getattr(gate, "bias", None) is None and getattr(up, "bias", None) is None
            and should_fuse(M, gate.out_features, gate.in_features)
            and gate.weight.stride() == up.weight.stride()):
        return self.down_proj(thin_linear_silu_mul(x, gate.weight, up.weight))
    return self.down_proj(self.act_fn(gate(x)) * up(x))


def _patch_mlps(model: nn.Module) -> list[nn.Module]:
    patched = []
    for mod in model.modules():
        if all(hasattr(mod, a) for a in ("gate_proj", "up_proj", "down_proj", "act_fn")) \
                and _is_silu(mod.act_fn) and "forward" not in mod.__dict__:
            mod.forward = _gate_up_forward.__get__(mod)
            patched.append(mod)
    return patched


class _QKVShare:
    """The merged launch of one attention module's q/k/v: its input and outputs
    until each of the three projections has taken its part."""

    def __init__(self):
        self.parts: list["_QKVPart"] = []
        self.x = None
        self.out = None
        self.taken = [False, False, False]


class _QKVPart(ThinLinear):
    """q_proj, k_proj or v_proj (index i) of a merged q/k/v; aliases the
    original parameters like ThinLinear (same `state_dict()` keys and tensors)."""

    def __init__(self, linear: nn.Linear, share: _QKVShare, i: int, config=None):
        super().__init__(linear, config=config)
        self.__dict__["_share"] = share   # plain attribute: not a submodule, not in state_dict
        self.__dict__["_i"] = i

    def forward(self, x):
        sh, i = self._share, self._i
        if sh.x is x and sh.out is not None and not sh.taken[i]:
            sh.taken[i] = True
            out = sh.out[i]
            if all(sh.taken):
                sh.x = sh.out = None
            return out
        M = x.numel() // x.shape[-1] if x.shape[-1] else 0
        if self.config is None and should_fuse(M, self.out_features, self.in_features):
            sh.out = thin_linear_cat(x, [p.weight for p in sh.parts])
            sh.x = x
            sh.taken = [j == i for j in range(3)]
            return sh.out[i]
        return super().forward(x)


def _merge_qkv(model: nn.Module, saved: dict[str, nn.Module], config) -> None:
    for name, mod in model.named_modules():
        parts = [getattr(mod, a, None) for a in ("q_proj", "k_proj", "v_proj")]
        if not all(isinstance(p, ThinLinear) for p in parts):
            continue
        if any(p.bias is not None for p in parts) or len({p.in_features for p in parts}) != 1:
            continue
        paths = [f"{name}.{a}" if name else a for a in ("q_proj", "k_proj", "v_proj")]
        if not all(p in saved for p in paths):
            continue
        share = _QKVShare()
        for i, (attr, path) in enumerate(zip(("q_proj", "k_proj", "v_proj"), paths)):
            new = _QKVPart(saved[path][2], share, i, config=config)
            share.parts.append(new)
            setattr(mod, attr, new)


def apply_to_model(model: nn.Module, enable: bool = True,
                   targets=DEFAULT_TARGETS,
                   config: tuple[int, int, int, int] | None = None,
                   fuse_gate_up: bool = False, fuse_qkv: bool = False) -> int:
    """Swap the target `nn.Linear` modules for `ThinLinear` (or restore them).

    Idempotent in both directions.  Returns the number of modules swapped (or
    restored).  `ThinLinear` aliases the original parameters.
    """
    key = id(model)
    if not enable:
        saved = _ORIGINALS.pop(key, None)
        for mod in _MLP_PATCHED.pop(key, []):
            mod.__dict__.pop("forward", None)
        if not saved:
            return 0
        for owner, attr, orig in saved.values():
            setattr(owner, attr, orig)
        reset_workspace()
        return len(saved)

    if key in _ORIGINALS:
        return 0
    wanted = frozenset(targets)
    saved = {path: (owner, attr, lin) for path, owner, attr, lin in _linear_slots(model, wanted)}
    for owner, attr, lin in saved.values():
        setattr(owner, attr, ThinLinear(lin, config=config))
    if saved:
        _ORIGINALS[key] = saved
        if fuse_gate_up:
            _MLP_PATCHED[key] = _patch_mlps(model)
        if fuse_qkv:
            _merge_qkv(model, saved, config)
    return len(saved)


def is_applied(model: nn.Module) -> bool:
    return id(model) in _ORIGINALS


class fused_linear:
    """Context manager form, for tests:  with fused_toggle.fused_linear(model): ..."""

    def __init__(self, model: nn.Module, enable: bool = True, **kw):
        self.model, self.enable, self.kw = model, enable, kw
        self.n = 0

    def __enter__(self):
        self.n = apply_to_model(self.model, self.enable, **self.kw)
        return self

    def __exit__(self, *exc):
        if self.enable:
            apply_to_model(self.model, False)
        return False


def warmup(model: nn.Module, block_length: int = 4, extra_M=()) -> None:
    """Run every patched module once per M the pipeline uses, before graph capture.

    Nothing is JIT-compiled here (the kernels are built ahead of time), but the
    first call per device sizes the cached workspace, sets the kernels'
    shared-memory limits and resolves the driver's tensor-map entry point; doing
    that outside capture keeps the captured graph free of allocations.
    """
    Ms = {1, block_length, 2 * block_length, 96, 97, *extra_M}
    mods = [m for _, m in model.named_modules() if isinstance(m, ThinLinear)]
    devs = set()
    with torch.inference_mode():
        for mod in mods:
            devs.add(mod.weight.device)
            for M in sorted(Ms):
                mod(torch.zeros(M, mod.in_features, device=mod.weight.device, dtype=mod.weight.dtype))
        for mlp in _MLP_PATCHED.get(id(model), []):
            w = mlp.gate_proj.weight
            for M in sorted(Ms):
                mlp(torch.zeros(M, w.shape[1], device=w.device, dtype=w.dtype))
    for d in devs:
        torch.cuda.synchronize(d)


# ─────────────────────────────────────────────────────────────────────
# LLaDA2 MoE expert dispatch  (moe_dispatch_fused.py)
# ─────────────────────────────────────────────────────────────────────
_MOE_ATTR = "_simsd_fused_moe"


def _free_expert_weights(experts) -> None:
    for e in experts:
        for name in ("gate_proj", "up_proj", "down_proj"):
            lin = getattr(e, name)
            lin.weight.data = lin.weight.data.new_empty(0)


def apply_moe_to_model(model: nn.Module, enable: bool = True, pack_dir=None) -> int:
    """Switch LLaDA2 MoE blocks to the fused dispatch.  Idempotent.

    Stacks each block's expert weights (releasing the per-expert copies) and
    patches the block class's `moe_infer` once.  Disabling is not supported
    (the per-expert weights are gone): it raises NotImplementedError, as the
    reference does.  Must run before any CUDA-graph capture.

    `pack_dir` (a directory): each block's stacked weights are persisted there
    as `<module path>.simsd-experts` (kernels/expert_pack.py) the first time
    and read back from that file on later installs, on the device the block's
    experts live on.
    """
    from .moe_dispatch_fused import moe_dispatch, stack_expert_weights

    n = 0
    for name, mod in model.named_modules():
        if mod.__class__.__name__ != "LLaDA2MoeSparseMoeBlock":
            continue
        if enable:
            if getattr(mod, _MOE_ATTR, None) is not None:
                continue
            if pack_dir is not None:
                from pathlib import Path

                from .expert_pack import load_packed, pack_stacked
                path = Path(pack_dir) / f"{name or 'moe'}.simsd-experts"
                dev = mod.experts[0].gate_proj.weight.device
                if path.exists():
                    stacked = load_packed(path, dev)
                    _free_expert_weights(mod.experts)
                else:
                    stacked = stack_expert_weights(mod.experts)
                    pack_stacked(path, *stacked)
            else:
                stacked = stack_expert_weights(mod.experts)
            setattr(mod, _MOE_ATTR, stacked)
            n += 1
        elif getattr(mod, _MOE_ATTR, None) is not None:
            raise NotImplementedError(
                "apply_moe_to_model(enable=False) is not supported: stacking released "
                "the per-expert weights; reload the checkpoint to get the stock path back.")
    if n == 0:
        return 0

    cls = next(m.__class__ for m in model.modules()
               if m.__class__.__name__ == "LLaDA2MoeSparseMoeBlock")
    if not getattr(cls, "_simsd_moe_patched", False):
        stock = cls.moe_infer

        def moe_infer(self, x, topk_ids, topk_weight):
            packed = getattr(self, _MOE_ATTR, None)
            if packed is None:
                return stock(self, x, topk_ids, topk_weight)
            return moe_dispatch(x, topk_ids, topk_weight, *packed)

        cls.moe_infer = moe_infer
        cls._simsd_moe_stock = stock
        cls._simsd_moe_patched = True
    return n


def is_moe_applied(model: nn.Module) -> bool:
    return any(getattr(m, _MOE_ATTR, None) is not None for m in model.modules())
