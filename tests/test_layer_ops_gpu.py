"""GPU parity of the verify forward's layer ops (kernels/layer_ops.py) against
the torch expressions they replace (the harness's fp32 RMSNorm and rotary
embedding, kernels/sdar_verify.py): elementwise steps are bit-exact; the
RMSNorm mean square is an fp32 sum in the kernel's own order, so an output may
differ from torch's by one rounding step of the output type."""
from __future__ import annotations

import pytest
import torch

from kernels.layer_ops import qk_norm_rope, rmsnorm, verify_attention
from kernels.sdar_verify import RMSNorm, _rotate_half, rope_cos_sin

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _ulp_close(a: torch.Tensor, b: torch.Tensor, frac_max: float = 0.01, inner: torch.Tensor | None = None):
    """Equal, or one bf16/fp16 step apart at a small fraction of the elements.
    `inner`: for y = w * round(h * inv), |w * round(h * inv)| - a one-step change
    of the inner rounding (a mean square summed in another order) moves y by up
    to one step of that product before y's own rounding."""
    a, b = a.float(), b.float()
    diff = (a - b).abs()
    step = torch.maximum(a.abs(), b.abs()) * 2 ** -7 + 1e-30   # one bf16 step (fp16: finer)
    if inner is not None:
        step = step + inner.float().abs() * 2 ** -7
    assert bool((diff <= step).all()), float((diff / step).max())
    assert float((diff > 0).float().mean()) <= frac_max


# n a multiple of 8 takes the 16-byte-vector kernel (1..8 vectors a thread),
# other n the scalar one
@pytest.mark.parametrize("rows,n,dtype", [(32, 4096, torch.bfloat16), (1, 4096, torch.bfloat16),
                                          (7, 1000, torch.float16), (64, 2048, torch.bfloat16),
                                          (3, 16384, torch.bfloat16), (4, 1024, torch.bfloat16),
                                          (5, 1001, torch.bfloat16), (2, 6, torch.float16)])
def test_rmsnorm_matches_torch(rows, n, dtype):
    g = torch.Generator(device=DEV).manual_seed(rows + n)
    x = (torch.randn(rows, n, generator=g, device=DEV) * 3).to(dtype)
    r = torch.randn(rows, n, generator=g, device=DEV).to(dtype)
    norm = RMSNorm(n, 1e-6).to(DEV, dtype)
    with torch.no_grad():
        norm.weight.copy_((torch.randn(n, generator=g, device=DEV) * 0.5 + 1).to(dtype))
    with torch.inference_mode():
        y = rmsnorm(x, norm.weight, 1e-6)
        h, y2 = rmsnorm(x, norm.weight, 1e-6, residual=r)
        ref = norm(x)
        href = r + x
        ref2 = norm(href)
    torch.cuda.synchronize()

    def inner(v):   # |w| * |round(h * inv)| of the reference's expression
        v32 = v.float()
        nv = (v32 * torch.rsqrt(v32.pow(2).mean(-1, keepdim=True) + 1e-6)).to(dtype)
        return norm.weight.float().abs() * nv.float().abs()

    _ulp_close(y, ref, inner=inner(x))
    assert torch.equal(h, href)
    _ulp_close(y2, ref2, inner=inner(href))


def test_qk_norm_rope_matches_torch():
    L, Hq, Hk, D, P = 32, 32, 8, 128, 100
    g = torch.Generator(device=DEV).manual_seed(5)
    bf = torch.bfloat16
    qkv = torch.randn(L, (Hq + 2 * Hk) * D, generator=g, device=DEV).to(bf)
    qn, kn = RMSNorm(D, 1e-6).to(DEV, bf), RMSNorm(D, 1e-6).to(DEV, bf)
    with torch.no_grad():
        qn.weight.copy_((torch.randn(D, generator=g, device=DEV) * 0.3 + 1).to(bf))
        kn.weight.copy_((torch.randn(D, generator=g, device=DEV) * 0.3 + 1).to(bf))
    pos = torch.arange(P, P + L, device=DEV)
    cos, sin = rope_cos_sin(pos, D, 1e6, bf)
    kc = torch.zeros(Hk, P + L, D, dtype=bf, device=DEV)
    vc = torch.zeros_like(kc)
    with torch.inference_mode():
        q = qk_norm_rope(qkv, Hq, Hk, qn.weight, kn.weight, cos, sin, 1e-6, kc, vc, P)
        x = qkv.view(1, L, Hq + 2 * Hk, D)
        qr = qn(x[:, :, :Hq]).transpose(1, 2)
        kr = kn(x[:, :, Hq:Hq + Hk]).transpose(1, 2)
        vr = x[:, :, Hq + Hk:].transpose(1, 2)
        c, s = cos[None, None], sin[None, None]
        qr = qr * c + _rotate_half(qr) * s
        kr = kr * c + _rotate_half(kr) * s
    torch.cuda.synchronize()

    def close_rows(a, b):
        # the rotary sum can cancel, so its rounding step is measured on the
        # head row's scale: within one bf16 step of the row's largest value
        a, b = a.float(), b.float()
        scale = b.abs().amax(-1, keepdim=True) * 2 ** -7 + 1e-30
        assert bool(((a - b).abs() <= scale).all())
        assert float(((a - b) != 0).float().mean()) <= 0.05

    close_rows(q, qr[0])
    close_rows(kc[:, P:], kr[0])
    assert torch.equal(vc[:, P:], vr[0])
    assert bool((kc[:, :P] == 0).all()) and bool((vc[:, :P] == 0).all())   # other rows untouched


# Lk up to 24 x 128 keys runs the tcgen05 cluster kernel (1-3 key tiles per
# CTA, clusters of 2..8), longer contexts the mma.sync split kernel + combine;
# mask rows of a 16-byte multiple take the vector mask loads
@pytest.mark.parametrize("Hq,Hk,L,Lk,cap,pmask,mpad", [(32, 8, 32, 2080, 2080, 0.0, 5), (32, 8, 32, 2080, 2100, 0.3, 5),
                                                       (16, 8, 8, 300, 320, 0.5, 5), (32, 8, 4, 129, 129, 0.0, 5),
                                                       (8, 8, 16, 1000, 1000, 0.9, 5), (32, 8, 32, 2080, 2112, 0.2, 0),
                                                       (32, 8, 32, 3072, 3072, 0.1, 0), (8, 8, 16, 4000, 4000, 0.2, 0),
                                                       (32, 8, 32, 100, 100, 0.0, 12)])
def test_verify_attention_matches_fp32_reference(Hq, Hk, L, Lk, cap, pmask, mpad):
    g = torch.Generator(device=DEV).manual_seed(Lk + L)
    bf = torch.bfloat16
    q = torch.randn(Hq, L, 128, generator=g, device=DEV).to(bf)
    kc = torch.randn(Hk, cap, 128, generator=g, device=DEV).to(bf)
    vc = torch.randn(Hk, cap, 128, generator=g, device=DEV).to(bf)
    if cap > Lk:
        vc[:, Lk:] = float("nan")                       # rows past Lk never reach the output
    mask = torch.rand(L, Lk + mpad, generator=g, device=DEV) >= pmask
    mask[:, 0] = True                                   # every row sees a key
    mask[0, 1:] = False                                 # row 0: one key only
    scale = 128 ** -0.5
    with torch.inference_mode():
        o = verify_attention(q, kc, vc, Lk, mask, scale).view(L, Hq, 128)
    G = Hq // Hk
    kf = kc[:, :Lk].float().repeat_interleave(G, 0)
    vf = vc[:, :Lk].float().repeat_interleave(G, 0)
    s = (q.float() @ kf.transpose(1, 2)) * scale
    s = s.masked_fill(~mask[None, :, :Lk], float("-inf"))
    pr = torch.softmax(s, -1)
    ref = (pr @ vf).transpose(0, 1)                     # [L, Hq, 128]
    # Per element: P is rounded to bf16 before the PV product (2^-9 relative
    # per weight, so at most 2^-9 * sum_j p_j |v_j| on the output), the output
    # rounds to bf16 once (2^-9 |o|); the bound allows twice each.
    spread = (pr @ vf.abs()).transpose(0, 1)
    bound = 2 ** -8 * spread + 2 ** -8 * ref.abs() + 1e-6
    err = (o.float() - ref).abs()
    assert bool((err <= bound).all()), float((err / bound).max())


def test_verify_attention_fully_masked_row_is_zero():
    bf = torch.bfloat16
    g = torch.Generator(device=DEV).manual_seed(3)
    q = torch.randn(32, 32, 128, generator=g, device=DEV).to(bf)
    kc = torch.randn(8, 500, 128, generator=g, device=DEV).to(bf)
    vc = torch.randn(8, 500, 128, generator=g, device=DEV).to(bf)
    mask = torch.ones(32, 500, dtype=torch.bool, device=DEV)
    mask[5] = False
    with torch.inference_mode():
        o = verify_attention(q, kc, vc, 500, mask, 0.1).view(32, 32, 128)
    assert bool((o[5] == 0).all()) and bool(torch.isfinite(o.float()).all())
