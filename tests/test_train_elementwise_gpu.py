"""K4 training element-wise kernels against plain PyTorch fp32 references of
the same ops (autograd for the gradients), through the C ABI.

Tolerances: outputs and input gradients within 2e-2 max-abs of fp32 scaled by
the reference's magnitude; weight gradients (sums over thousands of rows)
within 1e-2 relative L2. The forwards also follow the transformers modules'
own bf16 rounding steps (differences of at most two bf16 ulps, rare)."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def _maxabs(a, b):
    return float((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-12))


def _rmsnorm_fp32(x, w, eps):
    var = x.pow(2).mean(-1, keepdim=True)
    return w * (x * torch.rsqrt(var + eps))


@pytest.mark.parametrize("rows,dim", [(1, 256), (777, 1024), (4096, 2048), (300, 768)])
def test_rmsnorm_fwd_bwd(rows, dim):
    dev = _dev()
    from mouse_core_b200 import kernels as K
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    g = torch.Generator(device="cpu").manual_seed(rows + dim)
    x = (torch.randn(rows, dim, generator=g) * 3).bfloat16().to(dev)
    w = (1 + 0.2 * torch.randn(dim, generator=g)).bfloat16().to(dev)
    dy = torch.randn(rows, dim, generator=g).bfloat16().to(dev)
    y, rstd = K.rmsnorm_fwd(x, w, 1e-6)

    mod = Qwen3RMSNorm(dim, eps=1e-6).to(dev, torch.bfloat16)
    with torch.no_grad():
        mod.weight.copy_(w)
        y_mod = mod(x)
    # the module's own bf16 steps: rstd may differ in its last fp32 bit, which
    # moves a rounding by at most one ulp of bf16(x * rstd) and of the product
    ulp = y_mod.float().abs() * 2.0 ** -7 + 1e-30
    assert bool(((y.float() - y_mod.float()).abs() <= 2 * ulp).all())
    assert float((y != y_mod).float().mean()) < 1e-2

    xf = x.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    yf = _rmsnorm_fp32(xf, wf, 1e-6)
    (yf * dy.float()).sum().backward()
    assert _maxabs(y, yf.detach()) < 2e-2
    assert torch.allclose(rstd, torch.rsqrt(x.float().pow(2).mean(-1) + 1e-6), rtol=1e-5)

    dx, dw = K.rmsnorm_bwd(dy, x, w, rstd)
    assert dw.dtype == torch.float32
    assert _maxabs(dx, xf.grad) < 2e-2
    assert _rel(dw, wf.grad) < 1e-2


def test_rmsnorm_rejects_unsupported_width():
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    x = torch.zeros(4, 320, dtype=torch.bfloat16, device=dev)
    with pytest.raises(_lib.KernelError, match="256"):
        K.rmsnorm_fwd(x, torch.ones(320, dtype=torch.bfloat16, device=dev), 1e-6)


def _rope_fp32(x, cos, sin):
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos + rot * sin


@pytest.mark.parametrize("hd,norm", [(128, True), (64, True), (128, False)])
def test_qk_norm_rope_fwd_bwd_strided(hd, norm):
    dev = _dev()
    from mouse_core_b200 import kernels as K

    L, Hq, Hkv = 1000, 4, 2
    g = torch.Generator(device="cpu").manual_seed(hd)
    width = (Hq + 2 * Hkv) * hd
    qkv = (torch.randn(L, width, generator=g) * 2).bfloat16().to(dev)
    w = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16().to(dev) if norm else None
    pos = torch.arange(L) % 333
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2).float() / hd))
    ang = pos[:, None].float() * inv[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    cos, sin = ang.cos().bfloat16().to(dev), ang.sin().bfloat16().to(dev)

    xk = qkv[:, Hq * hd:(Hq + Hkv) * hd]  # the k columns: strided rows
    y, rstd = K.qk_norm_rope_fwd(xk, Hkv, hd, w, 1e-6, cos, sin)
    assert y.shape == (L, Hkv, hd) and (rstd is None) == (not norm)

    xf = xk.float().reshape(L, Hkv, hd).requires_grad_(True)
    wf = w.float().requires_grad_(True) if norm else None
    n = _rmsnorm_fp32(xf, wf, 1e-6) if norm else xf
    yf = _rope_fp32(n, cos.float()[:, None, :], sin.float()[:, None, :])
    dy = torch.randn(L, Hkv, hd, generator=g).bfloat16().to(dev)
    (yf * dy.float()).sum().backward()
    assert _maxabs(y, yf.detach()) < 2e-2

    dqkv = torch.zeros_like(qkv)
    dw = K.qk_norm_rope_bwd(dy, xk, w, cos, sin, rstd, dqkv[:, Hq * hd:(Hq + Hkv) * hd])
    dx = dqkv[:, Hq * hd:(Hq + Hkv) * hd].reshape(L, Hkv, hd)
    assert _maxabs(dx, xf.grad) < 2e-2
    # the kernel writes only its own columns of the fused gradient
    assert not dqkv[:, :Hq * hd].any() and not dqkv[:, (Hq + Hkv) * hd:].any()
    if norm:
        assert _rel(dw, wf.grad) < 1e-2
    else:
        assert dw is None


def test_qk_norm_rope_matches_module_rounding():
    """Forward equals Qwen3's q_norm followed by apply_rotary_pos_emb in bf16
    to within one bf16 ulp (the same rounding after each op)."""
    dev = _dev()
    from mouse_core_b200 import kernels as K
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

    L, H, hd = 513, 3, 128
    g = torch.Generator(device="cpu").manual_seed(9)
    x = torch.randn(L, H * hd, generator=g).bfloat16().to(dev)
    w = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16().to(dev)
    ang = torch.arange(L)[:, None].float() * (1.0 / (1e6 ** (torch.arange(0, hd, 2).float() / hd)))[None]
    ang = torch.cat((ang, ang), dim=-1)
    cos, sin = ang.cos().bfloat16().to(dev), ang.sin().bfloat16().to(dev)
    y, _ = K.qk_norm_rope_fwd(x, H, hd, w, 1e-6, cos, sin)
    mod = Qwen3RMSNorm(hd, eps=1e-6).to(dev, torch.bfloat16)
    with torch.no_grad():
        mod.weight.copy_(w)
        n = mod(x.view(1, L, H, hd)).transpose(1, 2)  # [1, H, L, hd]
        ref, _ = apply_rotary_pos_emb(n, n, cos[None], sin[None])
    ref = ref[0].transpose(0, 1)
    ulp = ref.float().abs() * 2.0 ** -7 + 2.0 ** -14
    assert float(((y.float() - ref.float()).abs() > 2 * ulp).float().mean()) < 1e-3


@pytest.mark.parametrize("rows,inter", [(1, 2), (1000, 3072), (257, 1000)])
def test_silu_mul_fwd_bwd(rows, inter):
    dev = _dev()
    from mouse_core_b200 import kernels as K

    g = torch.Generator(device="cpu").manual_seed(rows)
    gu = (torch.randn(rows, 2 * inter, generator=g) * 3).bfloat16().to(dev)
    dh = torch.randn(rows, inter, generator=g).bfloat16().to(dev)
    h = K.silu_mul(gu)
    # the module's rounding: bf16(silu(gate)) * up, rounded
    g16, u16 = gu[:, :inter], gu[:, inter:]
    ref = torch.nn.functional.silu(g16) * u16
    ulp = ref.float().abs() * 2.0 ** -7 + 1e-30
    assert bool(((h.float() - ref.float()).abs() <= ulp).all())
    assert float((h != ref).float().mean()) < 1e-3

    guf = gu.float().requires_grad_(True)
    hf = torch.nn.functional.silu(guf[:, :inter]) * guf[:, inter:]
    (hf * dh.float()).sum().backward()
    dgu = K.silu_mul_bwd(gu, dh)
    assert _maxabs(dgu, guf.grad) < 2e-2
