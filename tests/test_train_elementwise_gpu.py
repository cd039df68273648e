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


@pytest.mark.parametrize("rows,dim", [(1, 256), (777, 1024), (300, 2048)])
def test_add_rmsnorm_fwd_bwd(rows, dim):
    """The residual add fused in front of the norm: the sum equals the bf16
    add bit for bit, the norm follows the module's rounding; the backward with
    the residual-path gradient equals fp32 autograd of sum -> (sum, norm)."""
    dev = _dev()
    from mouse_core_b200 import kernels as K
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm

    g = torch.Generator(device="cpu").manual_seed(rows * 7 + dim)
    a = (torch.randn(rows, dim, generator=g) * 2).bfloat16().to(dev)
    b = (torch.randn(rows, dim, generator=g) * 2).bfloat16().to(dev)
    w = (1 + 0.2 * torch.randn(dim, generator=g)).bfloat16().to(dev)
    dy = torch.randn(rows, dim, generator=g).bfloat16().to(dev)
    ds = torch.randn(rows, dim, generator=g).bfloat16().to(dev)
    total, y, rstd = K.add_rmsnorm_fwd(a, b, w, 1e-6)
    assert torch.equal(total, b + a)
    mod = Qwen3RMSNorm(dim, eps=1e-6).to(dev, torch.bfloat16)
    with torch.no_grad():
        mod.weight.copy_(w)
        y_mod = mod(b + a)
    ulp = y_mod.float().abs() * 2.0 ** -7 + 1e-30
    assert bool(((y.float() - y_mod.float()).abs() <= 2 * ulp).all())

    sf = total.float().requires_grad_(True)
    wf = w.float().requires_grad_(True)
    yf = _rmsnorm_fp32(sf, wf, 1e-6)
    ((yf * dy.float()).sum() + (sf * ds.float()).sum()).backward()
    dx, dw = K.rmsnorm_bwd(dy, total, w, rstd, dsum=ds)
    assert _maxabs(dx, sf.grad) < 2e-2
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


def _tables(L, hd, period=333):
    pos = torch.arange(L) % period
    inv = 1.0 / (1e6 ** (torch.arange(0, hd, 2).float() / hd))
    ang = pos[:, None].float() * inv[None, :]
    ang = torch.cat((ang, ang), dim=-1)
    return ang.cos().bfloat16(), ang.sin().bfloat16()


@pytest.mark.parametrize("hd,Hq,Hkv,norm,pad", [(128, 16, 8, True, 0), (64, 4, 2, True, 0), (128, 4, 2, False, 0),
                                                (64, 6, 1, True, 64), (128, 3, 1, True, 8)])
def test_qkv_heads_fwd_bwd(hd, Hq, Hkv, norm, pad):
    """q/k norm + RoPE and the v copy from one (optionally row-padded) fused
    projection, and the gradient written back into the whole fused gradient."""
    dev = _dev()
    from mouse_core_b200 import kernels as K

    L = 1000
    g = torch.Generator(device="cpu").manual_seed(hd + Hq)
    width = (Hq + 2 * Hkv) * hd
    store = (torch.randn(L, width + pad, generator=g) * 2).bfloat16().to(dev)
    qkv = store[:, :width]  # row stride width + pad
    qw = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16().to(dev) if norm else None
    kw = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16().to(dev) if norm else None
    cos, sin = (t.to(dev) for t in _tables(L, hd))
    q, k, v, q_rstd, k_rstd = K.qkv_heads_fwd(qkv, Hq, Hkv, hd, cos, sin, qw, kw, 1e-6, 1e-5)
    assert (q_rstd is None) == (not norm)
    assert torch.equal(v, qkv[:, (Hq + Hkv) * hd:].reshape(L, Hkv, hd))

    xf = qkv.float().requires_grad_(True)
    xq = xf[:, :Hq * hd].reshape(L, Hq, hd)
    xk = xf[:, Hq * hd:(Hq + Hkv) * hd].reshape(L, Hkv, hd)
    xv = xf[:, (Hq + Hkv) * hd:].reshape(L, Hkv, hd)
    if norm:
        qwf = qw.float().requires_grad_(True)
        kwf = kw.float().requires_grad_(True)
        xq, xk = _rmsnorm_fp32(xq, qwf, 1e-6), _rmsnorm_fp32(xk, kwf, 1e-5)
    c, s_ = cos.float()[:, None, :], sin.float()[:, None, :]
    qf, kf = _rope_fp32(xq, c, s_), _rope_fp32(xk, c, s_)
    assert _maxabs(q, qf.detach()) < 2e-2 and _maxabs(k, kf.detach()) < 2e-2
    dq = torch.randn(L, Hq, hd, generator=g).bfloat16().to(dev)
    dk = torch.randn(L, Hkv, hd, generator=g).bfloat16().to(dev)
    dv = torch.randn(L, Hkv, hd, generator=g).bfloat16().to(dev)
    ((qf * dq.float()).sum() + (kf * dk.float()).sum() + (xv * dv.float()).sum()).backward()

    dstore = torch.zeros(L, width + 16, dtype=torch.bfloat16, device=dev)
    dqkv, dqw, dkw = K.qkv_heads_bwd(dq, dk, dv, qkv, cos, sin, qw, kw, q_rstd, k_rstd, dqkv=dstore[:, :width])
    assert _maxabs(dqkv[:, :(Hq + Hkv) * hd], xf.grad[:, :(Hq + Hkv) * hd]) < 2e-2
    assert torch.equal(dqkv[:, (Hq + Hkv) * hd:], dv.reshape(L, -1))
    assert not dstore[:, width:].any()  # the row padding is never written
    if norm:
        assert _rel(dqw, qwf.grad) < 1e-2 and _rel(dkw, kwf.grad) < 1e-2
    else:
        assert dqw is None and dkw is None


def test_qkv_heads_match_module_rounding():
    """q equals Qwen3's q_norm followed by apply_rotary_pos_emb in bf16 up to
    rare two-ulp differences (the same rounding after each op)."""
    dev = _dev()
    from mouse_core_b200 import kernels as K
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb

    L, H, Hkv, hd = 513, 4, 2, 128
    g = torch.Generator(device="cpu").manual_seed(9)
    qkv = torch.randn(L, (H + 2 * Hkv) * hd, generator=g).bfloat16().to(dev)
    w = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16().to(dev)
    cos, sin = (t.to(dev) for t in _tables(L, hd, period=L))
    q, _, _, _, _ = K.qkv_heads_fwd(qkv, H, Hkv, hd, cos, sin, w, w, 1e-6, 1e-6)
    mod = Qwen3RMSNorm(hd, eps=1e-6).to(dev, torch.bfloat16)
    with torch.no_grad():
        mod.weight.copy_(w)
        n = mod(qkv[:, :H * hd].reshape(1, L, H, hd)).transpose(1, 2)  # [1, H, L, hd]
        ref, _ = apply_rotary_pos_emb(n, n, cos[None], sin[None])
    ref = ref[0].transpose(0, 1)
    ulp = ref.float().abs() * 2.0 ** -7 + 2.0 ** -14
    assert float(((q.float() - ref.float()).abs() > 2 * ulp).float().mean()) < 1e-3


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
