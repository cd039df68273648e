"""K13 (the QKV projection with K2 as its epilogue) against its definition.

mb_qkv_append must give what the fp32-residual decode layer computed before
it: the fp32 GEMM x W^T (+ bias) followed by mb_kv_append_f32 (q/k RMSNorm,
RoPE, bf16 q, k/v at their page slots). The two differ only in the GEMM's
order of summation, so nearly every bf16 output is the same and the rest
differ by a rounding step. The RoPE table is checked against float64 NumPy.
Shapes: the decode model's (hd 128, q/k norms), the large-batch model's
(hd 64, no norms) and a small one with a bias; token counts that are not a
multiple of the 128-token tile; slots of -1 (rows that sit out a step).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


CASES = [
    # T, hidden, Hq, Hkv, hd, norms, bias, page
    (256, 1024, 16, 8, 128, True, False, 128),
    (300, 2048, 32, 8, 64, False, False, 64),
    (5, 512, 4, 2, 128, True, True, 64),
]


@pytest.mark.parametrize("T,hidden,Hq,Hkv,hd,norms,bias,page", CASES)
def test_qkv_append_matches_gemm_then_kv_append(T, hidden, Hq, Hkv, hd, norms, bias, page):
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    g = torch.Generator(device=dev).manual_seed(T + hd)
    N = (Hq + 2 * Hkv) * hd
    x = (torch.randn(T, hidden, generator=g, device=dev)).bfloat16()
    w = (torch.randn(N, hidden, generator=g, device=dev) * hidden ** -0.5).bfloat16()
    b = (torch.randn(N, generator=g, device=dev) * 0.1).bfloat16() if bias else None
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device=dev)).bfloat16() if norms else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device=dev)).bfloat16() if norms else None
    rng = np.random.default_rng(T)
    pos = torch.from_numpy(rng.integers(0, 8192, size=T).astype(np.int32)).to(dev)
    P = (T + page - 1) // page + 3
    slots = rng.permutation(P * page)[:T].astype(np.int32)
    slots[::7] = -1  # rows that sit out: q only
    slot = torch.from_numpy(slots).to(dev)
    inv_freq = (1e6 ** (-torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd)).contiguous()
    scaling = 1.0 if norms else 0.9

    kp_ref = torch.full((P, Hkv, page, hd), 3.0, dtype=torch.bfloat16, device=dev)
    vp_ref = kp_ref.clone()
    qkv = torch.mm(x, w.t(), out_dtype=torch.float32)
    if b is not None:
        qkv = qkv + b.float()
    q_ref = K.kv_append(qkv, pos, Hq, Hkv, hd, inv_freq, scaling, qn, kn, 1e-6, slot=slot, k_pool=kp_ref,
                        v_pool=vp_ref)

    kp, vp = torch.full_like(kp_ref, 3.0), torch.full_like(vp_ref, 3.0)
    rope = K.rope_table(pos, inv_freq, hd, scaling)
    q = K.qkv_append(x, w, b, rope, Hq, Hkv, hd, qn, kn, 1e-6, slot=slot, k_pool=kp, v_pool=vp)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    ang = pos.cpu().double().numpy()[:, None] * inv_freq.cpu().double().numpy()[None, :]
    want = np.stack([np.cos(ang), np.sin(ang)], -1) * scaling
    assert np.abs(rope.cpu().double().numpy() - want).max() < 2e-3  # fp32 argument of up to 8192 rad

    for name, got, ref in (("q", q, q_ref), ("k_pool", kp, kp_ref), ("v_pool", vp, vp_ref)):
        got, ref = got.float(), ref.float()
        same = float((got == ref).float().mean())
        assert same > 0.97, f"{name}: only {same:.4f} of the elements equal"
        # Elsewhere a rounding step of bf16 (8 bits) of the larger magnitude.
        bound = 2 ** -7 * torch.maximum(got.abs(), ref.abs()) + 1e-6
        assert bool(((got - ref).abs() <= bound).all()), f"{name}: a difference beyond one bf16 step"
    untouched = torch.ones(P * page, dtype=torch.bool)
    untouched[torch.from_numpy(slots[slots >= 0]).long()] = False
    flat = kp.permute(0, 2, 1, 3).reshape(P * page, Hkv, hd)
    assert bool((flat[untouched.to(dev)] == 3.0).all()), "a slot that no token owns was written"


def test_qkv_append_rejects_bad_shapes():
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    x = torch.zeros(4, 64, dtype=torch.bfloat16, device=dev)
    rope = torch.zeros(4, 64, 2, dtype=torch.float32, device=dev)
    with pytest.raises(ValueError):
        K.qkv_append(x, torch.zeros(100, 64, dtype=torch.bfloat16, device=dev), None, rope, 1, 1, 128)
    w = torch.zeros(3 * 64, 64, dtype=torch.bfloat16, device=dev)  # 3 heads of 64: not whole 128-row tiles
    with pytest.raises(_lib.KernelError, match="multiple of 128"):
        K.qkv_append(x, w, None, torch.zeros(4, 32, 2, dtype=torch.float32, device=dev), 1, 1, 64)
