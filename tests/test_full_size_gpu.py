"""Parity at the benchmark workloads' full sizes, through properties that do
not need the oracle to run the whole workload.

* K1 on the decode benchmark's exact attention shape (256 rows, cached
  lengths U[64,4096], 16/8 heads, hd 128, 128-token pages scattered through a
  shuffled pool): rows are independent, so sampled rows (the longest, the
  shortest and random ones) must equal the float64 oracle run on that row
  alone.
* K5 + K6 (stored dS) on the packed-training benchmark's exact stream (8 rows
  x 16384 tokens, 64 segments U[256,4096], 16/8 heads, hd 128): segments are
  independent, so each sampled segment's outputs and gradients must equal the
  oracle run on that segment alone.

Tolerance: 2e-2 max-abs, scaled by the reference's largest magnitude when
that exceeds 1 (bf16 inputs and outputs, fp32 accumulation)."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _close(got, ref, what):
    scale = max(1.0, float(np.abs(ref).max()))
    err = float(np.abs(got - ref).max())
    assert err <= ATOL * scale, f"{what}: max abs err {err} (scale {scale})"


def test_decode_attention_full_decode_workload():
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    B, Hq, Hkv, hd, page = 256, 16, 8, 128, 128
    rng = np.random.default_rng(11)
    lens = rng.integers(64, 4097, size=B) + 1  # after this step's append
    npg = (lens + page - 1) // page
    P = int(npg.sum()) + 7
    perm = rng.permutation(P).astype(np.int32)
    bt = np.full((B, int(npg.max())), -1, dtype=np.int32)
    o = 0
    for b in range(B):
        bt[b, :npg[b]] = perm[o:o + npg[b]]
        o += npg[b]
    g = torch.Generator(device=dev).manual_seed(5)
    kp = torch.randn(P, Hkv, page, hd, generator=g, device=dev).bfloat16()
    vp = torch.randn(P, Hkv, page, hd, generator=g, device=dev).bfloat16()
    q = torch.randn(B, 1, Hq, hd, generator=g, device=dev).bfloat16()
    q_pos = (lens - 1).astype(np.int32).reshape(B, 1)
    scale = hd ** -0.5
    out = K.decode_attention(q, kp, vp, torch.from_numpy(bt).to(dev), torch.from_numpy(q_pos).to(dev),
                             torch.from_numpy(lens.astype(np.int32)).to(dev), scale, int(lens.max()))
    out = out.float().cpu().numpy()
    rows = sorted({int(np.argmax(lens)), int(np.argmin(lens))} | set(rng.choice(B, size=4, replace=False).tolist()))
    for b in rows:
        pages = torch.from_numpy(bt[b, :npg[b]].astype(np.int64)).to(dev)
        k_row = kp[pages].permute(0, 2, 1, 3).reshape(-1, Hkv, hd)[:lens[b]].float().cpu().numpy()
        v_row = vp[pages].permute(0, 2, 1, 3).reshape(-1, Hkv, hd)[:lens[b]].float().cpu().numpy()
        ref = oatt.cached_decode_attention(q[b:b + 1].float().cpu().numpy(), [k_row], [v_row], q_pos[b:b + 1],
                                           scale)
        _close(out[b:b + 1], ref, f"row {b} (length {lens[b]})")
    assert _lib.device_status() == 0


def _training_segments(seed=0, rows=8, row_len=16384, lo=256, hi=4096):
    """Per row, lengths U[lo, hi] until the row is full, the last truncated
    (the packed-training benchmark's stream)."""
    rng = np.random.default_rng(seed)
    segs = []
    for _ in range(rows):
        total = 0
        while total < row_len:
            s = min(int(rng.integers(lo, hi + 1)), row_len - total)
            segs.append(s)
            total += s
    return segs


def test_packed_attention_full_training_stream_segments():
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.packed import pair_count

    segs = _training_segments()
    seq = np.concatenate([np.full(n, i, dtype=np.int64) for i, n in enumerate(segs)])
    L, Hq, Hkv, hd = seq.shape[0], 16, 8, 128
    assert L == 8 * 16384 and len(segs) == 64
    g = torch.Generator(device=dev).manual_seed(7)
    q = torch.randn(L, Hq, hd, generator=g, device=dev).bfloat16()
    k = torch.randn(L, Hkv, hd, generator=g, device=dev).bfloat16()
    v = torch.randn(L, Hkv, hd, generator=g, device=dev).bfloat16()
    do = torch.randn(L, Hq, hd, generator=g, device=dev).bfloat16()
    scale = hd ** -0.5
    _, rs, tl, _, re = K.segment_meta(torch.from_numpy(seq).to(dev), tile=128, with_run_end=True)
    out, lse = K.varlen_attention_fwd(q, k, v, rs, tl, scale)
    dq, dk, dv = K.varlen_attention_bwd(q, k, v, out, do, lse, rs, re, scale, tile_lo=tl,
                                        pair_off=K.varlen_pair_offsets(tl, L), n_pairs=pair_count(seq))
    torch.cuda.synchronize()
    starts = np.concatenate([[0], np.cumsum(segs)[:-1]])
    order = np.argsort(segs)
    # the three shortest segments, and the first segment that straddles a 128-token tile boundary
    picks = list(order[:3]) + [next(i for i in range(len(segs)) if starts[i] % 128 and segs[i] <= 900)]
    for i in picks:
        a, n = int(starts[i]), int(segs[i])
        one = np.zeros(n, dtype=np.int64)
        qs, ks, vs, dos = (t[a:a + n].float().cpu().numpy() for t in (q, k, v, do))
        ref_out, _ = oatt.packed_attention_fwd(qs, ks, vs, one, scale)
        ref_dq, ref_dk, ref_dv = oatt.packed_attention_bwd(qs, ks, vs, one, scale, dos)
        for name, got, ref in (("out", out, ref_out), ("dq", dq, ref_dq), ("dk", dk, ref_dk), ("dv", dv, ref_dv)):
            _close(got[a:a + n].float().cpu().numpy(), ref, f"segment {i} ({n} tokens at {a}) {name}")
    assert math.isfinite(float(dq.float().abs().max())) and math.isfinite(float(dk.float().abs().max()))
    assert _lib.device_status() == 0
