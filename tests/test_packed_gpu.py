"""GPU parity of the packed-training path: K7 segment metadata (bit-exact with
the oracle) and the K5 tcgen05 segment-causal attention forward (within 2e-2
max-abs of the float64 oracle on the same bf16 inputs; lse within 1e-2 in
log2 units). The oracle is pinned to the reference's SDPA-mask path by
tests/test_oracle_golden.py; the 2048-token case is also checked against the
reference's own sampled outputs."""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import policy as opol
from tests.golden_io import cfg1_inputs, cfg1_segments, load

pytestmark = pytest.mark.gpu

ATOL = 2e-2
LOG2E = 1.0 / math.log(2.0)


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


def _seq_from_lengths(lengths):
    return np.concatenate([np.full(n, i, dtype=np.int64) for i, n in enumerate(lengths)])


@pytest.mark.parametrize("case", ["sorted", "unsorted", "single", "tiny"])
def test_segment_meta_bit_exact(case):
    dev = _dev()
    from mouse_core_b200 import kernels as K

    rng = np.random.default_rng(5)
    if case == "sorted":
        seq = _seq_from_lengths(rng.integers(1, 700, size=40))
    elif case == "unsorted":
        seq = np.array([0, 0, 3, 3, 3, 1, 1, 0, 2] * 500, dtype=np.int64)
    elif case == "single":
        seq = np.zeros(9000, dtype=np.int64)
    else:
        seq = np.array([7], dtype=np.int64)
    pos, rs, tl, flags, re = K.segment_meta(torch.from_numpy(seq).to(dev), tile=128, with_run_end=True)
    torch.cuda.synchronize()
    ref = opol.position_ids(seq)
    L = seq.shape[0]
    boundary = np.ones(L + 1, dtype=bool)
    boundary[1:L] = seq[1:] != seq[:-1]
    nxt = np.empty(L, dtype=np.int64)
    cur = L
    for i in range(L - 1, -1, -1):
        nxt[i] = cur
        if boundary[i]:
            cur = i
    assert np.array_equal(re.cpu().numpy(), nxt)
    assert np.array_equal(pos.cpu().numpy(), ref)
    assert np.array_equal(rs.cpu().numpy(), np.arange(seq.shape[0]) - ref)
    assert np.array_equal(tl.cpu().numpy(), (np.arange(seq.shape[0]) - ref)[::128])
    assert int(flags.item()) == int(np.any(np.diff(seq) < 0))


def _run_fwd(seq, q, k, v, dev):
    from mouse_core_b200 import kernels as K

    st = torch.from_numpy(seq).to(dev)
    _, rs, tl, flags = K.segment_meta(st, tile=128)
    assert int(flags.item()) == 0
    out, lse = K.varlen_attention_fwd(q.to(dev), k.to(dev), v.to(dev), rs, tl, q.shape[-1] ** -0.5)
    torch.cuda.synchronize()
    return out.float().cpu().numpy(), lse.cpu().numpy()


FWD_CASES = [
    # name, Hq, Hkv, hd, segment lengths
    ("g2_hd128", 16, 8, 128, [1, 700, 3, 129, 1, 127, 40]),
    ("g1_hd128", 4, 4, 128, [300]),
    ("g4_hd64", 8, 2, 64, [17, 256, 244]),
    ("g2_hd64_long", 4, 2, 64, [2048]),
]


@pytest.mark.parametrize("name,Hq,Hkv,hd,lens", FWD_CASES)
def test_varlen_fwd_matches_oracle(name, Hq, Hkv, hd, lens):
    dev = _dev()
    seq = _seq_from_lengths(lens)
    L = seq.shape[0]
    q, k, v, _ = cfg1_inputs(11, L, Hq, Hkv, hd)
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out, lse = _run_fwd(seq, q, k, v, dev)
    ref, ref_lse = oatt.packed_attention_fwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), seq,
                                             hd ** -0.5)
    assert np.isfinite(out).all()
    err = np.abs(out - ref).max()
    assert err < ATOL, f"{name}: out max abs err {err}"
    lerr = np.abs(lse - ref_lse * LOG2E).max()
    assert lerr < 1e-2, f"{name}: lse max abs err {lerr}"
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


def test_varlen_fwd_packed_2048_against_reference_samples():
    """The 2048-token packed workload (segments U[16,512], 4/2 heads, hd 64):
    bf16 kernel vs the reference's fp32 SDPA-mask outputs (sampled)."""
    dev = _dev()
    g = load("packed_attn_cfg1.npz")
    segs = cfg1_segments(0)
    seq = _seq_from_lengths(segs)
    q, k, v, _ = cfg1_inputs(0, 2048, 4, 2, 64)
    out, _ = _run_fwd(seq, q.bfloat16(), k.bfloat16(), v.bfloat16(), dev)
    flat = out.reshape(-1)
    err = np.abs(flat[g["out_idx"]] - g["out_val"]).max()
    assert err < ATOL, f"max abs err vs reference samples {err}"


def _run_bwd(seq, q, k, v, do, dev):
    from mouse_core_b200 import kernels as K

    st = torch.from_numpy(seq).to(dev)
    _, rs, tl, flags, re = K.segment_meta(st, tile=128, with_run_end=True)
    qd, kd, vd, dod = q.to(dev), k.to(dev), v.to(dev), do.to(dev)
    scale = q.shape[-1] ** -0.5
    out, lse = K.varlen_attention_fwd(qd, kd, vd, rs, tl, scale)
    dq, dk, dv = K.varlen_attention_bwd(qd, kd, vd, out, dod, lse, rs, re, scale)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (dq, dk, dv)]


BWD_CASES = FWD_CASES + [("g2_hd128_many", 4, 2, 128, [5, 300, 1, 1, 1, 64, 129, 600])]


@pytest.mark.parametrize("name,Hq,Hkv,hd,lens", BWD_CASES)
def test_varlen_bwd_matches_oracle(name, Hq, Hkv, hd, lens):
    """dq, dk, dv (bf16, fp32 accumulation) vs the float64 analytic gradient on
    the same bf16 inputs: max-abs error within 2e-2 of each gradient's scale
    (its largest magnitude, at least 1)."""
    dev = _dev()
    seq = _seq_from_lengths(lens)
    L = seq.shape[0]
    q, k, v, do = cfg1_inputs(13, L, Hq, Hkv, hd)
    q, k, v, do = q.bfloat16(), k.bfloat16(), v.bfloat16(), do.bfloat16()
    got = _run_bwd(seq, q, k, v, do, dev)
    ref = oatt.packed_attention_bwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), seq, hd ** -0.5,
                                    do.float().numpy())
    for gname, g, r in zip(("dq", "dk", "dv"), got, ref):
        assert np.isfinite(g).all(), gname
        scale = max(1.0, float(np.abs(r).max()))
        err = np.abs(g - r).max()
        assert err <= ATOL * scale, f"{name} {gname}: max abs err {err} (scale {scale})"
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


def test_varlen_bwd_packed_2048_against_reference_samples():
    """Gradients of the 2048-token packed workload vs the reference's fp32
    SDPA-mask autograd (sampled entries)."""
    dev = _dev()
    g = load("packed_attn_cfg1.npz")
    seq = _seq_from_lengths(cfg1_segments(0))
    q, k, v, do = cfg1_inputs(0, 2048, 4, 2, 64)
    got = _run_bwd(seq, q.bfloat16(), k.bfloat16(), v.bfloat16(), do.bfloat16(), dev)
    for gname, arr in zip(("dq", "dk", "dv"), got):
        ref = g[f"{gname}_val"]
        scale = max(1.0, float(np.abs(ref).max()))
        err = np.abs(arr.reshape(-1)[g[f"{gname}_idx"]] - ref).max()
        assert err <= ATOL * scale, f"{gname}: max abs err vs reference samples {err}"
