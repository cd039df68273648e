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
    pos, rs, tl, flags = K.segment_meta(torch.from_numpy(seq).to(dev), tile=128)
    torch.cuda.synchronize()
    ref = opol.position_ids(seq)
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
