"""Failure detection on the GPU without a GPU fault.

Every wait in the kernels is bounded: after a limit of clock cycles it records
a code in the device status word and its CTA stops cleanly. In K1 the
consumers leave together at a barrier and the producer lets the loads it
issued land; in the tcgen05 kernels (the paged prefill, the packed forward
and the three backward kernels) the producer warp lets every TMA load it
issued land and the MMA warp commits every MMA it issued to a barrier of its
own and waits for it before TMEM is freed. Nothing of an incomplete item is
written. Here the limit is set to 0 through the C ABI
(``mb_set_wait_limit``), so a healthy pipeline's first wait that does not
succeed at once runs out: each launch must still finish, the host must read a
timeout code (1: a consumer, 2: the producer) from ``mb_device_status``, and
— with the default limit back — the same calls must match the oracle again,
so the context is still usable.

No wait here is on something that never happens, no kernel is broken and no
memory is touched out of bounds: the waits end because their limit is 0.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from tests.test_decode_gpu import _paged_case

pytestmark = pytest.mark.gpu

ATOL = 2e-2
TIMEOUT_CODES = (1, 2)


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


def _timed_out_launches(call):
    """Run ``call`` with a wait limit of 0 until a launch reports a timeout
    (at most 5 launches, each of which must finish); the status codes seen."""
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0
    codes = []
    try:
        _lib.set_wait_limit(0)
        for _ in range(5):
            call()
            torch.cuda.synchronize()
            codes.append(_lib.device_status())
            if codes[-1]:
                break
    finally:
        _lib.set_wait_limit(None)
    assert any(c in TIMEOUT_CODES for c in codes), codes
    assert all(c in (0,) + TIMEOUT_CODES for c in codes), codes
    return codes


# S = 1: split mode (work list + merges); S = 40: block mode (prefill rows);
# S = 70: the tcgen05 paged prefill, one tile per CTA and persistent CTAs
# over a tile counter (a workspace given).
@pytest.mark.parametrize("S,workspace", [(1, False), (40, False), (70, False), (70, True)])
def test_decode_attention_wait_timeout_is_reported_and_recovers(S, workspace):
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    B, Hq, Hkv, hd, page = 6, 16, 8, 128, 128
    n_new = [S] * B
    lens_after = [3000, 5000 if S == 1 else 700, 2049, 129, 4100 if S == 1 else 900, 64 if S < 64 else 96]
    q, kp, vp, bt, q_pos, k_rows, v_rows = _paged_case(B, Hq, Hkv, hd, page, S, lens_after, n_new, 21 + S)
    args = (q.to(dev), kp.to(dev), vp.to(dev), torch.from_numpy(bt).to(dev), torch.from_numpy(q_pos).to(dev),
            torch.tensor(lens_after, dtype=torch.int32, device=dev), hd ** -0.5, max(lens_after))
    kw = {"workspace": torch.empty(256, dtype=torch.uint8, device=dev)} if workspace else {}
    _timed_out_launches(lambda: K.decode_attention(*args, **kw))
    # Default limit again: the context is usable and the kernel exact.
    out = K.decode_attention(*args, **kw)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = oatt.cached_decode_attention(q.float().numpy(), [k.float().numpy() for k in k_rows],
                                       [v.float().numpy() for v in v_rows], q_pos, hd ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL


@pytest.mark.parametrize("stored", [False, True])  # dQ recomputed, or one GEMM over the stored dS blocks
def test_packed_attention_wait_timeout_is_reported_and_recovers(stored):
    """The packed forward and backward (tcgen05, TMEM, TMA rings) with a wait
    limit of 0: every launch finishes and reports a timeout; then, on the
    same context, forward and gradients match the float64 oracle."""
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.packed import pair_count
    from tests.golden_io import cfg1_inputs
    from tests.test_packed_gpu import _seq_from_lengths

    Hq, Hkv, hd = 16, 8, 128
    seq = _seq_from_lengths([1, 700, 3, 129, 1, 127, 40, 300])
    L = seq.shape[0]
    q, k, v, do = (t.bfloat16() for t in cfg1_inputs(31, L, Hq, Hkv, hd))
    qd, kd, vd, dod = q.to(dev), k.to(dev), v.to(dev), do.to(dev)
    _, rs, tl, flags, re = K.segment_meta(torch.from_numpy(seq).to(dev), tile=128, with_run_end=True)
    assert int(flags.item()) == 0
    scale = hd ** -0.5
    extra = {}
    if stored:
        extra = dict(tile_lo=tl, pair_off=K.varlen_pair_offsets(tl, L), n_pairs=pair_count(seq))
    out, lse = K.varlen_attention_fwd(qd, kd, vd, rs, tl, scale)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0

    _timed_out_launches(lambda: K.varlen_attention_fwd(qd, kd, vd, rs, tl, scale))
    _timed_out_launches(lambda: K.varlen_attention_bwd(qd, kd, vd, out, dod, lse, rs, re, scale, **extra))

    # Default limit again: the same calls are exact on the same context.
    out2, lse2 = K.varlen_attention_fwd(qd, kd, vd, rs, tl, scale)
    grads = K.varlen_attention_bwd(qd, kd, vd, out2, dod, lse2, rs, re, scale, **extra)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    qn, kn, vn = q.float().numpy(), k.float().numpy(), v.float().numpy()
    ref, _ = oatt.packed_attention_fwd(qn, kn, vn, seq, scale)
    assert np.abs(out2.float().cpu().numpy() - ref).max() < ATOL
    ref_g = oatt.packed_attention_bwd(qn, kn, vn, seq, scale, do.float().numpy())
    for name, g, r in zip(("dq", "dk", "dv"), grads, ref_g):
        bound = ATOL * max(1.0, float(np.abs(r).max()))
        assert np.abs(g.float().cpu().numpy() - r).max() <= bound, name


def test_qkv_projection_wait_timeout_is_reported_and_recovers():
    """K13 (the QKV GEMM with the K2 epilogue) with a wait limit of 0: each
    launch finishes and reports a timeout; with the default limit back the
    same call gives the GEMM-then-K2 outputs on the same context."""
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    T, hidden, Hq, Hkv, hd = 200, 1024, 16, 8, 128
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(T, hidden, generator=g, device=dev).bfloat16()
    w = (torch.randn((Hq + 2 * Hkv) * hd, hidden, generator=g, device=dev) * hidden ** -0.5).bfloat16()
    pos = torch.arange(T, dtype=torch.int32, device=dev) * 7
    inv_freq = (1e6 ** (-torch.arange(0, hd, 2, device=dev, dtype=torch.float32) / hd)).contiguous()
    rope = K.rope_table(pos, inv_freq, hd)
    _timed_out_launches(lambda: K.qkv_append(x, w, None, rope, Hq, Hkv, hd))
    q = K.qkv_append(x, w, None, rope, Hq, Hkv, hd)
    q_ref = K.kv_append(torch.mm(x, w.t(), out_dtype=torch.float32), pos, Hq, Hkv, hd, inv_freq)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    diff = (q.float() - q_ref.float()).abs()
    assert bool((diff <= 2 ** -7 * torch.maximum(q.float().abs(), q_ref.float().abs()) + 1e-6).all())
