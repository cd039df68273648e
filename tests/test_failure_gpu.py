"""Failure detection on the GPU without a GPU fault.

Every wait in the kernels is bounded: after a limit of clock cycles it records
a code in the device status word and its CTA stops cleanly (the consumers
leave together at a barrier, the producer lets the loads it issued land, and
nothing of an incomplete item is written). Here the limit is set to 0 through
the C ABI (``mb_set_wait_limit``), so a healthy decode-attention pipeline's
first wait that does not succeed at once runs out: the launch must still
finish, the host must read a timeout code (1: a consumer, 2: the producer)
from ``mb_device_status``, and — with the default limit back — the same call
must match the oracle again, so the context is still usable.

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


@pytest.mark.parametrize("S", [1, 40])  # split mode (work list + merges) and block mode (prefill rows)
def test_decode_attention_wait_timeout_is_reported_and_recovers(S):
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    B, Hq, Hkv, hd, page = 6, 16, 8, 128, 128
    n_new = [S] * B
    lens_after = [3000, 5000 if S == 1 else 700, 2049, 129, 4100 if S == 1 else 900, 64]
    q, kp, vp, bt, q_pos, k_rows, v_rows = _paged_case(B, Hq, Hkv, hd, page, S, lens_after, n_new, 21 + S)
    args = (q.to(dev), kp.to(dev), vp.to(dev), torch.from_numpy(bt).to(dev), torch.from_numpy(q_pos).to(dev),
            torch.tensor(lens_after, dtype=torch.int32, device=dev), hd ** -0.5, max(lens_after))
    assert _lib.device_status() == 0
    codes = []
    try:
        _lib.set_wait_limit(0)
        for _ in range(5):  # each launch must finish; some wait of the pipeline runs out
            K.decode_attention(*args)
            torch.cuda.synchronize()
            codes.append(_lib.device_status())
            if codes[-1]:
                break
    finally:
        _lib.set_wait_limit(None)
    assert any(c in TIMEOUT_CODES for c in codes), codes
    assert all(c in (0,) + TIMEOUT_CODES for c in codes), codes
    # Default limit again: the context is usable and the kernel exact.
    out = K.decode_attention(*args)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    ref = oatt.cached_decode_attention(q.float().numpy(), [k.float().numpy() for k in k_rows],
                                       [v.float().numpy() for v in v_rows], q_pos, hd ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL
