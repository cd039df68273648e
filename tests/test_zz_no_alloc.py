"""mb_decode_attention_noalloc against mb_decode_attention.

Some callers cannot allocate device memory — an FFI caller that only holds
the pointers its framework handed it, or a process whose device memory
belongs to another framework's allocator — so they cannot pass the workspace
mb_decode_attention needs. mb_decode_attention_noalloc runs the same kernels
out of a scratch array compiled into the library. Here it is called through
the C ABI twice in a row, first on a shape with many long rows (many split
work items, so partial results fill much of the scratch), then on a smaller
one that reuses the scratch the first call left behind; each result must
match the workspace entry point within the 2e-2 max-abs tolerance of the
other attention tests, and neither call may change the device memory in use
(torch's allocator or the driver's free-memory count).

This file sorts last so that a run stopping at the first failure has already
run every other test.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

ATOL = 2e-2


def _case(B, Hq, Hkv, hd, page, S, seed, dev, max_before=3000):
    rng = np.random.default_rng(seed)
    n_new = rng.integers(0, S + 1, size=B)
    n_new[0] = S
    before = rng.integers(0, max_before, size=B)
    before[-1] = 0
    lens = (before + n_new).astype(np.int64)
    npg = [math.ceil(int(L) / page) for L in lens]
    P = sum(npg) + 2
    perm = rng.permutation(P).astype(np.int32)
    maxp = max(max(npg), 1)
    bt = np.full((B, maxp), -1, dtype=np.int32)
    i = 0
    for b in range(B):
        for j in range(npg[b]):
            bt[b, j] = perm[i]
            i += 1
    col = np.arange(S)[None, :]
    q_pos = np.maximum(before[:, None] + col - (S - n_new)[:, None], 0).astype(np.int32)
    g = torch.Generator(device=dev).manual_seed(seed)
    q = torch.randn(B, S, Hq, hd, generator=g, device=dev).bfloat16()
    kp = torch.randn(P, Hkv, page, hd, generator=g, device=dev).bfloat16()
    vp = torch.randn(P, Hkv, page, hd, generator=g, device=dev).bfloat16()
    return (q, kp, vp, torch.from_numpy(bt).to(dev), torch.from_numpy(q_pos).to(dev),
            torch.from_numpy(lens.astype(np.int32)).to(dev), int(lens.max()))


@pytest.mark.gpu
def test_noalloc_matches_workspace_entry_point_twice():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import _lib, build
    from mouse_core_b200 import kernels as K

    build.build()
    lib = _lib.load()
    dev = torch.device("cuda")
    # Split mode both times (the scratch is used): the first shape has many
    # long rows, so it lays out more work items and partials than the second.
    shapes = ((96, 16, 8, 128, 128, 1, 1, 12000), (6, 32, 8, 64, 64, 2, 2, 3000))
    cases = []
    for B, Hq, Hkv, hd, page, S, seed, max_before in shapes:
        q, kp, vp, bt, q_pos, kv_len, max_kv = _case(B, Hq, Hkv, hd, page, S, seed, dev, max_before)
        ref = K.decode_attention(q, kp, vp, bt, q_pos, kv_len, hd ** -0.5, max_kv)
        cases.append((B, Hq, Hkv, hd, page, S, q, kp, vp, bt, q_pos, kv_len, max_kv, ref,
                      torch.full_like(q, float("nan"))))
    need = [lib.mb_decode_workspace_bytes(c[0], c[2], (c[1] // c[2]) * c[5], c[3], c[12]) for c in cases]
    assert need[0] > 4 * need[1] and need[0] <= 32 * 1024 * 1024, need
    torch.cuda.synchronize()
    used_before = torch.cuda.memory_allocated()
    free_before, _ = torch.cuda.mem_get_info()
    stream = torch.cuda.current_stream().cuda_stream
    for B, Hq, Hkv, hd, page, S, q, kp, vp, bt, q_pos, kv_len, max_kv, ref, out in cases:
        rc = lib.mb_decode_attention_noalloc(q.data_ptr(), kp.data_ptr(), vp.data_ptr(), kp.shape[0], bt.data_ptr(),
                                             bt.shape[1], q_pos.data_ptr(), kv_len.data_ptr(), B, S, Hq, Hkv, hd,
                                             page, ctypes.c_float(hd ** -0.5), max_kv, out.data_ptr(), stream)
        assert rc == 0, lib.mb_last_error()
    torch.cuda.synchronize()
    free_after, _ = torch.cuda.mem_get_info()
    assert torch.cuda.memory_allocated() == used_before
    # The workspace the first shape would need (several MiB) was never allocated.
    assert free_before - free_after < need[0] // 2, (free_before, free_after, need[0])
    for c in cases:
        ref, out = c[13], c[14]
        assert torch.isfinite(out.float()).all()
        err = (out.float() - ref.float()).abs().max().item()
        assert err <= ATOL, f"noalloc differs from the workspace entry point by {err}"
    assert _lib.device_status() == 0


def test_noalloc_rejects_a_shape_beyond_its_scratch():
    """Argument checking only: returns MB_ERR_WORKSPACE before any CUDA call."""
    from mouse_core_b200 import _lib, build

    build.build()
    lib = _lib.load()
    B, Hq, Hkv, hd, page, S, max_kv = 4096, 32, 8, 128, 128, 4, 16384
    assert lib.mb_decode_workspace_bytes(B, Hkv, (Hq // Hkv) * S, hd, max_kv) > 32 * 1024 * 1024
    rc = lib.mb_decode_attention_noalloc(None, None, None, 1, None, 128, None, None, B, S, Hq, Hkv, hd, page,
                                         ctypes.c_float(0.1), max_kv, None, None)
    assert rc == 3  # MB_ERR_WORKSPACE
    assert b"MB_NOALLOC_SCRATCH_BYTES" in lib.mb_last_error()
