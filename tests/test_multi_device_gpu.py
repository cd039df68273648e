"""One process driving two GPUs: each kernel is prepared for launch per device.

A kernel that needs more than 48 KB of shared memory must have its
shared-memory attribute set on every device it runs on, and the library
caches that set-up (and its occupancy figures) per device. Here the same
inputs go through the tcgen05 kernels (packed forward and backward, the QKV
projection with the K2 epilogue), the decode attention (split and prefill
modes) and the RMSNorm backward on device 0 and then device 1 of one
process; the results must be identical. Skipped with fewer than two GPUs.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _run_all(dev):
    from mouse_core_b200 import kernels as K

    outs = []
    with torch.cuda.device(dev):
        g = torch.Generator(device=dev).manual_seed(0)
        # packed segment-causal attention, forward and stored-dS backward
        seq = np.repeat(np.arange(3), [300, 129, 600]).astype(np.int64)
        L = seq.shape[0]
        q = torch.randn(L, 16, 128, generator=g, device=dev).bfloat16()
        k = torch.randn(L, 8, 128, generator=g, device=dev).bfloat16()
        v = torch.randn(L, 8, 128, generator=g, device=dev).bfloat16()
        do = torch.randn(L, 16, 128, generator=g, device=dev).bfloat16()
        _, rs, tl, _, re = K.segment_meta(torch.from_numpy(seq).to(dev), tile=128, with_run_end=True)
        out, lse = K.varlen_attention_fwd(q, k, v, rs, tl, 128 ** -0.5)
        from mouse_core_b200.packed import pair_count

        grads = K.varlen_attention_bwd(q, k, v, out, do, lse, rs, re, 128 ** -0.5, tile_lo=tl,
                                       pair_off=K.varlen_pair_offsets(tl, L), n_pairs=pair_count(seq))
        outs += [out, lse, *grads]
        # decode attention: one-token rows (split mode) and a 70-token chunk (tcgen05 prefill)
        B, page, P = 3, 128, 40
        kp = torch.randn(P, 8, page, 128, generator=g, device=dev).bfloat16()
        vp = torch.randn(P, 8, page, 128, generator=g, device=dev).bfloat16()
        bt = torch.arange(B * 12, device=dev, dtype=torch.int32).view(B, 12)
        kv_len = torch.tensor([1500, 700, 96], dtype=torch.int32, device=dev)
        for S in (1, 70):
            qd = torch.randn(B, S, 16, 128, generator=g, device=dev).bfloat16()
            q_pos = (kv_len[:, None] - S + torch.arange(S, device=dev, dtype=torch.int32)[None, :]).int()
            outs.append(K.decode_attention(qd, kp, vp, bt, q_pos.contiguous(), kv_len, 128 ** -0.5, 1500))
        # the QKV projection with the K2 epilogue
        x = torch.randn(200, 1024, generator=g, device=dev).bfloat16()
        w = (torch.randn(32 * 128, 1024, generator=g, device=dev) * 1024 ** -0.5).bfloat16()
        pos = torch.arange(200, dtype=torch.int32, device=dev)
        inv = (1e6 ** (-torch.arange(0, 128, 2, device=dev, dtype=torch.float32) / 128)).contiguous()
        outs.append(K.qkv_append(x, w, None, K.rope_table(pos, inv, 128), 16, 8, 128))
        # RMSNorm backward (its block count is cached per device)
        xr = torch.randn(512, 1024, generator=g, device=dev).bfloat16()
        wr = torch.randn(1024, generator=g, device=dev).bfloat16()
        y, rstd = K.rmsnorm_fwd(xr, wr, 1e-6)
        dy = torch.randn(y.shape, generator=g, device=dev).to(y.dtype)
        outs += list(K.rmsnorm_bwd(dy, xr, wr, rstd))
        torch.cuda.synchronize(dev)
    return [t.cpu() for t in outs]


def test_every_kernel_runs_on_a_second_device_of_the_process():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    from mouse_core_b200 import _lib, build

    build.build()
    a = _run_all(torch.device("cuda", 0))
    b = _run_all(torch.device("cuda", 1))
    for i, (x, y) in enumerate(zip(a, b)):
        assert torch.equal(x, y), f"output {i} differs between the devices"
    assert _lib.device_status() == 0
