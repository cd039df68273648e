"""GPU parity of the cached-decode path (K1 paged attention, K2 append, glue
kernels, the paged session) against the CPU oracle, which is itself pinned to
the reference by tests/test_oracle_golden.py.

Tolerances: kernels compute in bf16 with fp32 accumulation; attention and
append outputs must be within 2e-2 max-abs of the float64 oracle on the same
bf16 inputs. Whole-model hidden states carry the bf16 residual stream
(rounded to 2^-8 relative at every add), so they must be within atol 2e-2 +
rtol 1e-2 of the oracle on the golden fixtures and within 2e-2 x the row's
largest magnitude on the randomised schedules."""

from __future__ import annotations

import gc
import math
import weakref

import numpy as np
import pytest
import torch

from oracle import attention as oatt
from oracle import decoder as odec
from oracle import policy as opol
from tests.golden_io import decoder_from_fixture, load

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


def _paged_case(B, Hq, Hkv, hd, page, S, lens_after, n_new, seed):
    """Random q and per-row logical K/V scattered into a shuffled page pool."""
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, S, Hq, hd, generator=g).bfloat16()
    k_rows = [torch.randn(L, Hkv, hd, generator=g).bfloat16() for L in lens_after]
    v_rows = [torch.randn(L, Hkv, hd, generator=g).bfloat16() for L in lens_after]
    npg = [math.ceil(L / page) for L in lens_after]
    P = sum(npg) + 3
    perm = np.random.default_rng(seed).permutation(P).astype(np.int32)
    maxp = max(max(npg), 1)
    bt = np.full((B, maxp), -1, dtype=np.int32)
    kp = torch.zeros(P, Hkv, page, hd, dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    nxt = 0
    for b, L in enumerate(lens_after):
        for i in range(npg[b]):
            pg = int(perm[nxt])
            nxt += 1
            bt[b, i] = pg
            lo, hi = i * page, min(L, (i + 1) * page)
            kp[pg, :, : hi - lo] = k_rows[b][lo:hi].transpose(0, 1)
            vp[pg, :, : hi - lo] = v_rows[b][lo:hi].transpose(0, 1)
    lens_before = np.array(lens_after) - np.array(n_new)
    q_pos, _ = opol.decode_positions(lens_before, n_new, S)
    return q, kp, vp, bt, q_pos.astype(np.int32), k_rows, v_rows


CASES = [
    # B, Hq, Hkv, hd, page, S, seed
    (7, 16, 8, 128, 128, 1, 0),     # decode, split mode, G=2
    (5, 32, 8, 64, 64, 1, 1),       # G=4, hd 64, page 64
    (4, 32, 8, 64, 64, 4, 2),       # R = 16: largest split-mode row count
    (4, 32, 8, 64, 128, 5, 3),      # R = 20: block mode
    (3, 16, 8, 128, 128, 40, 4),    # ragged prefill chunk, 2 query blocks
    (3, 4, 4, 128, 64, 3, 5),       # no GQA sharing
    (2, 8, 2, 64, 64, 70, 6),       # G=4 prefill, 280 rows: tcgen05 prefill (S >= 64), partial tile
    (3, 16, 8, 128, 128, 256, 7),   # tcgen05 prefill: two query tiles per row over a cached history
    (2, 16, 8, 128, 64, 1024, 8),   # a 1024-token window (the rebuild prefill), 64-token pages
    (3, 4, 4, 128, 128, 130, 9),    # no GQA pairing (one q-head per CTA), a 2-row second tile
    (4, 32, 8, 64, 64, 96, 10),     # hd 64, G = 4
]


@pytest.mark.parametrize("B,Hq,Hkv,hd,page,S,seed", CASES)
def test_decode_attention_matches_oracle(B, Hq, Hkv, hd, page, S, seed):
    dev = _dev()
    from mouse_core_b200 import kernels as K

    rng = np.random.default_rng(100 + seed)
    n_new = rng.integers(0, S + 1, size=B)
    n_new[0] = S
    before = rng.integers(0, 1500, size=B)
    before[-1] = 0 if B > 2 else before[-1]          # an empty history
    if B > 3:
        before[1] = 512 - n_new[1]                     # a chunk boundary
        before[2] = 1024 + 1 - n_new[2]
    lens_after = (before + n_new).tolist()
    q, kp, vp, bt, q_pos, k_rows, v_rows = _paged_case(B, Hq, Hkv, hd, page, S, lens_after, n_new, seed)
    scale = hd ** -0.5
    out = K.decode_attention(q.to(dev), kp.to(dev), vp.to(dev), torch.from_numpy(bt).to(dev),
                             torch.from_numpy(q_pos).to(dev), torch.tensor(lens_after, dtype=torch.int32, device=dev),
                             scale, max(lens_after))
    torch.cuda.synchronize()
    ref = oatt.cached_decode_attention(q.float().numpy(), [k.float().numpy() for k in k_rows],
                                       [v.float().numpy() for v in v_rows], q_pos, scale)
    got = out.float().cpu().numpy()
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max()
    assert err < ATOL, f"max abs err {err}"
    if S >= 64:  # the tcgen05 prefill again, persistent over a tile counter in a workspace
        ws = torch.full((256,), 7, dtype=torch.uint8, device=dev)
        out2 = K.decode_attention(q.to(dev), kp.to(dev), vp.to(dev), torch.from_numpy(bt).to(dev),
                                  torch.from_numpy(q_pos).to(dev),
                                  torch.tensor(lens_after, dtype=torch.int32, device=dev), scale, max(lens_after),
                                  workspace=ws)
        assert np.abs(out2.float().cpu().numpy() - ref).max() < ATOL
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


def test_decode_attention_long_rows_split_combine():
    """Rows spanning many split chunks (the cross-CTA merge) at decode shape."""
    dev = _dev()
    from mouse_core_b200 import kernels as K

    B, Hq, Hkv, hd, page, S = 7, 16, 8, 128, 128, 1
    lens_after = [4096, 3001, 1, 5000, 2048, 777, 9000]
    n_new = [1] * B
    q, kp, vp, bt, q_pos, k_rows, v_rows = _paged_case(B, Hq, Hkv, hd, page, S, lens_after, n_new, 9)
    out = K.decode_attention(q.to(dev), kp.to(dev), vp.to(dev), torch.from_numpy(bt).to(dev),
                             torch.from_numpy(q_pos).to(dev), torch.tensor(lens_after, dtype=torch.int32, device=dev),
                             hd ** -0.5, max(lens_after))
    ref = oatt.cached_decode_attention(q.float().numpy(), [k.float().numpy() for k in k_rows],
                                       [v.float().numpy() for v in v_rows], q_pos, hd ** -0.5)
    assert np.abs(out.float().cpu().numpy() - ref).max() < ATOL


@pytest.mark.parametrize("hd,qk_norm", [(128, True), (64, False), (64, True)])
def test_kv_append_matches_oracle(hd, qk_norm):
    dev = _dev()
    from mouse_core_b200 import kernels as K

    T, Hq, Hkv, page, P = 37, 8, 2, 64, 9
    g = torch.Generator().manual_seed(hd)
    qkv = torch.randn(T, (Hq + 2 * Hkv) * hd + 8, generator=g).bfloat16()[:, : (Hq + 2 * Hkv) * hd]
    pos = torch.randint(0, 20000, (T,), generator=g, dtype=torch.int32)
    slots = torch.randperm(P * page, generator=g)[:T].to(torch.int32)
    slots[5] = -1  # a pad token: not cached
    qw = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16() if qk_norm else None
    kw = (1 + 0.3 * torch.randn(hd, generator=g)).bfloat16() if qk_norm else None
    theta = 1e6 if hd == 128 else 5e5
    inv_freq = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.float32) / hd))
    kp = torch.zeros(P, Hkv, page, hd, dtype=torch.bfloat16, device=dev)
    vp = torch.zeros_like(kp)
    qkv_d = torch.zeros(T, (Hq + 2 * Hkv) * hd + 8, dtype=torch.bfloat16, device=dev)
    qkv_d[:, : (Hq + 2 * Hkv) * hd] = qkv.to(dev)
    q_out = K.kv_append(qkv_d[:, : (Hq + 2 * Hkv) * hd], pos.to(dev), Hq, Hkv, hd, inv_freq.to(dev), 1.0,
                        None if qw is None else qw.to(dev), None if kw is None else kw.to(dev), 1e-6,
                        slot=slots.to(dev), k_pool=kp, v_pool=vp)
    x = qkv.float().numpy().astype(np.float64)
    qx = x[:, : Hq * hd].reshape(T, Hq, hd)
    kx = x[:, Hq * hd:(Hq + Hkv) * hd].reshape(T, Hkv, hd)
    vx = x[:, (Hq + Hkv) * hd:].reshape(T, Hkv, hd)
    if qk_norm:
        qx = odec.rms_norm(qx, qw.float().numpy(), 1e-6)
        kx = odec.rms_norm(kx, kw.float().numpy(), 1e-6)
    p = pos.numpy()
    qr = odec.rope(qx, p, inv_freq.numpy())
    kr = odec.rope(kx, p, inv_freq.numpy())
    assert np.abs(q_out.float().cpu().numpy() - qr).max() < ATOL
    kpc, vpc = kp.float().cpu().numpy(), vp.float().cpu().numpy()
    written = np.zeros((P, page), dtype=bool)
    for t in range(T):
        s = int(slots[t])
        if s < 0:
            continue
        pg, off = divmod(s, page)
        written[pg, off] = True
        assert np.abs(kpc[pg, :, off] - kr[t]).max() < ATOL
        assert np.abs(vpc[pg, :, off] - vx[t]).max() < 1e-2
    assert (kpc.transpose(0, 2, 1, 3)[~written] == 0).all(), "append wrote outside its slots"


def test_rmsnorm_and_silu_mul_match_fp32():
    dev = _dev()
    from mouse_core_b200 import kernels as K

    g = torch.Generator().manual_seed(0)
    x = torch.randn(33, 1024, generator=g).bfloat16().to(dev)
    r = torch.randn(33, 1024, generator=g).bfloat16().to(dev)
    w = (1 + 0.1 * torch.randn(1024, generator=g)).bfloat16().to(dev)
    s, n = K.rmsnorm(x, w, 1e-6, residual=r)
    s_ref = (x.float() + r.float()).bfloat16().float()
    assert torch.equal(s.float(), s_ref)
    n_ref = s_ref * torch.rsqrt(s_ref.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    assert (n.float() - n_ref).abs().max().item() < 3e-2
    gu = torch.randn(9, 2 * 3072, generator=g).bfloat16().to(dev)
    o = K.silu_mul(gu)
    ref = torch.nn.functional.silu(gu[:, :3072].float()) * gu[:, 3072:].float()
    assert (o.float() - ref).abs().max().item() < 3e-2


def _backbone_from_fixture(rec, arch, dev):
    from mouse_core_b200.backbone import LlamaBackbone, Qwen3Backbone

    if arch == "qwen3":
        bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    else:
        bb = LlamaBackbone(hidden_dim=128, num_layers=2, num_heads=2, num_key_value_heads=1)
    sd = {k[2:]: torch.from_numpy(v.astype(np.float32)) for k, v in rec.items() if k.startswith("w:")}
    missing, unexpected = bb.model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in m for m in missing)
    bb.model.rotary_emb.inv_freq.copy_(torch.from_numpy(rec["inv_freq"]))
    return bb.to(device=dev, dtype=torch.bfloat16).eval()


@pytest.mark.parametrize("arch", ["qwen3", "llama"])
def test_session_matches_reference_golden(arch):
    """Ragged schedule incl. empty first chunks, zero-length rows and a pool
    that must grow: real columns match the reference's FlexDecodeSession."""
    dev = _dev()
    rec = load(f"decode_{arch}.npz")
    bb = _backbone_from_fixture(rec, arch, dev)
    sess = bb.decode_session(batch_size=3, capacity=4, num_pages=1)  # must grow
    # The oracle with the same bf16-rounded weights and inputs isolates kernel error.
    rec16 = {k: (v.astype(np.float32) if k.startswith("w:") else v) for k, v in rec.items()}
    for k in list(rec16):
        if k.startswith("w:"):
            rec16[k] = torch.from_numpy(rec16[k]).bfloat16().float().numpy()
    dec16, _ = decoder_from_fixture(rec16)
    osess = odec.DecodeSessionOracle(dec16, 3)
    for ci, lens in enumerate(rec["schedule"].tolist()):
        emb = torch.from_numpy(rec[f"c{ci}_emb"])
        h, layers = sess.forward(embeds=emb.to(dev), lengths=lens, output_hidden_states=True)
        h = h.float().cpu().numpy()
        assert np.isfinite(h).all(), "NaN/inf leaked from padding"
        S = h.shape[1]
        ref = rec[f"c{ci}_out"]
        o16 = osess.forward(emb.bfloat16().float().numpy(), lens)
        for b, n in enumerate(lens):
            if n:
                np.testing.assert_allclose(h[b, S - n:], o16[b, S - n:], atol=ATOL, rtol=1e-2)
                np.testing.assert_allclose(h[b, S - n:], ref[b, S - n:], atol=5e-2, rtol=2e-2)
    assert sess.lengths.cpu().tolist() == rec["final_lengths"].tolist()
    assert sess.pages.num_pages >= 3, "the pool should have grown"


@pytest.mark.parametrize("fused_qkv", [False, True])  # cuBLAS QKV + K2, or K13 (the GEMM with K2 as epilogue)
def test_session_random_schedule_fuzz(fused_qkv):
    """Randomised ragged schedules on a Qwen3-shaped model (hd 128, GQA 2):
    every real step equals the oracle session, with either QKV projection."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(7)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    with torch.no_grad():
        for n_, p in bb.model.named_parameters():
            if "norm" in n_:
                p.copy_(1 + 0.2 * torch.randn_like(p))
            else:
                p.mul_(3.0)  # make attention non-trivial
        for p in bb.model.parameters():
            p.copy_(p.bfloat16().float())
    sd = {k: v.detach().numpy() for k, v in bb.model.state_dict().items() if "rotary" not in k}
    cfg = odec.config_from_hf(bb.model.config, bb.model.rotary_emb.inv_freq.numpy())
    dec = odec.DecoderOracle(sd, cfg)
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    rng = np.random.default_rng(3)
    B = 5
    sess = bb.decode_session(batch_size=B, capacity=16)
    sess.fused_qkv = fused_qkv
    osess = odec.DecodeSessionOracle(dec, B)
    for call in range(6):
        lens = rng.integers(0, 9, size=B)
        if call == 0:
            lens[1] = 300  # a long prefill row: block mode for S > 8
        S = max(int(lens.max()), 1)
        emb = torch.randn(B, S, 256).bfloat16()
        h = sess.forward(embeds=emb.to(dev), lengths=lens.tolist()).float().cpu().numpy()
        o = osess.forward(emb.float().numpy(), lens)
        for b, n in enumerate(lens):
            if n:
                # bf16 residual stream: error bound scales with the row's magnitude
                scale = max(1.0, float(np.abs(o[b, S - n:]).max()))
                assert np.abs(h[b, S - n:] - o[b, S - n:]).max() <= ATOL * scale, (call, b)


def test_session_freed_by_refcount_alone():
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    bb = Qwen3Backbone(hidden_dim=128, num_layers=1, num_heads=2, num_key_value_heads=1, head_dim=64)
    bb = bb.to(device=dev, dtype=torch.bfloat16)
    sess = bb.decode_session(batch_size=2, capacity=64)
    sess.forward(embeds=torch.randn(2, 3, 128, device=dev), lengths=[3, 1])
    wr = weakref.ref(sess)
    gc.disable()
    try:
        del sess
        assert wr() is None, "session stayed alive without cyclic GC"
    finally:
        gc.enable()


def test_session_rejects_bad_inputs():
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    bb = Qwen3Backbone(hidden_dim=128, num_layers=1, num_heads=2, num_key_value_heads=1, head_dim=64)
    with pytest.raises(TypeError):
        bb.to(dev).decode_session(batch_size=2, capacity=8)  # fp32 model
    bb = bb.to(device=dev, dtype=torch.bfloat16)
    sess = bb.decode_session(batch_size=2, capacity=8)
    with pytest.raises(ValueError, match="batch_size"):
        sess.forward(embeds=torch.randn(3, 1, 128, device=dev), lengths=[1, 1, 1])
    with pytest.raises(ValueError):
        sess.forward(embeds=torch.randn(2, 1, 128, device=dev), lengths=[2, 1])


def test_session_graph_replay_matches_eager():
    """Single-token steps replay a captured CUDA graph; they must equal the
    eager path step for step, across page boundaries and a block-table
    widening (which forces a re-capture)."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(9)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    B = 4
    graph_sess = bb.decode_session(batch_size=B, capacity=64, page_size=64)
    eager_sess = bb.decode_session(batch_size=B, capacity=64, page_size=64)
    eager_sess.use_graphs = False
    g = torch.Generator().manual_seed(4)
    pre = torch.randn(B, 60, 256, generator=g).bfloat16().to(dev)
    lens = [60, 3, 0, 59]
    a = graph_sess.forward(embeds=pre, lengths=lens)
    b = eager_sess.forward(embeds=pre, lengths=lens)
    assert torch.equal(a, b)
    for step in range(80):  # crosses the 64-token page and widens the table past 64 slots
        x = torch.randn(B, 1, 256, generator=g).bfloat16().to(dev)
        a = graph_sess.forward(embeds=x, lengths=[1] * B)
        b = eager_sess.forward(embeds=x, lengths=[1] * B)
        assert (a.float() - b.float()).abs().max().item() <= 1e-3, step
    assert graph_sess._graph is not None
    assert graph_sess.lengths.tolist() == eager_sess.lengths.tolist()


@pytest.mark.parametrize("hd,page,Hq,Hkv", [(128, 128, 16, 8), (64, 64, 32, 16), (128, 64, 16, 8)])
def test_shared_chunk_plan_matches_plain_plan(hd, page, Hq, Hkv):
    """One-token decode over rows that hold forked prefixes on the same pages:
    the plan that gives a shared 2048-token chunk one work item for a block of
    rows (mb_decode_plan_shared) matches the plan that reads the chunk once
    per row (mb_decode_plan) — bit for bit on every row that holds whole
    chunks only, within one bf16 rounding where a row's chunk is split into a
    shared head and its own tail (two partials instead of one) — and both
    match the oracle. Rows: a root's branches filling an aligned block and spilling into
    the next one, a second group that does not start a block, lone rows, a
    branch forked inside a chunk, and rows shorter than one chunk."""
    dev = _dev()
    from mouse_core_b200 import kernels as K

    G = Hq // Hkv
    NG = 16 // G
    rng = np.random.default_rng(hd + page)
    gen = torch.Generator().manual_seed(hd + page)
    chunk = 2048
    ppc = chunk // page
    # Per row: (root id or None, pages shared with that root). Root 0's
    # branches fill the first aligned block and spill into the next one;
    # root 1's branches sit after the second block's start, behind rows of
    # root 0; in the third block two short rows come first and root 2's
    # branches alternate with lone rows (a member mask with gaps), one of
    # them forked inside its second chunk (it shares that chunk's head and
    # has the rest as a tail item); one of root 1's branches forks inside
    # its second chunk too.
    layout = [(0, 3 * ppc)] * (NG + 2) + [(None, 0), (1, 2 * ppc), (1, 2 * ppc), (1, ppc + ppc // 2)]
    layout += [(None, 0)] * (2 * NG - len(layout))
    layout += [("short", 0), ("short", 0)] + [(2, 2 * ppc), (None, 0)] * 2 + [(2, ppc + ppc // 2), (None, 0)]
    layout += [(2, 2 * ppc)]
    B = len(layout)
    lens = []
    for root, ns in layout:
        if root == "short":
            lens.append(int(rng.integers(1, chunk)))
        elif root is None:
            lens.append(int(rng.integers(1, 3 * chunk)))
        else:
            lens.append(ns * page + int(rng.integers(1, 3 * page)))
    npg = [math.ceil(L / page) for L in lens]
    maxp = max(npg)
    bt = np.full((B, maxp), -1, dtype=np.int32)
    nxt = 0
    root_pages = {}
    for r, (root, ns) in enumerate(layout):
        start = 0
        if isinstance(root, int):
            if root not in root_pages:
                root_pages[root] = list(range(nxt, nxt + 3 * ppc))
                nxt += 3 * ppc
            bt[r, :ns] = root_pages[root][:ns]
            start = ns
        for i in range(start, npg[r]):
            bt[r, i] = nxt
            nxt += 1
    P = nxt + 1
    kp = torch.randn(P, Hkv, page, hd, generator=gen).bfloat16()
    vp = torch.randn(P, Hkv, page, hd, generator=gen).bfloat16()
    q = torch.randn(B, 1, Hq, hd, generator=gen).bfloat16()
    kv_len = torch.tensor(lens, dtype=torch.int32)
    q_pos = (kv_len - 1).view(B, 1).to(torch.int32)
    d = lambda t: t.to(dev)  # noqa: E731
    kp_d, vp_d, bt_d, q_d, kvl_d, qp_d = map(d, (kp, vp, torch.from_numpy(bt), q, kv_len, q_pos))
    scale = hd ** -0.5
    cap = max(lens)
    ws = torch.empty(K.decode_workspace_bytes(B, Hkv, G, hd, cap), dtype=torch.uint8, device=dev)
    K.decode_plan(kvl_d, Hkv, G, hd, cap, ws)
    plain = K.decode_attention(q_d, kp_d, vp_d, bt_d, qp_d, kvl_d, scale, cap, workspace=ws, plan_ready=True)
    K.decode_plan(kvl_d, Hkv, G, hd, cap, ws, block_table=bt_d, page_size=page)
    shared = K.decode_attention(q_d, kp_d, vp_d, bt_d, qp_d, kvl_d, scale, cap, workspace=ws, plan_ready=True)
    torch.cuda.synchronize()
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0
    split_rows = [r for r, (root, ns) in enumerate(layout) if isinstance(root, int) and ns % ppc]
    whole = [r for r in range(B) if r not in split_rows]
    assert torch.equal(plain[whole], shared[whole])
    d = (plain.float() - shared.float()).abs()
    assert float(d.max()) <= 2 ** -8 * max(1.0, float(plain.float().abs().max())), float(d.max())
    # Oracle on every row (float64, same bf16 inputs).
    k_rows = [torch.cat([kp[bt[b, i]].transpose(0, 1) for i in range(npg[b])])[:lens[b]].float().numpy()
              for b in range(B)]
    v_rows = [torch.cat([vp[bt[b, i]].transpose(0, 1) for i in range(npg[b])])[:lens[b]].float().numpy()
              for b in range(B)]
    ref = oatt.cached_decode_attention(q.float().numpy(), k_rows, v_rows, q_pos.numpy(), scale)
    err = np.abs(shared.float().cpu().numpy() - ref).max()
    assert err < ATOL, f"max abs err {err}"


def test_fork_shares_prefix_pages_and_matches_independent_rows():
    """Branches forked at arbitrary points share the root's full pages, copy
    only the partial last page, and decode exactly like rows that computed
    the same prefix themselves."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(3)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    page, R, G = 64, 2, 3          # 2 roots, 3 branches each
    B = R + R * G
    g = torch.Generator().manual_seed(8)
    root_len = [200, 131]
    ctx = [torch.randn(L, 256, generator=g).bfloat16() for L in root_len]
    forks = [[200, 64, 1], [131, 128, 70]]  # fork points (full-page, page-aligned, partial cases)

    shared = bb.decode_session(batch_size=B, capacity=256, page_size=page)
    S = max(root_len)
    emb = torch.zeros(B, S, 256, dtype=torch.bfloat16)
    for r in range(R):
        emb[r, S - root_len[r]:] = ctx[r]
    shared.forward(embeds=emb.to(dev), lengths=root_len + [0] * (R * G))
    free_before = shared.pages.free_pages
    src, dst, plen = [], [], []
    for r in range(R):
        for j in range(G):
            src.append(r)
            dst.append(R + r * G + j)
            plen.append(forks[r][j])
    shared.fork(src, dst, plen)
    n_partial = sum(1 for p_ in plen if p_ % page)
    assert shared.pages.free_pages == free_before - n_partial  # only partial pages were copied
    assert shared.lengths.cpu().tolist()[R:] == plen

    # Independent reference: every branch row prefills its own prefix.
    indep = bb.decode_session(batch_size=B, capacity=256, page_size=page)
    emb2 = torch.zeros(B, S, 256, dtype=torch.bfloat16)
    lens2 = list(root_len) + plen
    for r in range(R):
        emb2[r, S - root_len[r]:] = ctx[r]
    for i, (s_, p_) in enumerate(zip(src, plen)):
        if p_:
            emb2[R + i, S - p_:] = ctx[s_][:p_]
    indep.forward(embeds=emb2.to(dev), lengths=lens2)

    for step in range(5):
        x = torch.randn(B, 1, 256, generator=g).bfloat16().to(dev)
        a = shared.forward(embeds=x, lengths=[1] * B)
        b = indep.forward(embeds=x, lengths=[1] * B)
        assert (a.float() - b.float()).abs().max().item() <= 2e-2, step
    # Releasing the branches returns their private pages; shared pages stay with the roots.
    shared.reset_rows(dst)
    assert shared.pages.npages[:R].tolist() == [int(np.ceil((L + 5) / page)) for L in root_len]


def test_device_step_matches_host_step():
    """Steps of at most one token per row whose positions, slots and lengths
    the device derives (K8) equal the host-prepared steps bit for bit, across
    page openings, a pool growth, a block-table widening, rows sitting out,
    rows emptied between steps (restarted by the device step, sitting out,
    or re-sent by a multi-token chunk), a fork and multi-token chunks; the
    page tables agree on host and device wherever a row holds pages."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(11)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    B, page = 6, 64
    fast = bb.decode_session(batch_size=B, capacity=64, page_size=page, num_pages=8)
    host = bb.decode_session(batch_size=B, capacity=64, page_size=page, num_pages=8)
    host.use_device_step = False
    taken = [0]
    inner = fast._device_step

    def counted(n):
        ok = inner(n)
        taken[0] += ok
        return ok

    fast._device_step = counted
    g = torch.Generator().manual_seed(5)
    rng = np.random.default_rng(2)

    def both(S, lens):
        x = torch.randn(B, S, 256, generator=g).bfloat16().to(dev)
        a = fast.forward(embeds=x, lengths=lens)
        b = host.forward(embeds=x, lengths=lens)
        assert torch.equal(a, b), (S, lens)
        assert fast._len.tolist() == host._len.tolist()
        assert np.array_equal(fast.pages.table, host.pages.table)
        w = fast.pages.max_pages
        held = np.arange(w)[None, :] < fast.pages.npages[:, None]  # emptied rows keep stale device entries
        assert np.array_equal(fast._bt_dev[:, :w].cpu().numpy()[held], fast.pages.table[held])

    both(60, rng.integers(1, 61, size=B).tolist())
    for step in range(160):
        if step == 30:  # emptied, then refilled by a multi-token chunk (host path re-sends the table)
            fast.reset_rows([1, 3])
            host.reset_rows([1, 3])
            both(9, [0, 9, 0, 4, 0, 0])
        elif step == 60:
            fast.fork([0, 2], [4, 5], [17, 64])
            host.fork([0, 2], [4, 5], [17, 64])
        elif step == 100:
            both(1, [1, 0, 1, 1, 0, 1])  # rows sitting out
        elif step in (110, 130):  # emptied between steps: the device step restarts them
            fast.reset_rows([2, 5])
            host.reset_rows([2, 5])
        elif step == 120:  # one emptied row sits out its first step, the other restarts
            fast.reset_rows([0, 4])
            host.reset_rows([0, 4])
            both(1, [0, 1, 1, 1, 1, 1])
        both(1, [1] * B)
    assert taken[0] >= 145, taken[0]
    assert fast.pages.num_pages > 8 and fast.pages.max_pages > 2  # grew and widened on the way


def test_decode_step_meta_reports_rows_past_the_table():
    """K8 on a row whose next token would land past the block table's width
    records kDevBadPage and writes no table entry; other rows step normally."""
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200 import kernels as K

    page, width = 64, 2
    bt = torch.tensor([[5, 6], [7, -1], [8, 9]], dtype=torch.int32, device=dev)
    kv_len = torch.tensor([70, 64, 128], dtype=torch.int32, device=dev)  # row 2 is full
    new_page = torch.tensor([-1, 11, 12], dtype=torch.int32, device=dev)
    q_pos, slot = torch.empty_like(kv_len), torch.empty_like(kv_len)
    _lib.device_status()  # clear
    K.decode_step_meta(bt, q_pos, kv_len, slot, page, new_page)
    assert _lib.device_status() == 3  # kDevBadPage
    assert bt.cpu().tolist() == [[5, 6], [7, 11], [8, 9]]
    assert q_pos.cpu().tolist() == [70, 64, 128]
    assert slot.cpu().tolist() == [6 * page + 6, 11 * page + 0, -1]
    assert kv_len.cpu().tolist() == [71, 65, 129]


def test_decode_step_graph_matches_forward_and_head():
    """decode_step runs the embedding gather, the layer stack, the final norm
    and the caller's head as one CUDA graph; step for step it must give what
    forward + the head give, across page openings, rows sitting out, rows
    emptied between steps (K8 restarts) and a multi-token chunk between."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(13)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    B, page, V = 5, 64, 50
    g = torch.Generator().manual_seed(1)
    table = torch.randn(V, 256, generator=g).bfloat16().to(dev)
    w = (torch.randn(4, 256, generator=g) / 16).to(dev)

    def embed(ids):
        return table[ids]

    def head(h):
        # forward() hands back the model dtype; decode_step gives the head the
        # fp32 residual stream, so round it the same way before comparing.
        return torch.nn.functional.linear(torch.nn.functional.rms_norm(h.bfloat16().float(), (256,), None, 1e-5), w)

    fast = bb.decode_session(batch_size=B, capacity=64, page_size=page)
    ref = bb.decode_session(batch_size=B, capacity=64, page_size=page)
    ref.use_graphs = False
    rng = np.random.default_rng(3)
    pre = rng.integers(0, V, size=(B, 40))
    lens = [40, 7, 0, 33, 12]
    x = table[torch.from_numpy(pre).to(dev)]
    fast.forward(embeds=x, lengths=lens)
    ref.forward(embeds=x, lengths=lens)
    replays = 0
    for step in range(90):
        if step in (20, 50):
            fast.reset_rows([1, 4])
            ref.reset_rows([1, 4])
        if step == 35:  # a multi-token chunk: the host path, then graph steps again
            ids2 = torch.from_numpy(rng.integers(0, V, size=(B, 3))).to(dev)
            a = fast.forward(embeds=table[ids2], lengths=[3, 0, 2, 1, 3])
            b = ref.forward(embeds=table[ids2], lengths=[3, 0, 2, 1, 3])
            assert (a.float() - b.float()).abs().max().item() <= 1e-2
        ids = torch.from_numpy(rng.integers(0, V, size=B)).to(dev)
        n = [1] * B if step % 7 else [1, 0, 1, 1, 0]
        before = fast._step_graph
        out = fast.decode_step(ids, n, embed, head).clone()
        replays += before is not None and fast._step_graph is before
        h = ref.forward(embeds=table[ids].view(B, 1, 256), lengths=n)
        want = head(h[:, -1])
        live = torch.tensor(n, device=dev).bool()
        err = (out[live] - want[live]).abs().max().item()
        assert err <= 1e-3 * max(1.0, want.abs().max().item()), (step, err)
        assert fast._len.tolist() == ref._len.tolist()
    assert replays >= 70, replays
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


def test_fp32_residual_glue_kernels():
    """The fp32 residual-stream glue: the add stays exact in fp32, the norm
    and SiLU product are rounded once to bf16, and K2 reading an fp32 QKV
    projection matches K2 reading its bf16 rounding within bf16 precision."""
    dev = _dev()
    from mouse_core_b200 import kernels as K

    g = torch.Generator().manual_seed(3)
    x = torch.randn(33, 1024, generator=g).to(dev)
    d = torch.randn(33, 1024, generator=g).to(dev)
    w = (1 + 0.1 * torch.randn(1024, generator=g)).bfloat16().to(dev)
    s, n = K.rmsnorm_f32(x, w, 1e-6, delta=d)
    assert s.dtype == torch.float32 and n.dtype == torch.bfloat16
    assert torch.equal(s, x + d)
    want = (s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float())
    assert (n.float() - want).abs().max().item() <= 1e-2 * want.abs().max().item()
    xb = torch.randn(5, 1024, generator=g).bfloat16().to(dev)  # the embeddings entering layer 0
    s0, n0 = K.rmsnorm_f32(xb, w, 1e-6)
    assert torch.equal(s0, xb.float())
    x2 = x.clone()
    s2, _ = K.rmsnorm_f32(x2, w, 1e-6, delta=d, sum_out=x2)  # in place
    assert s2.data_ptr() == x2.data_ptr() and torch.equal(x2, x + d)
    gu = torch.randn(9, 2 * 3072, generator=g).to(dev)
    o = K.silu_mul_f32(gu)
    ref = torch.nn.functional.silu(gu[:, :3072]) * gu[:, 3072:]
    assert bool(((o.float() - ref).abs() <= ref.abs() * 2.0 ** -8 + 1e-30).all())  # one bf16 rounding
    # K2 on an fp32 qkv vs on the same values in bf16: both round once at the output.
    Hq, Hkv, hd = 16, 8, 128
    qkv = torch.randn(7, (Hq + 2 * Hkv) * hd, generator=g).to(dev)
    qkv16 = qkv.bfloat16().float()
    pos = torch.arange(7, dtype=torch.int32, device=dev) * 37
    inv = (1e6 ** (-torch.arange(0, hd, 2, dtype=torch.float32) / hd)).to(dev)
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16().to(dev)
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).bfloat16().to(dev)
    ko, vo = (torch.empty(7, Hkv, hd, dtype=torch.bfloat16, device=dev) for _ in range(2))
    ko16, vo16 = (torch.empty_like(ko) for _ in range(2))
    q32 = K.kv_append(qkv16, pos, Hq, Hkv, hd, inv, 1.0, qw, kw, 1e-6, k_out=ko, v_out=vo)
    q16 = K.kv_append(qkv16.bfloat16(), pos, Hq, Hkv, hd, inv, 1.0, qw, kw, 1e-6, k_out=ko16, v_out=vo16)
    assert torch.equal(q32, q16) and torch.equal(ko, ko16) and torch.equal(vo, vo16)
