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


def _run_bwd(seq, q, k, v, do, dev, stored=False):
    """K6 gradients; ``stored`` takes the path whose dQ is one GEMM over the
    dS blocks the dK/dV kernel stores (pair count from the host ids, checked
    against the device offsets)."""
    from mouse_core_b200 import kernels as K
    from mouse_core_b200.packed import pair_count

    st = torch.from_numpy(seq).to(dev)
    _, rs, tl, flags, re = K.segment_meta(st, tile=128, with_run_end=True)
    qd, kd, vd, dod = q.to(dev), k.to(dev), v.to(dev), do.to(dev)
    scale = q.shape[-1] ** -0.5
    out, lse = K.varlen_attention_fwd(qd, kd, vd, rs, tl, scale)
    extra = {}
    if stored:
        pair_off = K.varlen_pair_offsets(tl, seq.shape[0])
        n_pairs = pair_count(seq)
        T = (seq.shape[0] + 127) // 128
        per_tile = np.arange(T) - tl.cpu().numpy() // 128 + 1
        assert np.array_equal(pair_off.cpu().numpy(), np.concatenate([[0], np.cumsum(per_tile)]))
        assert int(pair_off[-1].item()) == n_pairs
        extra = dict(tile_lo=tl, pair_off=pair_off, n_pairs=n_pairs)
    dq, dk, dv = K.varlen_attention_bwd(qd, kd, vd, out, dod, lse, rs, re, scale, **extra)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (dq, dk, dv)]


BWD_CASES = FWD_CASES + [("g2_hd128_many", 4, 2, 128, [5, 300, 1, 1, 1, 64, 129, 600])]


@pytest.mark.parametrize("stored", [False, True])
@pytest.mark.parametrize("name,Hq,Hkv,hd,lens", BWD_CASES)
def test_varlen_bwd_matches_oracle(name, Hq, Hkv, hd, lens, stored):
    """dq, dk, dv (bf16, fp32 accumulation) vs the float64 analytic gradient on
    the same bf16 inputs: max-abs error within 2e-2 of each gradient's scale
    (its largest magnitude, at least 1); both dQ paths."""
    dev = _dev()
    seq = _seq_from_lengths(lens)
    L = seq.shape[0]
    q, k, v, do = cfg1_inputs(13, L, Hq, Hkv, hd)
    q, k, v, do = q.bfloat16(), k.bfloat16(), v.bfloat16(), do.bfloat16()
    got = _run_bwd(seq, q, k, v, do, dev, stored)
    ref = oatt.packed_attention_bwd(q.float().numpy(), k.float().numpy(), v.float().numpy(), seq, hd ** -0.5,
                                    do.float().numpy())
    for gname, g, r in zip(("dq", "dk", "dv"), got, ref):
        assert np.isfinite(g).all(), gname
        scale = max(1.0, float(np.abs(r).max()))
        err = np.abs(g - r).max()
        assert err <= ATOL * scale, f"{name} {gname}: max abs err {err} (scale {scale})"
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


@pytest.mark.parametrize("stored", [False, True])
def test_varlen_bwd_packed_2048_against_reference_samples(stored):
    """Gradients of the 2048-token packed workload vs the reference's fp32
    SDPA-mask autograd (sampled entries); both dQ paths."""
    dev = _dev()
    g = load("packed_attn_cfg1.npz")
    seq = _seq_from_lengths(cfg1_segments(0))
    q, k, v, do = cfg1_inputs(0, 2048, 4, 2, 64)
    got = _run_bwd(seq, q.bfloat16(), k.bfloat16(), v.bfloat16(), do.bfloat16(), dev, stored)
    for gname, arr in zip(("dq", "dk", "dv"), got):
        ref = g[f"{gname}_val"]
        scale = max(1.0, float(np.abs(ref).max()))
        err = np.abs(arr.reshape(-1)[g[f"{gname}_idx"]] - ref).max()
        assert err <= ATOL * scale, f"{gname}: max abs err vs reference samples {err}"


# ---------------------------------------------------------------- flex_packed_forward


def _qwen3_fixture_model(rec, dev):
    from mouse_core_b200.backbone import Qwen3Backbone

    bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    sd = {k[2:]: torch.from_numpy(v.astype(np.float32)) for k, v in rec.items() if k.startswith("w:")}
    bb.model.load_state_dict(sd, strict=False)
    bb.model.rotary_emb.inv_freq.copy_(torch.from_numpy(rec["inv_freq"]))
    return bb.to(device=dev, dtype=torch.bfloat16)


def test_flex_packed_forward_matches_reference_golden():
    dev = _dev()
    from mouse_core_b200 import flex_packed_forward
    from oracle import decoder as odec
    from tests.golden_io import decoder_from_fixture

    rec = dict(load("packed_fwd_qwen3.npz"))
    bb = _qwen3_fixture_model(rec, dev)
    emb = torch.from_numpy(rec["emb"])
    seq = torch.from_numpy(rec["seq"])
    with torch.no_grad():
        h, layers = flex_packed_forward(model=bb.model, embeds=emb.to(dev), sequence_ids=seq.to(dev),
                                        output_hidden_states=True)
    h = h.float().cpu().numpy()
    assert h.shape == rec["out"].shape and len(layers) == 2
    rec16 = dict(rec)
    for key in list(rec16):
        if key.startswith("w:"):
            rec16[key] = torch.from_numpy(rec16[key].astype(np.float32)).bfloat16().float().numpy()
    rec16.update(num_layers=np.array(2), n_heads=np.array(2), n_kv_heads=np.array(1), head_dim=np.array(64),
                 qk_norm=np.array(True))
    dec16, _ = decoder_from_fixture(rec16)
    o16 = odec.packed_forward(dec16, emb.bfloat16().float().numpy(), rec["seq"])
    np.testing.assert_allclose(h, o16, atol=ATOL, rtol=1e-2)
    np.testing.assert_allclose(h, rec["out"], atol=5e-2, rtol=2e-2)


def _train_model(dev, hd, seed=0):
    from mouse_core_b200.backbone import Qwen3Backbone

    torch.manual_seed(seed)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=hd)
    with torch.no_grad():
        for name, prm in bb.model.named_parameters():
            if "norm" not in name:
                prm.mul_(4.0)  # non-trivial attention at init
            prm.copy_(prm.bfloat16().float())
    return bb


@pytest.mark.parametrize("hd,ids", [(64, "sorted"), (128, "sorted"), (64, "unsorted")])
def test_flex_packed_gradients_match_fp32_torch(hd, ids):
    """Loss gradients w.r.t. embeds and weights: bf16 tcgen05 path vs the
    reference's dense-mask SDPA path run in fp32 (plain PyTorch) on the GPU."""
    dev = _dev()
    import copy

    from mouse_core_b200 import flex_packed_forward
    from mouse_core_b200.packing import flat_sequence_causal_mask, flat_sequence_position_ids

    bb = _train_model(dev, hd)
    ref_bb = copy.deepcopy(bb).to(device=dev, dtype=torch.float32)
    ours = bb.to(device=dev, dtype=torch.bfloat16)
    if ids == "sorted":
        seq = torch.from_numpy(_seq_from_lengths([100, 1, 300, 17, 200]))
    else:
        seq = torch.tensor(([0] * 40 + [1] * 25 + [0] * 60 + [2] * 90 + [1] * 30) * 2, dtype=torch.long)
    L = seq.shape[0]
    g = torch.Generator().manual_seed(1)
    emb = torch.randn(L, 256, generator=g).bfloat16().float()
    w = torch.randn(L, 256, generator=g)

    e1 = emb.to(dev).requires_grad_(True)
    h1 = flex_packed_forward(model=ours.model, embeds=e1, sequence_ids=seq.to(dev))
    (h1.float() * w.to(dev)).sum().backward()

    e2 = emb.to(dev).requires_grad_(True)
    sd = seq.to(dev)
    mask = flat_sequence_causal_mask(sequence_ids=sd, dtype=torch.float32)
    pos = flat_sequence_position_ids(sd)
    h2 = ref_bb(e2[None], attention_mask=mask, position_ids=pos)[0]
    (h2 * w.to(dev)).sum().backward()

    def rel(a, b):
        return float((a.detach().float() - b.detach().float()).norm() / (b.detach().float().norm() + 1e-12))

    assert rel(h1, h2) < 2e-2
    assert rel(e1.grad, e2.grad) < 3e-2
    p1 = dict(ours.model.named_parameters())
    for name, p2 in ref_bb.model.named_parameters():
        if p2.grad is None:
            continue
        assert rel(p1[name].grad, p2.grad) < 3e-2, name


def test_flex_packed_forward_isolates_sequences():
    """Changing one segment's embeddings leaves every other segment's outputs
    bitwise unchanged (segments never attend across ids)."""
    dev = _dev()
    from mouse_core_b200 import flex_packed_forward

    bb = _train_model(dev, 128).to(device=dev, dtype=torch.bfloat16)
    seq = torch.from_numpy(_seq_from_lengths([130, 70, 260])).to(dev)
    g = torch.Generator().manual_seed(2)
    emb = torch.randn(460, 256, generator=g).to(dev)
    emb2 = emb.clone()
    emb2[130:200] = torch.randn(70, 256, generator=g).to(dev)
    with torch.no_grad():
        a = flex_packed_forward(model=bb.model, embeds=emb, sequence_ids=seq)
        b = flex_packed_forward(model=bb.model, embeds=emb2, sequence_ids=seq)
    assert torch.equal(a[:130], b[:130]) and torch.equal(a[200:], b[200:])
    assert not torch.equal(a[130:200], b[130:200])


def test_flex_packed_forward_rejects_bad_shapes():
    dev = _dev()
    from mouse_core_b200 import flex_packed_forward

    bb = _train_model(dev, 64).to(device=dev, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=r"\[L, D\]"):
        flex_packed_forward(model=bb.model, embeds=torch.zeros(1, 4, 256, device=dev),
                            sequence_ids=torch.zeros(4, dtype=torch.long, device=dev))
    with pytest.raises(ValueError, match="sequence_ids"):
        flex_packed_forward(model=bb.model, embeds=torch.zeros(4, 256, device=dev),
                            sequence_ids=torch.zeros(3, dtype=torch.long, device=dev))


def test_flex_packed_llama3_rope_gradients_match_fp32_torch():
    """Llama stack (no q/k norm; Llama-3 frequency-scaled RoPE through the
    model's own rotary_emb): the fused training layer's output and gradients
    vs the dense-mask SDPA path in fp32, within 3e-2 or 1.5x the error of the
    stock modules run in bf16 on the same dense path (without the q/k norm the
    attention logits are unbounded and bf16 rounding alone moves the result)."""
    dev = _dev()
    import copy

    from mouse_core_b200 import flex_packed_forward
    from mouse_core_b200.backbone import LlamaBackbone
    from mouse_core_b200.packing import flat_sequence_causal_mask, flat_sequence_position_ids

    torch.manual_seed(4)
    bb = LlamaBackbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2,
                       rope_parameters={"rope_type": "llama3", "rope_theta": 500000.0, "factor": 8.0,
                                        "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                        "original_max_position_embeddings": 256})
    with torch.no_grad():
        for name, prm in bb.model.named_parameters():
            if "norm" not in name:
                prm.mul_(2.0)
            prm.copy_(prm.bfloat16().float())
    ref_bb = copy.deepcopy(bb).to(device=dev, dtype=torch.float32)
    stock16 = copy.deepcopy(bb).to(device=dev, dtype=torch.bfloat16)
    ours = bb.to(device=dev, dtype=torch.bfloat16)
    seq = torch.from_numpy(_seq_from_lengths([700, 33, 290]))
    L = seq.shape[0]
    g = torch.Generator().manual_seed(5)
    emb = torch.randn(L, 256, generator=g).bfloat16().float()
    w = torch.randn(L, 256, generator=g)

    e1 = emb.to(dev).requires_grad_(True)
    h1 = flex_packed_forward(model=ours.model, embeds=e1, sequence_ids=seq.to(dev))
    (h1.float() * w.to(dev)).sum().backward()
    e2 = emb.to(dev).requires_grad_(True)
    sd = seq.to(dev)
    pos = flat_sequence_position_ids(sd)
    h2 = ref_bb(e2[None], attention_mask=flat_sequence_causal_mask(sequence_ids=sd, dtype=torch.float32),
                position_ids=pos)[0]
    (h2 * w.to(dev)).sum().backward()
    e3 = emb.to(dev).bfloat16().requires_grad_(True)
    h3 = stock16(e3[None], attention_mask=flat_sequence_causal_mask(sequence_ids=sd, dtype=torch.bfloat16),
                 position_ids=pos)[0]
    (h3.float() * w.to(dev)).sum().backward()

    def rel(a, b):
        return float((a.detach().float() - b.detach().float()).norm() / (b.detach().float().norm() + 1e-12))

    def bound(stock_err):
        return max(3e-2, 1.5 * stock_err)

    assert rel(h1, h2) < bound(rel(h3, h2))
    assert rel(e1.grad, e2.grad) < bound(rel(e3.grad, e2.grad))
    p1 = dict(ours.model.named_parameters())
    p3 = dict(stock16.model.named_parameters())
    for name, p2 in ref_bb.model.named_parameters():
        if p2.grad is not None:
            assert rel(p1[name].grad, p2.grad) < bound(rel(p3[name].grad, p2.grad)), name
