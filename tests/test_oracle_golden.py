"""Pin the CPU oracle against fixtures produced by the reference itself and
against the known-answer vectors of the reference's own tests
(tests/test_kv_policy.py, test_segment_attention.py, test_packing.py,
test_flex_packed_correctness.py in micahr234/mouse-core)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import attention as oatt
from oracle import decoder as odec
from oracle import policy as opol
from tests.golden_io import cfg1_inputs, cfg1_segments, decoder_from_fixture, load


# -- known answers quoted from the reference's tests ------------------------

def test_known_answers_kv_policy():
    assert opol.resolve_cache_bounds(512, None) == (512, 256)
    assert opol.resolve_cache_bounds(512, 512) == (512, 511)
    got = opol.rebuild_starts(context_start=0, start_cache=256, max_cache=512, ends=np.array([600, 600]))
    assert got.tolist() == [344, 344]
    got = opol.rebuild_starts(context_start=80, start_cache=256, max_cache=512, ends=np.array([100]))
    assert got.tolist() == [80]
    assert opol.cache_needs_rebuild(has_cache=True, cached_starts=np.array([0]), cached_ends=np.array([512]),
                                    ends=np.array([513]), context_start=np.array([0]), max_cache=512,
                                    batch_complete=True)
    assert not opol.cache_needs_rebuild(has_cache=True, cached_starts=np.array([100]),
                                        cached_ends=np.array([356]), ends=np.array([357]),
                                        context_start=np.array([0]), max_cache=512, batch_complete=True)
    assert opol.cache_needs_rebuild(has_cache=True, cached_starts=np.array([0]), cached_ends=np.array([10]),
                                    ends=np.array([20]), context_start=np.array([15]), max_cache=512,
                                    batch_complete=True)


def test_known_answers_positions_and_mask():
    assert opol.position_ids(np.array([0, 0, 0, 1, 1, 2])).tolist() == [0, 1, 2, 0, 1, 0]
    allow = opol.segment_causal_allow(np.array([0, 0, 1, 1]))
    expect = np.array([[1, 0, 0, 0], [1, 1, 0, 0], [0, 0, 1, 0], [0, 0, 1, 1]], dtype=bool)
    assert (allow == expect).all()


def test_known_answer_left_align():
    emb = np.zeros((1, 5, 2), dtype=np.float32)
    emb[0, 0], emb[0, 1], emb[0, 2] = 1.0, 2.0, 3.0
    a, ai = opol.left_align_content(emb, np.array([[2]]))
    assert ai.tolist() == [[4]]
    assert np.allclose(a[0, 2:, 0], [1, 2, 3]) and np.allclose(a[0, :2], 0)


# -- fixtures produced by the reference -------------------------------------

def test_position_ids_and_mask_match_reference():
    g = load("index_maps.npz")
    names = sorted({k[4:-3] for k in g if k.startswith("pos_") and k.endswith("_in")})
    assert names
    for name in names:
        got = opol.position_ids(g[f"pos_{name}_in"])
        assert np.array_equal(got, g[f"pos_{name}_out"].reshape(-1)), name
        if f"mask_{name}_allow" in g:
            assert np.array_equal(opol.segment_causal_allow(g[f"pos_{name}_in"]), g[f"mask_{name}_allow"])


def test_packing_maps_match_reference():
    g = load("index_maps.npz")
    for c in range(4):
        a, ai = opol.left_align_content(g[f"la{c}_emb"], g[f"la{c}_idx"])
        assert np.array_equal(ai, g[f"la{c}_outidx"])
        assert np.array_equal(a, g[f"la{c}_out"])
        steps = g[f"fb{c}_steps"]
        B, S = steps.shape[0], int(steps.max())
        o, tl, li = opol.flat_to_batched_left_pad(g[f"fb{c}_emb"], g[f"fb{c}_seq"], g[f"fb{c}_pidx"], B, S,
                                                  steps.tolist())
        assert np.array_equal(o, g[f"fb{c}_out"])
        assert tl == g[f"fb{c}_tl"].tolist()
        assert np.array_equal(li, g[f"fb{c}_local"])


def test_kv_policy_matches_reference():
    g = load("kv_policy.json")
    for mx, st, expect in g["bounds"]:
        assert list(opol.resolve_cache_bounds(mx, st)) == expect
    for ends, ctx, st, mx, expect in g["starts"]:
        got = opol.rebuild_starts(ends=np.array(ends), context_start=ctx if isinstance(ctx, int) else np.array(ctx),
                                  start_cache=st, max_cache=mx)
        assert got.tolist() == expect
    for has, cs, ce, ends, ctx, mx, comp, expect in g["rebuild"]:
        got = opol.cache_needs_rebuild(has_cache=has, cached_starts=np.array(cs), cached_ends=np.array(ce),
                                       ends=np.array(ends), context_start=np.array(ctx), max_cache=mx,
                                       batch_complete=comp)
        assert got == expect


def test_packed_attention_small_matches_reference():
    g = load("packed_attn_small.npz")
    scale = g["q"].shape[-1] ** -0.5
    out, _ = oatt.packed_attention_fwd(g["q"], g["k"], g["v"], g["seq"], scale)
    assert np.abs(out - g["out"]).max() < 1e-5
    dq, dk, dv = oatt.packed_attention_bwd(g["q"], g["k"], g["v"], g["seq"], scale, g["do"])
    for got, ref in ((dq, g["dq"]), (dk, g["dk"]), (dv, g["dv"])):
        assert np.abs(got - ref).max() < 1e-4


def test_packed_attention_cfg1_matches_reference():
    g = load("packed_attn_cfg1.npz")
    segs = cfg1_segments(0)
    assert segs == g["segs"].tolist()
    seq = np.concatenate([np.full(s, i) for i, s in enumerate(segs)])
    q, k, v, do = (t.numpy() for t in cfg1_inputs(0, 2048, 4, 2, 64))
    out, _ = oatt.packed_attention_fwd(q, k, v, seq, 64 ** -0.5)
    dq, dk, dv = oatt.packed_attention_bwd(q, k, v, seq, 64 ** -0.5, do)
    for name, t in (("out", out), ("dq", dq), ("dk", dk), ("dv", dv)):
        flat = t.reshape(-1)
        assert np.abs(flat[g[f"{name}_idx"]] - g[f"{name}_val"]).max() < 1e-4, name
        assert abs(np.abs(flat).sum() - float(g[f"{name}_abssum"])) < 1e-5 * float(g[f"{name}_abssum"]) + 1e-3


@pytest.mark.parametrize("arch", ["qwen3", "llama"])
def test_decode_session_oracle_matches_reference(arch):
    rec = load(f"decode_{arch}.npz")
    dec, _ = decoder_from_fixture(rec)
    sess = odec.DecodeSessionOracle(dec, batch_size=3)
    for ci, lens in enumerate(rec["schedule"].tolist()):
        h, layers = sess.forward(rec[f"c{ci}_emb"], lens, output_hidden_states=True)
        S = h.shape[1]
        ref = rec[f"c{ci}_out"]
        for b, n in enumerate(lens):
            # Real (trailing) columns must agree to the reference's own 1e-5.
            if n:
                assert np.abs(h[b, S - n:] - ref[b, S - n:]).max() < 1e-5, (arch, ci, b)
        # Pad columns: the reference's values are deterministic; ours agree too.
        assert np.abs(h - ref).max() < 1e-4
        assert np.abs(layers[0] - rec[f"c{ci}_layer0"]).max() < 1e-4
    assert sess.lengths.tolist() == rec["final_lengths"].tolist()


def test_packed_forward_oracle_matches_reference():
    rec = load("packed_fwd_qwen3.npz")
    rec = dict(rec)
    rec.setdefault("num_layers", np.array(2))
    rec.setdefault("n_heads", np.array(2))
    rec.setdefault("n_kv_heads", np.array(1))
    rec.setdefault("head_dim", np.array(64))
    rec.setdefault("qk_norm", np.array(True))
    dec, _ = decoder_from_fixture(rec)
    h = odec.packed_forward(dec, rec["emb"], rec["seq"])
    assert np.abs(h - rec["out"]).max() < 1e-4


@pytest.mark.parametrize("per_row", [False, True])
def test_grow_rebuild_oracle_matches_reference(per_row):
    """The oracle's restatement of the caller loop that drives the
    grow-then-rebuild policy equals the reference's own loop (its kv_policy
    functions and FlexDecodeSession) call for call: batch rebuilds, and each
    env run alone for the per-row semantics."""
    rec = load("grow_rebuild_qwen3.npz")
    dec, _ = decoder_from_fixture(rec)
    B = int(rec["B"])
    loop = odec.GrowRebuildOracle(dec, B, rec["table"].astype(np.float64), int(rec["max_cache"]),
                                  int(rec["start_cache"]), per_row=per_row)
    rebuilt = 0
    for ci in range(int(rec["calls"])):
        ended = rec[f"c{ci}_ended"]
        out, fed = loop.step(rec[f"c{ci}_hist"], rec[f"c{ci}_ends"], rec[f"c{ci}_ctx"],
                             ended if per_row else bool(ended.any()))
        S = out.shape[1]
        for b in range(B):
            if per_row:
                ref, n = rec[f"c{ci}_row{b}_out"][0], int(rec[f"c{ci}_row{b}_fed"][0])
            else:
                ref, n = rec[f"c{ci}_out"][b], int(rec[f"c{ci}_fed"][b])
            assert int(fed[b]) == n, (ci, b)
            if n:
                assert np.abs(out[b, S - n:] - ref[ref.shape[0] - n:]).max() < 1e-5, (ci, b)
        rebuilt += int((fed > 3).sum())  # a window longer than any append is a rebuild
    assert rebuilt >= 5


def test_embedding_oracle_matches_reference():
    """NumericEmbedder.forward restated: table rows for discrete and learnable
    tokens, static Fourier features for rff / continuous ones."""
    from oracle import encoder as oenc

    rec = load("embedding.npz")
    tables = {int(t): rec[f"w:_tables.{t}.weight"] for t, k in zip(rec["meta_type_id"], rec["meta_kind"])
              if str(k) != "fourier"}
    fourier = [int(t) for t, k in zip(rec["meta_type_id"], rec["meta_kind"]) if str(k) == "fourier"]
    for ci in range(2):
        got = oenc.embed_tokens(rec[f"c{ci}_token_types"], rec[f"c{ci}_token_ids"], rec[f"c{ci}_scalars"], tables,
                                fourier, rec["w:fourier.freqs"], rec["w:fourier.phases"],
                                float(rec["w:fourier.output_scale"]), int(rec["hidden_dim"]))
        assert np.abs(got - rec[f"c{ci}_embeds"]).max() < 1e-5
