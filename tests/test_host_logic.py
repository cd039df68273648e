"""Host-side logic of mouse_core_b200 on CPU: the kv_policy and packing maps
must equal the reference's outputs bit for bit (fixtures made by the
reference itself), the page table must behave as a refcounted pool, and the
FMA-pipe exp2 of the attention backward must meet its error bound."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mouse_core_b200 as mb
from mouse_core_b200.pages import PageTable
from tests.golden_io import load


def test_kv_policy_bit_exact_with_reference():
    g = load("kv_policy.json")
    for mx, st, expect in g["bounds"]:
        assert list(mb.resolve_cache_bounds(mx, st)) == expect
    for ends, ctx, st, mx, expect in g["starts"]:
        got = mb.rebuild_starts(ends=np.array(ends), context_start=ctx if isinstance(ctx, int) else np.array(ctx),
                                start_cache=st, max_cache=mx)
        assert got.dtype == np.int64 and got.tolist() == expect
    for has, cs, ce, ends, ctx, mx, comp, expect in g["rebuild"]:
        got = mb.cache_needs_rebuild(has_cache=has, cached_starts=np.array(cs), cached_ends=np.array(ce),
                                     ends=np.array(ends), context_start=np.array(ctx), max_cache=mx,
                                     batch_complete=comp)
        assert got is expect


def test_rows_needing_rebuild_agrees_with_batch_rule():
    g = load("kv_policy.json")
    for has, cs, ce, ends, ctx, mx, comp, expect in g["rebuild"]:
        if not has or not comp or len(ends) != len(cs):
            continue
        rows = mb.rows_needing_rebuild(cached_starts=np.array(cs), cached_ends=np.array(ce), ends=np.array(ends),
                                       context_start=np.array(ctx), max_cache=mx)
        assert bool(rows.any()) == expect


def test_position_ids_and_mask_bit_exact():
    g = load("index_maps.npz")
    names = sorted({k[4:-3] for k in g if k.startswith("pos_") and k.endswith("_in")})
    for name in names:
        seq = torch.tensor(g[f"pos_{name}_in"], dtype=torch.long)
        got = mb.flat_sequence_position_ids(seq)
        assert torch.equal(got, torch.tensor(g[f"pos_{name}_out"]).view(1, -1)), name
        if f"mask_{name}_allow" in g:
            m = mb.flat_sequence_causal_mask(sequence_ids=seq, dtype=torch.float32)
            assert torch.equal(m[0, 0] == 0, torch.tensor(g[f"mask_{name}_allow"]))


def test_packing_maps_bit_exact():
    g = load("index_maps.npz")
    for c in range(4):
        a, ai = mb.left_align_content(torch.tensor(g[f"la{c}_emb"]), torch.tensor(g[f"la{c}_idx"]))
        assert torch.equal(ai, torch.tensor(g[f"la{c}_outidx"]))
        assert torch.equal(a, torch.tensor(g[f"la{c}_out"]))
        steps = g[f"fb{c}_steps"]
        B, S = steps.shape[0], int(steps.max())
        o, tl, li = mb.flat_to_batched_left_pad(torch.tensor(g[f"fb{c}_emb"]), torch.tensor(g[f"fb{c}_seq"]),
                                                torch.tensor(g[f"fb{c}_pidx"]), B, S, steps.tolist())
        assert torch.equal(o, torch.tensor(g[f"fb{c}_out"]))
        assert tl == g[f"fb{c}_tl"].tolist()
        assert torch.equal(li, torch.tensor(g[f"fb{c}_local"]))


def test_page_table_allocate_release_share():
    pt = PageTable(batch_size=3, num_pages=8, page_size=64, max_pages=1)
    add = pt.pages_needed(np.array([1, 130, 0]))
    assert add.tolist() == [1, 3, 0]
    pt.allocate(add)
    assert pt.free_pages == 4 and pt.max_pages >= 3
    used = set(pt.table[0, :1].tolist()) | set(pt.table[1, :3].tolist())
    assert len(used) == 4 and all(0 <= p < 8 for p in used)
    # slots land in the right pages
    s = pt.slots(np.array([1, 1]), np.array([0, 129]))
    assert s[0] == pt.table[1, 0] * 64 and s[1] == pt.table[1, 2] * 64 + 1
    # copy-free sharing keeps pages alive until every holder lets go
    pt.share(2, 1, 2)
    assert (pt.table[2, :2] == pt.table[1, :2]).all() and pt.free_pages == 4
    pt.release_rows([1])
    assert pt.free_pages == 5  # only the unshared third page came back
    pt.release_rows([2, 0])
    assert pt.free_pages == 8
    # growth registers new pages
    pt.grow_pool(12)
    pt.allocate(np.array([12, 0, 0]) // 1)
    assert pt.free_pages == 0
    try:
        pt.allocate(np.array([1, 0, 0]))
    except RuntimeError as e:
        assert "exhausted" in str(e)
    else:
        raise AssertionError("allocation beyond the pool must raise")


def test_page_table_release_after_growth_with_pages_in_use():
    """Pages held across a pool growth return to the free list when their
    rows are released, and every page id is handed out exactly once."""
    pt = PageTable(batch_size=3, num_pages=4, page_size=64, max_pages=1)
    pt.allocate(np.array([2, 2, 0]))
    pt.grow_pool(8)
    pt.allocate(np.array([0, 0, 3]))
    pt.grow_pool(20)
    pt.release_rows([0, 1, 2])
    assert pt.free_pages == 20
    pt.allocate(np.array([7, 6, 7]))
    assert sorted(pt.table[pt.table >= 0].tolist()) == list(range(20))


def test_open_pages_hands_out_what_allocate_does():
    a = PageTable(batch_size=5, num_pages=16, page_size=64, max_pages=4)
    b = PageTable(batch_size=5, num_pages=16, page_size=64, max_pages=4)
    for pt in (a, b):
        pt.allocate(np.array([1, 0, 2, 1, 0]))
        pt.release_rows([3])
    rows = np.array([0, 1, 3, 4])
    b.dirty = False
    ids = b.open_pages(rows)
    a.allocate(np.isin(np.arange(5), rows).astype(np.int64))
    assert np.array_equal(a.table, b.table) and np.array_equal(a.npages, b.npages)
    assert np.array_equal(a.refcount, b.refcount) and a.free_pages == b.free_pages
    assert ids.tolist() == b.table[rows, b.npages[rows] - 1].tolist()
    assert not b.dirty


def _fma32(a, b, c):
    """float32 fused multiply-add (the float64 product of two float32s is exact)."""
    return (a.astype(np.float64) * b + c).astype(np.float32)


def test_exp2_fma_error_bound():
    """The FMA-pipe 2^x of the attention kernels (`exp2_fma`, and its packed
    pair form `exp2_fma2`, whose steps round the same way; tcgen05.cuh),
    restated step by step in float32: magic-number rounding to n, a cubic in
    f = x - n on [-0.5, 0.5], n added to the exponent field. Its relative
    error stays below 1.1e-4 (under bf16's half-ulp of 2^-9) over the softmax
    range, and the clamp keeps very negative inputs at ~1e-38."""
    x = np.linspace(-126.0, 0.0, 2_000_001, dtype=np.float32)
    x = np.concatenate([x, np.array([0.49999997, -0.5, -0.50000006, 1e-8, -1e-8], dtype=np.float32)])
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic)).astype(np.float32)
    assert float(np.abs(f).max()) <= 0.5
    p = _fma32(np.float32(0.0550089821), f, np.float32(0.242210975))
    p = _fma32(p, f, np.float32(0.693282916))
    p = _fma32(p, f, np.float32(1.0))
    bits = (p.view(np.int32).astype(np.int64) + (t.view(np.int32).astype(np.int64) << 23)) & 0xFFFFFFFF
    y = bits.astype(np.uint32).view(np.float32).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y - ref) / ref
    assert float(rel.max()) < 1.1e-4
    clamped = np.float32(-126.0)
    assert 0.0 < float(np.exp2(np.float64(clamped))) < 1e-37


def test_pair_count_matches_brute_force():
    """Pairs of (128-query tile, 128-key tile) the segment-causal attention
    visits: a pair is visited when some query of the tile sees some key of the
    other tile (same run, key <= query)."""
    from mouse_core_b200.packed import pair_count

    rng = np.random.default_rng(4)
    for lens in ([1], [128], [129], [300, 1, 1, 700], list(rng.integers(1, 400, size=20)), [2048, 5]):
        ids = np.repeat(np.arange(len(lens)), lens)
        L = ids.shape[0]
        T = (L + 127) // 128
        brute = 0
        for i in range(T):
            q = np.arange(128 * i, min(128 * i + 128, L))
            for j in range(i + 1):
                k = np.arange(128 * j, min(128 * j + 128, L))
                brute += bool(((ids[q][:, None] == ids[k][None, :]) & (k[None, :] <= q[:, None])).any())
        assert pair_count(ids) == brute, lens
    assert pair_count(np.zeros(0, dtype=np.int64)) == 0


def test_install_patches_and_restores_the_reference_hot_path(monkeypatch):
    """``install()`` swaps exactly the hot-path functions of an importable
    ``mouse_core`` (here stand-in modules with the same names) for ours, and
    ``uninstall()`` puts every original back."""
    import sys
    import types

    from mouse_core_b200 import integration, kv_policy, packing
    from mouse_core_b200.decode import PagedDecodeSession

    def orig(*a, **k):
        raise AssertionError("original called")

    mods = {}
    for name in ("mouse_core", "mouse_core.models", "mouse_core.models.backbone", "mouse_core.models.backbone.base",
                 "mouse_core.models.backbone.flex_train", "mouse_core.models.embedding",
                 "mouse_core.models.embedding.packing", "mouse_core.models.base", "mouse_core.models.kv_policy",
                 "mouse_core.models.embedding.embedding"):
        mods[name] = types.ModuleType(name)
        monkeypatch.setitem(sys.modules, name, mods[name])

    class Backbone:
        decode_session = orig

    mods["mouse_core.models.backbone.base"].Backbone = Backbone

    class NumericEmbedder:
        forward = orig

    mods["mouse_core.models.embedding.embedding"].NumericEmbedder = NumericEmbedder
    mods["mouse_core.models.backbone.flex_train"].flex_packed_forward = orig
    mods["mouse_core.models.embedding.packing"].left_align_content = orig
    mods["mouse_core.models.base"]._flat_to_batched_left_pad = orig
    for fn in ("resolve_cache_bounds", "rebuild_starts", "cache_needs_rebuild"):
        setattr(mods["mouse_core.models.kv_policy"], fn, orig)

    integration.install()
    try:
        assert mods["mouse_core.models.embedding.packing"].left_align_content is packing.left_align_content
        assert mods["mouse_core.models.base"]._flat_to_batched_left_pad is packing.flat_to_batched_left_pad
        assert mods["mouse_core.models.kv_policy"].cache_needs_rebuild is kv_policy.cache_needs_rebuild
        from mouse_core_b200.packed import flex_packed_forward

        assert mods["mouse_core.models.backbone.flex_train"].flex_packed_forward is flex_packed_forward
        assert Backbone.decode_session is not orig
        assert NumericEmbedder.forward is not orig
        try:
            Backbone().decode_session(batch_size=2, capacity=8)  # no ``model``: the reference's error
        except NotImplementedError:
            pass
        else:
            raise AssertionError("a backbone without a model must not get a session")
        assert PagedDecodeSession is not None
    finally:
        integration.uninstall()
    assert Backbone.decode_session is orig
    assert NumericEmbedder.forward is orig
    assert mods["mouse_core.models.embedding.packing"].left_align_content is orig
    assert mods["mouse_core.models.base"]._flat_to_batched_left_pad is orig
    assert mods["mouse_core.models.backbone.flex_train"].flex_packed_forward is orig
    for fn in ("resolve_cache_bounds", "rebuild_starts", "cache_needs_rebuild"):
        assert getattr(mods["mouse_core.models.kv_policy"], fn) is orig


def test_decode_rope_frequencies_survive_a_bf16_cast():
    """Casting a backbone to bf16 rounds its rotary module's inv_freq buffer;
    the decode session recomputes the config's fp32 frequencies (default and
    Llama-3 rope types) instead."""
    import torch

    from mouse_core_b200.backbone import LlamaBackbone, Qwen3Backbone
    from mouse_core_b200.decode import rope_frequencies

    for bb in (Qwen3Backbone(hidden_dim=256, num_layers=1, num_heads=2, num_key_value_heads=1, head_dim=128,
                             rope_parameters={"rope_type": "default", "rope_theta": 1e6}),
               LlamaBackbone(hidden_dim=256, num_layers=1, num_heads=4, num_key_value_heads=2,
                             max_position_embeddings=16384,
                             rope_parameters={"rope_type": "llama3", "rope_theta": 5e5, "factor": 32.0,
                                              "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                                              "original_max_position_embeddings": 8192})):
        exact = bb.model.rotary_emb.inv_freq.clone()
        bb = bb.to(torch.bfloat16)
        assert not torch.equal(bb.model.rotary_emb.inv_freq.float(), exact)  # the cast rounded the buffer
        inv, scaling = rope_frequencies(bb.model.rotary_emb, bb.model.config, torch.device("cpu"))
        assert inv.dtype == torch.float32 and torch.equal(inv, exact)
        assert scaling == float(bb.model.rotary_emb.attention_scaling)


def test_pack_windows_into_fixed_rows():
    """Windows stay whole, every window lands once, rows respect the token
    budget, offsets tile each row in the windows' original order, and
    sequence ids / cu_seqlens describe the same segments."""
    import numpy as np
    import torch

    from mouse_core_b200.packing import flat_sequence_position_ids, pack_rows, pack_windows

    rng = np.random.default_rng(3)
    lengths = rng.integers(256, 4097, size=37)
    row, off, tokens = pack_windows(lengths, 16384)
    assert tokens.max() <= 16384 and tokens.sum() == lengths.sum()
    assert tokens.size <= int(np.ceil(lengths.sum() / 16384)) + 2  # first fit decreasing is near the bound
    for r in range(tokens.size):
        ids = np.flatnonzero(row == r)
        assert np.array_equal(off[ids], np.concatenate([[0], np.cumsum(lengths[ids])[:-1]]))
    with pytest.raises(ValueError):
        pack_windows([5, 20000], 16384)
    windows = [{"token_ids": rng.integers(0, 1024, size=n), "reward": rng.random(n)} for n in lengths]
    rows = pack_rows(windows, 16384)
    seen = np.concatenate([r["window_ids"] for r in rows])
    assert np.array_equal(np.sort(seen), np.arange(lengths.size))
    for r in rows:
        n = r["token_ids"].shape[0]
        assert n <= 16384 and r["sequence_ids"].shape == (n,) and r["cu_seqlens"][-1] == n
        assert np.array_equal(np.diff(r["cu_seqlens"]), lengths[r["window_ids"]])
        assert np.array_equal(r["token_ids"][:lengths[r["window_ids"][0]]], windows[r["window_ids"][0]]["token_ids"])
        pos = flat_sequence_position_ids(torch.from_numpy(r["sequence_ids"])).numpy().reshape(-1)
        assert np.array_equal(pos[r["cu_seqlens"][:-1]], np.zeros(len(r["window_ids"])))
