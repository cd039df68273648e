"""Grow-then-rebuild decoding end to end on the GPU.

``GrowRebuildDecoder`` runs the caller loop that applies the reference's
grow-then-rebuild policy (kv_policy.py:14-72, driven by ``run_eval``'s
``_act_from_contexts`` in examples/02_train_offline.ipynb) on the paged
session: ``cache_needs_rebuild`` / ``rows_needing_rebuild`` decide, the
rebuilt rows are emptied (``reset_rows``) and re-prefilled from
``rebuild_starts`` in the same ragged call as the appended rows. Every real
token's hidden state is compared after every call with the oracle's loop
(``oracle.decoder.GrowRebuildOracle``, pinned to the reference's own loop by
tests/test_oracle_golden.py): batch mode against the reference's whole-batch
rebuild, per-row mode against each env run alone.

Tolerance: the oracle runs in float64 on the same bf16-rounded weights and
embeddings, so the difference is the kernels' bf16 arithmetic. The hidden
states carry the bf16 residual stream (each add rounds to 2^-8 relative), so
the bound is 2e-2 x max(1, the token's largest magnitude), as for the other
whole-decoder checks.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import decoder as odec
from tests.golden_io import decoder_from_fixture, grow_rebuild_schedule, load

pytestmark = pytest.mark.gpu

ATOL = 2e-2


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


def _check(out, fed, ref_out, ref_fed, where):
    h = out.float().cpu().numpy()
    assert np.isfinite(h).all(), where
    assert fed.tolist() == np.asarray(ref_fed).tolist(), where
    S, Sr = h.shape[1], ref_out.shape[1]
    worst = 0.0
    for b, n in enumerate(fed.tolist()):
        if n:
            a, r = h[b, S - n:], ref_out[b, Sr - n:]
            err = float(np.abs(a - r).max())
            bound = ATOL * max(1.0, float(np.abs(r).max()))
            assert err <= bound, (where, b, err, bound)
            worst = max(worst, err)
    return worst


@pytest.mark.parametrize("per_row", [False, True])
def test_grow_rebuild_matches_reference_loop_fixture(per_row):
    """The reference's own loop recorded on a tiny Qwen3 (tests/golden):
    ours and the bf16-weight oracle follow the same schedule; ours must match
    the oracle and make the same fed/rebuild decisions as the reference."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.grow_rebuild import GrowRebuildDecoder

    rec = load("grow_rebuild_qwen3.npz")
    B = int(rec["B"])
    bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    sd = {k[2:]: torch.from_numpy(v.astype(np.float32)) for k, v in rec.items() if k.startswith("w:")}
    missing, unexpected = bb.model.load_state_dict(sd, strict=False)
    assert not unexpected and all("rotary" in m for m in missing)
    bb.model.rotary_emb.inv_freq.copy_(torch.from_numpy(rec["inv_freq"]))
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    table16 = torch.from_numpy(rec["table"]).bfloat16()
    rec16 = dict(rec)
    for k in list(rec16):
        if k.startswith("w:"):
            rec16[k] = torch.from_numpy(rec[k].astype(np.float32)).bfloat16().float().numpy()
    dec16, _ = decoder_from_fixture(rec16)
    oracle = odec.GrowRebuildOracle(dec16, B, table16.float().numpy(), int(rec["max_cache"]),
                                    int(rec["start_cache"]), per_row=per_row)
    table_dev = table16.to(dev)
    ours = GrowRebuildDecoder(bb, B, lambda ids: table_dev[ids], max_cache=int(rec["max_cache"]),
                              start_cache=int(rec["start_cache"]), per_row=per_row, page_size=64)
    for ci in range(int(rec["calls"])):
        ended = rec[f"c{ci}_ended"]
        rb = ended if per_row else bool(ended.any())
        args = (rec[f"c{ci}_hist"], rec[f"c{ci}_ends"], rec[f"c{ci}_ctx"])
        out, fed = ours.step(*args, rebuild=rb)
        o_out, o_fed = oracle.step(*args, rebuild=rb)
        if per_row:
            ref_fed = [int(rec[f"c{ci}_row{b}_fed"][0]) for b in range(B)]
        else:
            ref_fed = rec[f"c{ci}_fed"]
        assert fed.tolist() == list(np.asarray(ref_fed).tolist()), ci  # the reference's decisions
        _check(out, fed, o_out, o_fed, ci)
    assert ours.rebuild_calls >= 5


@pytest.mark.parametrize("per_row", [False, True])
def test_grow_rebuild_random_loop_matches_oracle(per_row):
    """max_cache 96 / start_cache 40, 6 envs, 60 calls of ragged 0-5 token
    appends (so cached spans cross max_cache within the run) with task ends
    and context-start moves, on a Qwen3-shaped model
    (hd 128, GQA 2, 128-token pages so windows straddle page boundaries and
    rebuilt rows reuse freed pages)."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.grow_rebuild import GrowRebuildDecoder

    torch.manual_seed(17)
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
    B, calls, vocab = 6, 60, 97
    table16 = torch.randn(vocab, 256, generator=torch.Generator().manual_seed(6)).bfloat16()
    table_dev = table16.to(dev)
    oracle = odec.GrowRebuildOracle(dec, B, table16.float().numpy(), 96, 40, per_row=per_row)
    ours = GrowRebuildDecoder(bb, B, lambda ids: table_dev[ids], max_cache=96, start_cache=40, per_row=per_row)
    overflowed = 0
    for ci, (hist, ends, ctx, ended) in enumerate(grow_rebuild_schedule(23, B, calls, vocab, max_append=5)):
        overflowed += int((ends - ours.cached_starts > 96).sum()) if ours.session is not None else 0
        rb = ended if per_row else bool(ended.any())
        out, fed = ours.step(hist, ends, ctx, rebuild=rb)
        o_out, o_fed = oracle.step(hist, ends, ctx, rebuild=rb)
        _check(out, fed, o_out, o_fed, ci)
    assert ours.rebuild_calls >= 3, ours.rebuild_calls
    if per_row:  # batch mode rebuilds on every task end, before any span gets that long
        assert overflowed >= 2, overflowed  # rebuilds by max_cache, not only by task ends
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0


def test_grow_rebuild_crosses_max_cache_in_one_token_steps():
    """One token per env per call (the decode benchmark's stepping): rows
    cross max_cache at different calls, so per-row rebuilds re-prefill one
    window of start_cache tokens in the same call as the other rows' one-token
    appends; the output of every call equals the oracle's."""
    dev = _dev()
    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.grow_rebuild import GrowRebuildDecoder

    torch.manual_seed(5)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    with torch.no_grad():
        for p in bb.model.parameters():
            p.copy_(p.bfloat16().float())
    sd = {k: v.detach().numpy() for k, v in bb.model.state_dict().items() if "rotary" not in k}
    dec = odec.DecoderOracle(sd, odec.config_from_hf(bb.model.config, bb.model.rotary_emb.inv_freq.numpy()))
    bb = bb.to(device=dev, dtype=torch.bfloat16).eval()
    B, vocab, max_cache, start_cache = 4, 64, 160, 150
    table16 = torch.randn(vocab, 256, generator=torch.Generator().manual_seed(2)).bfloat16()
    table_dev = table16.to(dev)
    rng = np.random.default_rng(4)
    hist = rng.integers(0, vocab, size=(B, 400))
    ends = np.array([150, 100, 40, 145])
    ours = GrowRebuildDecoder(bb, B, lambda ids: table_dev[ids], max_cache=max_cache, start_cache=start_cache,
                              per_row=True, page_size=64)
    oracle = odec.GrowRebuildOracle(dec, B, table16.float().numpy(), max_cache, start_cache, per_row=True)
    for ci in range(40):
        out, fed = ours.step(hist, ends, 0)
        o_out, o_fed = oracle.step(hist, ends, 0)
        _check(out, fed, o_out, o_fed, ci)
        ends = ends + 1
    # After the first prefill, row 0 overflows at calls 11, 22 and 33 and row 3
    # at 16, 27 and 38, each re-windowed to its last 150 tokens.
    assert ours.rows_rebuilt == B + 6, ours.rows_rebuilt
