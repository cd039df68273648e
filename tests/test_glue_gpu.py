"""K9 decode-step layout glue on the GPU (``mb_flat_rank``, ``mb_flat_scatter``,
``mb_left_align`` behind ``flat_to_batched_left_pad`` / ``left_align_content``):
bit-exact against the fixtures the reference produced and against the
oracle's restatement on randomised layouts (interleaved ids, ids outside the
batch, rows without steps, negative prediction indices, three copy widths)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import mouse_core_b200 as mb
from oracle import policy as opol
from tests.golden_io import load

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def test_glue_matches_reference_fixtures():
    dev = _dev()
    g = load("index_maps.npz")
    for c in range(4):
        a, ai = mb.left_align_content(torch.tensor(g[f"la{c}_emb"]).to(dev), torch.tensor(g[f"la{c}_idx"]).to(dev))
        assert torch.equal(ai.cpu(), torch.tensor(g[f"la{c}_outidx"]))
        assert torch.equal(a.cpu(), torch.tensor(g[f"la{c}_out"]))
        steps = g[f"fb{c}_steps"]
        B, S = steps.shape[0], int(steps.max())
        o, tl, li = mb.flat_to_batched_left_pad(torch.tensor(g[f"fb{c}_emb"]).to(dev),
                                                torch.tensor(g[f"fb{c}_seq"]).to(dev),
                                                torch.tensor(g[f"fb{c}_pidx"]).to(dev), B, S, steps.tolist())
        assert torch.equal(o.cpu(), torch.tensor(g[f"fb{c}_out"]))
        assert tl == g[f"fb{c}_tl"].tolist()
        assert torch.equal(li.cpu(), torch.tensor(g[f"fb{c}_local"]))


@pytest.mark.parametrize("seed,B,D,dtype", [(0, 7, 1024, torch.bfloat16), (1, 300, 6, torch.bfloat16),
                                            (2, 33, 3, torch.bfloat16), (3, 64, 5, torch.float32),
                                            (4, 4096, 16, torch.bfloat16)])
def test_glue_matches_oracle_random(seed, B, D, dtype):
    """Ids interleaved at random (some outside [0, B)), per-row step counts
    0..S (some rows missing from step_counts), prediction indices into the
    row's own tokens (some written negative, counted from the end)."""
    dev = _dev()
    rng = np.random.default_rng(seed)
    S = int(rng.integers(1, 9))
    L = int(rng.integers(B, 4 * B + 2))
    seq = rng.integers(-1, B + 1, size=L)
    emb = torch.randn(L, D, generator=torch.Generator().manual_seed(seed)).to(dtype)
    cut = int(rng.integers(max(B - 3, 0), B + 1))  # rows past len(step_counts) take S steps
    steps_arg, pred = [], []
    for b in range(B):
        toks = np.flatnonzero(seq == b)
        if b < cut:
            n = int(min(rng.integers(0, S + 1), toks.shape[0]))
            picks = np.sort(rng.choice(toks, size=n, replace=False)) if n else np.zeros(0, dtype=np.int64)
            steps_arg.append(n)
        else:  # S indices, any tokens (another id's token gives that id's rank, as in the reference)
            picks = rng.choice(toks, size=S) if toks.shape[0] else rng.integers(0, L, size=S)
        picks = np.where(rng.random(picks.shape[0]) < 0.2, picks - L, picks)  # same tokens, negative form
        pred.extend(picks.tolist())
    pred_t = torch.tensor(pred, dtype=torch.long)

    o_ref, tl_ref, li_ref = opol.flat_to_batched_left_pad(emb.float().numpy(), seq, pred_t.numpy(), B, S,
                                                          steps_arg)
    o, tl, li = mb.flat_to_batched_left_pad(emb.to(dev), torch.from_numpy(seq).to(dev), pred_t.to(dev), B, S,
                                            steps_arg)
    assert tl == tl_ref
    assert np.array_equal(li.cpu().numpy(), li_ref)
    assert np.array_equal(o.float().cpu().numpy(), o_ref)

    a_ref, ai_ref = opol.left_align_content(o_ref, li_ref)
    a, ai = mb.left_align_content(o, li)
    assert np.array_equal(ai.cpu().numpy(), ai_ref)
    assert np.array_equal(a.float().cpu().numpy(), a_ref)
    # the CPU torch path agrees too
    a_cpu, ai_cpu = mb.left_align_content(o.cpu(), li.cpu())
    assert torch.equal(a_cpu, a.cpu()) and torch.equal(ai_cpu, ai.cpu())


def test_glue_rejects_out_of_range_prediction_index():
    dev = _dev()
    emb = torch.zeros(4, 8, device=dev)
    seq = torch.tensor([0, 0, 1, 1], device=dev)
    with pytest.raises(IndexError):
        mb.flat_to_batched_left_pad(emb, seq, torch.tensor([0, 9], device=dev), 2, 1, [1, 1])
    with pytest.raises(IndexError):  # fewer prediction indices than the step counts read
        mb.flat_to_batched_left_pad(emb, seq, torch.tensor([0], device=dev), 2, 1, [1, 1])
    with pytest.raises(IndexError):
        mb.left_align_content(torch.zeros(2, 3, 8, device=dev), torch.zeros(2, 0, dtype=torch.long, device=dev))
