"""Helpers that load the golden fixtures of ``tests/golden`` (written by
``tests/golden/make_golden.py`` from the reference itself)."""

from __future__ import annotations

import json
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def load(name):
    path = os.path.join(GOLDEN, name)
    if name.endswith(".json"):
        with open(path) as f:
            return json.load(f)
    return dict(np.load(path, allow_pickle=False))


def cfg1_segments(seed=0, L=2048, lo=16, hi=512):
    """Segment lengths of the 2048-token packed workload (seeded)."""
    rng = np.random.default_rng(seed)
    segs, total = [], 0
    while total < L:
        s = min(int(rng.integers(lo, hi + 1)), L - total)
        segs.append(s)
        total += s
    return segs


def cfg1_inputs(seed, L, Hq, Hkv, hd):
    """q, k, v, dout of the packed workload from a torch CPU generator."""
    import torch

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(L, Hq, hd, generator=g)
    k = torch.randn(L, Hkv, hd, generator=g)
    v = torch.randn(L, Hkv, hd, generator=g)
    do = torch.randn(L, Hq, hd, generator=g)
    return q, k, v, do


def decoder_from_fixture(rec):
    """(DecoderOracle, weights dict as float32 numpy) from a decode fixture."""
    from oracle.decoder import DecoderConfig, DecoderOracle

    weights = {k[2:]: v.astype(np.float32) for k, v in rec.items() if k.startswith("w:")}
    cfg = DecoderConfig(
        num_layers=int(rec["num_layers"]) if "num_layers" in rec else 2,
        n_heads=int(rec["n_heads"]) if "n_heads" in rec else 2,
        n_kv_heads=int(rec["n_kv_heads"]) if "n_kv_heads" in rec else 1,
        head_dim=int(rec["head_dim"]) if "head_dim" in rec else 64,
        eps=float(rec["eps"]),
        qk_norm=bool(rec["qk_norm"]) if "qk_norm" in rec else True,
        inv_freq=rec["inv_freq"].astype(np.float64),
        attention_scaling=float(rec["attention_scaling"]) if "attention_scaling" in rec else 1.0,
    )
    return DecoderOracle(weights, cfg), weights


def grow_rebuild_schedule(seed: int, B: int, calls: int, vocab: int, max_append: int = 3):
    """A caller-loop schedule for the grow-then-rebuild fixtures: before each
    call every env either ends its task (context cleared, ``context_start``
    back to 0, a forced rebuild as the reference's loop does on a task end),
    moves its ``context_start`` forward, or appends 0..``max_append`` new
    tokens. Yields
    ``(history [B, T], ends [B], context_start [B], task_ended [B])`` per call."""
    rng = np.random.default_rng(seed)
    hist = [[] for _ in range(B)]
    ctx = np.zeros(B, dtype=np.int64)
    for _ in range(calls):
        ended = np.zeros(B, dtype=bool)
        for b in range(B):
            u = rng.random()
            if hist[b] and u < 0.06:
                hist[b] = []
                ctx[b] = 0
                ended[b] = True
            elif len(hist[b]) > 4 and u < 0.09:
                ctx[b] = max(int(ctx[b]), len(hist[b]) - 3)
            else:
                hist[b].extend(int(t) for t in rng.integers(0, vocab, size=int(rng.integers(0, max_append + 1))))
        ends = np.array([len(h) for h in hist], dtype=np.int64)
        T = max(int(ends.max()), 1)
        arr = np.zeros((B, T), dtype=np.int64)
        for b in range(B):
            arr[b, :ends[b]] = hist[b]
        yield arr, ends, ctx.copy(), ended
