"""Integer restatements of the reference's host-side hot-path helpers.

Test infrastructure (see ``oracle/__init__.py``). Every function is bit-exact
with the reference function it cites; ``tests/test_oracle_golden.py`` pins
each one against fixtures produced by the reference itself.
"""

from __future__ import annotations

import numpy as np


# ---------------------------------------------------------------------------
# kv_policy  (src/mouse_core/models/kv_policy.py:14-72)
# ---------------------------------------------------------------------------

def resolve_cache_bounds(max_cache, start_cache=None):
    """Restates ``kv_policy.resolve_cache_bounds`` (kv_policy.py:14-29)."""
    mx = int(max_cache)
    if mx < 1:
        mx = 1
    if start_cache is None:
        st = mx // 2
        if st < 1:
            st = 1
    else:
        st = int(start_cache)
        if st < 1:
            st = 1
    if st >= mx:
        st = mx - 1 if mx - 1 >= 1 else 1
    return mx, st


def rebuild_starts(*, ends, context_start, start_cache, max_cache):
    """Restates ``kv_policy.rebuild_starts`` (kv_policy.py:32-43)."""
    e = np.asarray(ends, dtype=np.int64)
    c = np.asarray(context_start, dtype=np.int64)
    span = int(start_cache) if int(start_cache) < int(max_cache) else int(max_cache)
    cand = e - span
    return np.where(c > cand, c, cand).astype(np.int64)


def cache_needs_rebuild(*, has_cache, cached_starts, cached_ends, ends,
                        context_start, max_cache, batch_complete):
    """Restates ``kv_policy.cache_needs_rebuild`` (kv_policy.py:46-72)."""
    if (not has_cache) or (not batch_complete):
        return True
    e = np.asarray(ends, dtype=np.int64)
    cs = np.asarray(cached_starts, dtype=np.int64)
    ce = np.asarray(cached_ends, dtype=np.int64)
    ctx = np.asarray(context_start, dtype=np.int64)
    if e.shape != cs.shape or e.shape != ce.shape:
        return True
    for i in range(e.size):
        if e.flat[i] < ce.flat[i]:
            return True
    # context_start broadcasts against cached_starts, as in the reference.
    if np.any(ctx > cs):
        return True
    for i in range(e.size):
        if e.flat[i] - cs.flat[i] > int(max_cache):
            return True
    return False


# ---------------------------------------------------------------------------
# Segment position ids / mask  (models/base.py:1204-1236, flex_train.py:84-102)
# ---------------------------------------------------------------------------

def position_ids(sequence_ids):
    """Per-token RoPE position inside its *run* of equal ``sequence_ids``.

    Restates ``_flat_sequence_position_ids`` (base.py:1226-1236) and the
    inlined copy in ``flex_packed_forward`` (flex_train.py:84-92): the
    position restarts at 0 wherever ``sequence_ids[i] != sequence_ids[i-1]``.
    Written as an explicit scan rather than the reference's cummax.
    """
    seq = np.asarray(sequence_ids).reshape(-1)
    out = np.zeros(seq.shape[0], dtype=np.int64)
    start = 0
    for i in range(seq.shape[0]):
        if i > 0 and seq[i] != seq[i - 1]:
            start = i
        out[i] = i - start
    return out


def segment_causal_allow(sequence_ids):
    """Boolean ``[L, L]``: ``kv <= q`` and same id (base.py:1212-1216,
    flex_train.py:98-102). Note the reference compares ids, not runs."""
    seq = np.asarray(sequence_ids).reshape(-1)
    L = seq.shape[0]
    q = np.arange(L)[:, None]
    kv = np.arange(L)[None, :]
    return (kv <= q) & (seq[:, None] == seq[None, :])


# ---------------------------------------------------------------------------
# Decode-layout packing  (embedding/packing.py:8-28, base.py:1163-1201)
# ---------------------------------------------------------------------------

def left_align_content(embeds, prediction_indices):
    """Restates ``left_align_content`` (packing.py:8-28).

    ``row_len = prediction_indices[:, -1] + 1``; rows with ``row_len > 0``
    move ``embeds[b, :row_len]`` to the trailing columns and shift their
    indices by ``L - row_len``.
    """
    emb = np.asarray(embeds)
    idx = np.asarray(prediction_indices, dtype=np.int64)
    B, L = emb.shape[0], emb.shape[1]
    aligned = np.zeros_like(emb)
    out_idx = idx.copy()
    for b in range(B):
        rl = int(idx[b, -1]) + 1
        if rl == 0:
            continue
        off = L - rl
        aligned[b, off:] = emb[b, :rl]
        out_idx[b] = idx[b] + off
    return aligned, out_idx


def flat_to_batched_left_pad(embeds, sequence_ids, prediction_indices, B, S, step_counts):
    """Restates ``_flat_to_batched_left_pad`` (base.py:1163-1201).

    Returns ``(out [B, Lmax, D], token_lengths list, local_indices [B, S])``:
    row ``b`` holds the tokens whose id is ``b`` packed from column 0, and
    ``local_indices[b, S - n + s]`` is the in-row index of that row's
    ``s``-th prediction token (``n = step_counts[b]``).
    """
    emb = np.asarray(embeds)
    seq = np.asarray(sequence_ids).reshape(-1)
    pidx = np.asarray(prediction_indices, dtype=np.int64).reshape(-1)
    L, D = emb.shape
    token_lengths = [int(np.count_nonzero(seq == b)) for b in range(B)]
    lmax = max(token_lengths) if token_lengths else 0
    out = np.zeros((B, lmax, D), dtype=emb.dtype)
    local_of_abs = np.full(L, -1, dtype=np.int64)
    for b in range(B):
        where = np.nonzero(seq == b)[0]
        out[b, : where.shape[0]] = emb[where]
        local_of_abs[where] = np.arange(where.shape[0])
    local = np.zeros((B, S), dtype=np.int64)
    flat = 0
    for b in range(B):
        n = int(step_counts[b]) if b < len(step_counts) else S
        for s in range(n):
            local[b, S - n + s] = local_of_abs[pidx[flat + s]]
        flat += n
    return out, token_lengths, local


# ---------------------------------------------------------------------------
# Cached-decode bookkeeping  (backbone/flex_decode.py:176-196)
# ---------------------------------------------------------------------------

def decode_positions(cached_lengths, new_lengths, S):
    """Per-column positions of one ``FlexDecodeSession.forward`` call.

    Restates flex_decode.py:184-196: ``pos = lengths[b] + col - pad``
    (``pad = S - n``); the attention limit / RoPE position is
    ``max(pos, 0)``; column ``col`` is a real token iff ``col >= pad`` and its
    cache slot is ``pos``. Returns ``(q_pos [B,S], real [B,S] bool)``.
    """
    lens = np.asarray(cached_lengths, dtype=np.int64)
    n = np.asarray(new_lengths, dtype=np.int64)
    col = np.arange(S, dtype=np.int64)[None, :]
    pad = (S - n)[:, None]
    pos = lens[:, None] + col - pad
    return np.maximum(pos, 0), col >= pad
