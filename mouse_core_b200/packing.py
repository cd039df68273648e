"""Decode-layout and segment index maps of the packed/cached paths.

Same functions and results as the reference (bit-exact; checked against
fixtures it produced), written as whole-tensor gathers instead of the
reference's per-row Python loops with ``.item()`` host syncs:

* ``left_align_content``             embedding/packing.py:8-28
* ``flat_to_batched_left_pad``       models/base.py:1163-1201
* ``flat_sequence_position_ids``     models/base.py:1226-1236
* ``flat_sequence_causal_mask``      models/base.py:1204-1223

On CPU tensors they are whole-tensor torch ops (the reference's CPU path).
On CUDA tensors the two decode-step maps run as the K9 kernels
(``mb_flat_rank`` + ``mb_flat_scatter``, ``mb_left_align``): one rank/count
pass in a single CTA, one read-back of the counts (``token_lengths`` is a
host list and sets the output width), one scatter, one shift. The CUDA
training path computes position ids with the K7 segment kernel instead
(``mouse_core_b200.packed``).
"""

from __future__ import annotations

import numpy as np
import torch


def left_align_content(embeds: torch.Tensor, prediction_indices: torch.Tensor):
    """Shift right-padded rows so content sits in the trailing columns.

    Row ``b`` has ``prediction_indices[b, -1] + 1`` content columns; rows with
    content move it to columns ``L - row_len ..`` and shift their indices by
    ``L - row_len``. Returns ``(aligned_embeds, aligned_indices)``.
    """
    if embeds.is_cuda:
        return _left_align_content_cuda(embeds, prediction_indices)
    B, L = embeds.shape[0], embeds.shape[1]
    row_len = prediction_indices[:, -1] + 1
    has = row_len > 0
    offset = torch.where(has, L - row_len, torch.zeros_like(row_len))
    col = torch.arange(L, device=embeds.device)[None, :]
    src = col - offset[:, None]
    keep = (src >= 0) & has[:, None]
    gathered = torch.gather(embeds, 1, src.clamp_min(0)[..., None].expand(B, L, embeds.shape[2]))
    aligned = torch.where(keep[..., None], gathered, torch.zeros((), dtype=embeds.dtype, device=embeds.device))
    return aligned, prediction_indices + offset[:, None]


def _rank_within_id(sequence_ids: torch.Tensor) -> torch.Tensor:
    """Index of each token among the tokens sharing its id (stable order)."""
    L = sequence_ids.shape[0]
    if L == 0:
        return torch.zeros(0, dtype=torch.long, device=sequence_ids.device)
    order = torch.sort(sequence_ids, stable=True).indices
    sid = sequence_ids[order]
    first = torch.ones(L, dtype=torch.bool, device=sequence_ids.device)
    first[1:] = sid[1:] != sid[:-1]
    idx = torch.arange(L, device=sequence_ids.device)
    group_start = torch.cummax(torch.where(first, idx, torch.zeros_like(idx)), 0).values
    rank = torch.empty(L, dtype=torch.long, device=sequence_ids.device)
    rank[order] = idx - group_start
    return rank


def flat_to_batched_left_pad(embeds: torch.Tensor, sequence_ids: torch.Tensor, prediction_indices: torch.Tensor,
                             B: int, S: int, step_counts):
    """Scatter flat ``[L, D]`` embeds into right-padded ``[B, Lmax, D]`` rows.

    Returns ``(out, token_lengths, local_indices)``: ``token_lengths[b]`` is
    the number of tokens with id ``b`` (a Python list, as in the reference),
    and ``local_indices[b, S - n + s]`` the in-row index of row ``b``'s
    ``s``-th prediction token (``n = step_counts[b]``).
    """
    if embeds.is_cuda:
        return _flat_to_batched_left_pad_cuda(embeds, sequence_ids, prediction_indices, B, S, step_counts)
    L, D = embeds.shape
    dev = embeds.device
    seq = sequence_ids.to(dev).long()
    counts = torch.bincount(seq[(seq >= 0) & (seq < B)], minlength=B)[:B] if L else torch.zeros(B, dtype=torch.long)
    token_lengths = [int(c) for c in counts.tolist()]
    lmax = max(token_lengths) if token_lengths else 0
    sel = (seq >= 0) & (seq < B)
    # tokens of rows outside 0..B-1 have no in-row index (-1, as in the reference)
    rank = torch.where(sel, _rank_within_id(seq), torch.full_like(seq, -1))
    out = embeds.new_zeros(B, lmax, D)
    out[seq[sel], rank[sel]] = embeds[sel]
    steps = [int(step_counts[b]) if b < len(step_counts) else S for b in range(B)]
    local = torch.zeros(B, S, dtype=torch.long, device=dev)
    total = sum(steps)
    if total:
        n = torch.tensor(steps, dtype=torch.long, device=dev)
        rows = torch.repeat_interleave(torch.arange(B, device=dev), n)
        within = torch.arange(total, device=dev) - torch.repeat_interleave(torch.cumsum(n, 0) - n, n)
        cols = S - n[rows] + within
        local[rows, cols] = rank[prediction_indices[:total].to(dev).long()]
    return out, token_lengths, local


def _left_align_content_cuda(embeds: torch.Tensor, prediction_indices: torch.Tensor):
    """K9 ``mb_left_align``: one pass over the rows, no host sync."""
    from mouse_core_b200 import kernels as K

    if prediction_indices.dim() != 2 or prediction_indices.shape[1] == 0:
        raise IndexError("prediction_indices needs at least one column (its last column gives the row length)")
    if embeds.shape[0] != prediction_indices.shape[0]:
        raise ValueError("embeds and prediction_indices disagree on the batch size")
    pi = prediction_indices.to(embeds.device, torch.long).contiguous()
    aligned, idx = K.left_align(embeds.contiguous(), pi)
    return aligned, idx.to(prediction_indices.dtype)


def _flat_to_batched_left_pad_cuda(embeds, sequence_ids, prediction_indices, B, S, step_counts):
    """K9 ``mb_flat_rank`` + ``mb_flat_scatter``: ranks, counts and local
    indices in one kernel, one read-back of the counts (the result's row
    width and ``token_lengths`` are host values), then one scatter."""
    from mouse_core_b200 import kernels as K

    L, D = embeds.shape
    dev = embeds.device
    B, S = int(B), int(S)
    steps = np.full(B, S, dtype=np.int64)
    k = min(len(step_counts), B)
    if k:
        steps[:k] = np.asarray(list(step_counts[:k]), dtype=np.int64)
    offs = np.cumsum(steps) - steps
    host = torch.from_numpy(np.stack([steps, offs]).astype(np.int32))
    meta = host.to(dev, non_blocking=False)
    seq = sequence_ids.to(dev, torch.long).reshape(-1).contiguous()
    pred = prediction_indices.to(dev, torch.long).reshape(-1).contiguous()
    rank, stats, local = K.flat_rank(seq, pred, meta, B, S)
    st = stats.cpu().numpy()
    if st[B + 1]:
        raise IndexError("a prediction index is out of range for the flat tokens")
    token_lengths = [int(c) for c in st[:B]]
    out = K.flat_scatter(embeds.contiguous(), seq, rank, B, int(st[B]) if B else 0)
    return out, token_lengths, local


def flat_sequence_position_ids(sequence_ids: torch.Tensor) -> torch.Tensor:
    """RoPE positions ``[1, L]`` restarting at 0 at every run boundary
    (``sequence_ids[i] != sequence_ids[i-1]``)."""
    L = sequence_ids.shape[0]
    dev = sequence_ids.device
    if L == 0:
        return torch.zeros(1, 0, dtype=torch.long, device=dev)
    idx = torch.arange(L, device=dev)
    boundary = torch.ones(L, dtype=torch.bool, device=dev)
    boundary[1:] = sequence_ids[1:] != sequence_ids[:-1]
    run_start = torch.cummax(torch.where(boundary, idx, torch.zeros_like(idx)), 0).values
    return (idx - run_start).unsqueeze(0)


def flat_sequence_causal_mask(*, sequence_ids: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """Additive ``[1, 1, L, L]`` mask: 0 where ``kv <= q`` and ids match,
    ``finfo(dtype).min`` elsewhere (the CPU SDPA path's dense mask)."""
    L = sequence_ids.shape[0]
    idx = torch.arange(L, device=sequence_ids.device)
    allow = (idx[None, :] <= idx[:, None]) & (sequence_ids[:, None] == sequence_ids[None, :])
    out = torch.full((L, L), torch.finfo(dtype).min, dtype=dtype, device=sequence_ids.device)
    out.masked_fill_(allow, 0.0)
    return out.view(1, 1, L, L)


# ---------------------------------------------------------------------------
# Loader-side packing of training windows into fixed-length rows.
# ---------------------------------------------------------------------------

def pack_windows(lengths, row_len: int):
    """Assign windows of ``lengths[w]`` tokens to rows of at most ``row_len``
    tokens, first fit in decreasing length order (windows stay whole).

    The reference's loader puts a whole batch of windows into ONE flat stream
    (data/dataloader.py:314-339); the packed kernels work best on rows of a
    fixed token budget (stable shapes for the attention work lists and the
    activations). Returns ``(row [W], offset [W], row_tokens [R])``: window
    ``w`` occupies tokens ``offset[w] .. offset[w] + lengths[w]`` of row
    ``row[w]``; inside a row windows keep their original relative order.
    """
    lengths = np.asarray(lengths, dtype=np.int64).reshape(-1)
    if (lengths < 0).any():
        raise ValueError("window lengths must be >= 0")
    if lengths.size and int(lengths.max()) > row_len:
        raise ValueError(f"a window of {int(lengths.max())} tokens does not fit a row of {row_len}")
    order = np.argsort(-lengths, kind="stable")
    row = np.zeros(lengths.size, dtype=np.int64)
    free: list[int] = []
    for w in order:
        n = int(lengths[w])
        for r, f in enumerate(free):
            if f >= n:
                row[w] = r
                free[r] = f - n
                break
        else:
            row[w] = len(free)
            free.append(row_len - n)
    offset = np.zeros(lengths.size, dtype=np.int64)
    row_tokens = np.zeros(len(free), dtype=np.int64)
    for w in range(lengths.size):  # original order inside each row
        offset[w] = row_tokens[row[w]]
        row_tokens[row[w]] += lengths[w]
    return row, offset, row_tokens


def pack_rows(windows, row_len: int):
    """Pack windows (dicts of equally long per-token arrays, e.g. token ids,
    actions, rewards, done codes, targets) into rows of at most ``row_len``
    tokens. Each row is a dict of the concatenated arrays plus
    ``sequence_ids`` (the window's index inside the row, so the segment mask
    keeps windows apart and positions restart per window), ``cu_seqlens``
    (int32 ``[windows in row + 1]``) and ``window_ids`` (the windows it holds,
    in order)."""
    if not windows:
        return []
    keys = list(windows[0].keys())
    lengths = np.array([len(next(iter(w.values()))) for w in windows], dtype=np.int64)
    for w in windows:
        if list(w.keys()) != keys or any(len(v) != len(next(iter(w.values()))) for v in w.values()):
            raise ValueError("every window must hold the same keys, each with one entry per token")
    row, _, _ = pack_windows(lengths, row_len)
    rows = []
    for r in range(int(row.max()) + 1):
        ids = np.flatnonzero(row == r)
        out = {k: np.concatenate([np.asarray(windows[w][k]) for w in ids]) for k in keys}
        seg = lengths[ids]
        out["sequence_ids"] = np.repeat(np.arange(ids.size, dtype=np.int64), seg)
        out["cu_seqlens"] = np.concatenate([[0], np.cumsum(seg)]).astype(np.int32)
        out["window_ids"] = ids
        rows.append(out)
    return rows
