"""Grow-then-rebuild KV cache policy (same API and semantics as the reference).

Reference: src/mouse_core/models/kv_policy.py:14-72. A cached segment grows
from a ``start_cache`` prefill until appending would exceed ``max_cache``; then
the caller rebuilds by prefilling the latest ``start_cache`` steps. These are
host-side integer decisions over ``[B]`` arrays and stay in numpy; the results
are bit-exact with the reference (checked against fixtures it produced).

``rows_needing_rebuild`` is an addition for paged sessions: a paged cache can
rebuild only the rows that overflowed (``PagedDecodeSession.reset_rows`` +
a ragged prefill of those rows), where the reference must rebuild the batch.
"""

from __future__ import annotations

import numpy as np


def resolve_cache_bounds(max_cache: int, start_cache: int | None = None) -> tuple[int, int]:
    """``(max_cache, start_cache)``; ``start_cache`` defaults to
    ``max_cache // 2`` (at least 1) and is clamped to ``max(1, max_cache - 1)``
    when not below ``max_cache`` (kv_policy.py:14-29)."""
    max_cache = max(1, int(max_cache))
    start_cache = max(1, max_cache // 2) if start_cache is None else max(1, int(start_cache))
    if start_cache >= max_cache:
        start_cache = max(1, max_cache - 1)
    return max_cache, start_cache


def rebuild_starts(*, ends: np.ndarray, context_start: np.ndarray | int, start_cache: int,
                   max_cache: int) -> np.ndarray:
    """Inclusive history index each row's rebuild prefill starts at:
    ``max(context_start, ends - min(start_cache, max_cache))`` (kv_policy.py:32-43)."""
    ends = np.asarray(ends, dtype=np.int64)
    ctx = np.asarray(context_start, dtype=np.int64)
    return np.maximum(ctx, ends - min(int(start_cache), int(max_cache)))


def cache_needs_rebuild(*, has_cache: bool, cached_starts: np.ndarray, cached_ends: np.ndarray, ends: np.ndarray,
                        context_start: np.ndarray, max_cache: int, batch_complete: bool) -> bool:
    """Whether the policy must prefill instead of appending (kv_policy.py:46-72):
    no cache, incomplete batch, shape change, a rewind, a cleared context, or a
    cached span that would exceed ``max_cache``."""
    if not has_cache or not batch_complete:
        return True
    ends = np.asarray(ends, dtype=np.int64)
    cached_starts = np.asarray(cached_starts, dtype=np.int64)
    cached_ends = np.asarray(cached_ends, dtype=np.int64)
    context_start = np.asarray(context_start, dtype=np.int64)
    if ends.shape != cached_starts.shape or ends.shape != cached_ends.shape:
        return True
    if np.any(ends < cached_ends):
        return True
    if np.any(context_start > cached_starts):
        return True
    return bool(np.any(ends - cached_starts > int(max_cache)))


def rows_needing_rebuild(*, cached_starts: np.ndarray, cached_ends: np.ndarray, ends: np.ndarray,
                         context_start: np.ndarray, max_cache: int) -> np.ndarray:
    """Per-row form of ``cache_needs_rebuild`` for a same-shape batch: boolean
    ``[B]`` marking rows that rewound, lost context or would exceed ``max_cache``."""
    ends = np.asarray(ends, dtype=np.int64)
    cs = np.asarray(cached_starts, dtype=np.int64)
    ce = np.asarray(cached_ends, dtype=np.int64)
    ctx = np.broadcast_to(np.asarray(context_start, dtype=np.int64), ends.shape)
    return (ends < ce) | (ctx > cs) | (ends - cs > int(max_cache))
