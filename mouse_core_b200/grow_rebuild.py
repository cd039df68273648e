"""Grow-then-rebuild cached decoding on a paged session.

Reference: the grow-then-rebuild policy itself is three host functions
(src/mouse_core/models/kv_policy.py:14-72); what applies it is the caller's
loop, ``_act_from_contexts`` inside ``run_eval``
(examples/02_train_offline.ipynb, cell 11). On every call that loop either
appends each row's new steps to the cached segment, or — when
``cache_needs_rebuild`` says so (no cache yet, a rewound or cleared context,
a cached span that would exceed ``max_cache``) or when a task ended — drops
the session and prefills every row's latest ``start_cache`` steps
(``rebuild_starts``); ``Model.forward`` makes the new session at
models/base.py:932-934.

``GrowRebuildDecoder`` is that loop on a ``PagedDecodeSession``:

* ``per_row=False`` keeps the reference's batch semantics exactly: any rebuild
  re-windows every row. Dropping the session becomes emptying every row of
  the same paged session (its pages return to the pool; nothing is
  reallocated), which decodes identically because a row never reads a slot
  it has not written since it was emptied.
* ``per_row=True`` re-windows only the rows that need it
  (``rows_needing_rebuild``): the others keep appending. Every row then
  decodes exactly as the reference's loop would on a batch holding that env
  alone, and one env's overflow or task end no longer costs a prefill of the
  whole batch.

A rebuilt row and the appended rows of the same call go through ONE ragged
``forward`` (the rebuilt rows are emptied first, then receive their window as
a left-padded chunk), so a call is one pass over the layer stack whatever
mix of appends and rebuilds it holds. Steps are tokens here (one token per
step, as in the decode benchmark's transition tokens).
"""

from __future__ import annotations

from typing import Callable

import numpy as np
import torch

from mouse_core_b200.kv_policy import cache_needs_rebuild, rebuild_starts, resolve_cache_bounds, rows_needing_rebuild


class GrowRebuildDecoder:
    """Cached decoding of ``batch_size`` env streams under the grow-then-rebuild policy.

    Args:
        backbone: A backbone with ``decode_session`` (``Qwen3Backbone`` /
            ``LlamaBackbone``), bf16 on a CUDA device.
        batch_size: Number of env streams.
        embed: Maps a device int32 tensor of token ids to their embeddings
            (``[..., D]``, the backbone's dtype), e.g. an ``nn.Embedding``.
        max_cache / start_cache: Policy bounds, resolved by
            ``resolve_cache_bounds`` (kv_policy.py:14-29).
        per_row: Rebuild only the rows that need it (see the module docstring).
        page_size / num_pages: Passed to the session.
    """

    def __init__(self, backbone, batch_size: int, embed: Callable[[torch.Tensor], torch.Tensor], *, max_cache: int,
                 start_cache: int | None = None, per_row: bool = False, page_size: int = 128,
                 num_pages: int | None = None) -> None:
        self.backbone = backbone
        self.B = int(batch_size)
        self.embed = embed
        self.max_cache, self.start_cache = resolve_cache_bounds(max_cache, start_cache)
        self.per_row = bool(per_row)
        self.page_size = int(page_size)
        self.num_pages = num_pages
        self.session = None
        self.cached_starts = np.zeros(self.B, dtype=np.int64)
        self.cached_ends = np.zeros(self.B, dtype=np.int64)
        self.device = next(backbone.parameters()).device
        self._ids_host = torch.empty(0, dtype=torch.int32, pin_memory=True)
        self._ids_event = None
        # Counters for callers and tests: calls that rebuilt, rows rebuilt.
        self.rebuild_calls = 0
        self.rows_rebuilt = 0

    def adopt(self, session, cached_starts, cached_ends) -> None:
        """Continue from an existing session whose row ``b`` caches steps
        ``cached_starts[b]:cached_ends[b]`` of its context (for instance one
        a caller prefilled itself)."""
        if session.B != self.B:
            raise ValueError(f"session has batch_size {session.B}, expected {self.B}")
        self.session = session
        self.cached_starts = np.array(cached_starts, dtype=np.int64).reshape(self.B)
        self.cached_ends = np.array(cached_ends, dtype=np.int64).reshape(self.B)

    def _new_session(self):
        return self.backbone.decode_session(batch_size=self.B, capacity=self.max_cache, page_size=self.page_size,
                                            num_pages=self.num_pages)

    def rows_to_rebuild(self, ends: np.ndarray, context_start: np.ndarray, rebuild=False) -> np.ndarray:
        """Rows whose cached segment this call replaces by a fresh window.

        ``rebuild`` is ``True`` (every row), ``False``, or the rows whose task
        ended since the last call (a ``[B]`` boolean mask or row indices): in
        batch mode any of them rebuilds the batch, as the reference's loop
        does; per row, only they (and the rows the policy flags) rebuild."""
        everything = np.arange(self.B)
        forced = np.zeros(self.B, dtype=bool)
        if rebuild is True:
            forced[:] = True
        elif rebuild is not False and rebuild is not None:
            r = np.asarray(rebuild)
            if r.dtype == bool:
                if r.shape != (self.B,):
                    raise ValueError(f"a rebuild mask must have shape [{self.B}]")
                forced |= r
            else:
                forced[r.astype(np.int64).reshape(-1)] = True
        if self.session is None or (forced.any() and not self.per_row):
            return everything
        if self.per_row:
            flagged = rows_needing_rebuild(cached_starts=self.cached_starts, cached_ends=self.cached_ends, ends=ends,
                                           context_start=context_start, max_cache=self.max_cache)
            return np.flatnonzero(flagged | forced)
        if cache_needs_rebuild(has_cache=True, cached_starts=self.cached_starts, cached_ends=self.cached_ends,
                               ends=ends, context_start=context_start, max_cache=self.max_cache,
                               batch_complete=True):
            return everything
        return everything[:0]

    def _stage_ids(self, ids: np.ndarray) -> torch.Tensor:
        """Token ids to the device through a pinned buffer that no copy in
        flight still reads."""
        n = ids.size
        if self._ids_event is not None:
            self._ids_event.synchronize()
        if self._ids_host.numel() < n:
            self._ids_host = torch.empty(max(n, 2 * self._ids_host.numel()), dtype=torch.int32, pin_memory=True)
        host = self._ids_host[:n]
        host.numpy()[:] = ids.reshape(-1)
        dev = host.to(self.device, non_blocking=True)
        if self._ids_event is None:
            self._ids_event = torch.cuda.Event()
        self._ids_event.record()
        return dev.view(ids.shape)

    @torch.no_grad()
    def step(self, history: np.ndarray, ends, context_start=0, *, rebuild=False, head=None,
             output_hidden_states: bool = False):
        """Run one call of the caller loop.

        Args:
            history: ``[B, T]`` integer token ids; row ``b``'s context is
                ``history[b, :ends[b]]`` (``T`` must cover every ``ends[b]``).
            ends: ``[B]`` context lengths now (steps taken so far).
            context_start: Scalar or ``[B]``: first step of each row's current
                context (steps before it are never attended to).
            rebuild: ``True`` forces a rebuild of every row (the reference
                passes it when a task ended); a ``[B]`` mask or row indices
                name the rows whose task ended (see ``rows_to_rebuild``).
            head: Optional ``head(h [B, D]) -> tensor`` applied to each row's
                latest hidden state (e.g. the action head and its argmax);
                one-token calls then run gather, layers and head as one CUDA
                graph (``PagedDecodeSession.decode_step``) and return
                ``(head output, fed)`` — a graph buffer, valid until the next
                call.

        Returns:
            ``(h, fed)``: the session output ``[B, S, D]`` (left-padded: row
            ``b``'s ``fed[b]`` new tokens are its last columns, so ``h[:, -1]``
            is each fed row's latest hidden state) and ``fed [B]``, the tokens
            each row received (0 for a row with nothing new or an emptied
            context). With ``output_hidden_states`` the session's per-layer
            tuple is returned as a third element.
        """
        B = self.B
        hist = np.asarray(history)
        ends = np.asarray(ends, dtype=np.int64).reshape(-1)
        if ends.shape[0] != B or hist.ndim != 2 or hist.shape[0] != B:
            raise ValueError(f"history must be [B={B}, T] and ends [B={B}]")
        if (ends < 0).any() or (B and int(ends.max()) > hist.shape[1]):
            raise ValueError("ends must lie in [0, history.shape[1]]")
        ctx = np.broadcast_to(np.asarray(context_start, dtype=np.int64), (B,))
        rows = self.rows_to_rebuild(ends, ctx, rebuild)
        starts = self.cached_ends.copy()
        if rows.size:
            if self.session is None:
                self.session = self._new_session()
            else:
                self.session.reset_rows(rows)
            new = rebuild_starts(ends=ends[rows], context_start=ctx[rows], start_cache=self.start_cache,
                                 max_cache=self.max_cache)
            starts[rows] = new
            self.cached_starts[rows] = new
            self.rebuild_calls += 1
            self.rows_rebuilt += int(rows.size)
        fed = np.maximum(ends - starts, 0)
        S = max(int(fed.max()) if B else 0, 1)
        if S == 1:
            ids = hist[np.arange(B), np.maximum(ends - 1, 0)][:, None]
        else:
            col = np.arange(S, dtype=np.int64)[None, :]
            src = starts[:, None] + col - (S - fed)[:, None]  # left-padded: real tokens are the last fed[b]
            ids = hist[np.arange(B)[:, None], np.clip(src, 0, max(hist.shape[1] - 1, 0))]
        ids_dev = self._stage_ids(np.ascontiguousarray(ids, dtype=np.int32))
        if head is not None and not output_hidden_states:
            if S == 1:  # gather + layers + head as one graph replay
                out = self.session.decode_step(ids_dev[:, 0], fed, self.embed, head)
            else:
                out = head(self.session.forward(embeds=self.embed(ids_dev), lengths=fed)[:, -1])
            self.cached_ends = ends.copy()
            return out, fed
        out = self.session.forward(embeds=self.embed(ids_dev), lengths=fed, output_hidden_states=output_hidden_states)
        self.cached_ends = ends.copy()
        if output_hidden_states:
            h, hiddens = out
            return h, fed, hiddens
        return out, fed
