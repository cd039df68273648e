"""Token embedding of a flat TokenBatch: one pinned upload, one kernel.

Reference: ``NumericEmbedder.forward`` (src/mouse_core/models/embedding/
embedding.py:293-326) first copies the TokenBatch's arrays to the device one
by one (``TokenBatch.to_tensors``, token_batch.py:116-143), then makes one
masked gather per embedding table and one masked static-Fourier pass per
Fourier modality (encoding.py:67-86). Here the token arrays travel in one
host-to-device copy from a pinned staging buffer, and K11
(``mb_embed_tokens``) writes every token's row in one pass over the stream:
a table row copy or its Fourier features (fp32, rounded once to the output
dtype), zero for types with neither.

``embedder`` is the reference's ``NumericEmbedder`` or any module with the
same layout: ``_meta`` (entries with ``type_id`` and ``kind`` in
``discrete / fourier / learnable / image``), ``_tables`` (``str(type_id)`` ->
``nn.Embedding``), ``fourier`` (buffers ``freqs``, ``phases``,
``output_scale``) and ``hidden_dim``. ``install()`` routes the reference's
``NumericEmbedder.forward`` here for CUDA embedders.
"""

from __future__ import annotations

import numpy as np
import torch

from mouse_core_b200 import _lib

_KIND_CODE = {"discrete": 1, "learnable": 1, "image": 1, "fourier": 2}


class EmbedLayout:
    """Device-side description of an embedder's tables and Fourier banks,
    rebuilt when a table tensor is replaced (a new storage pointer)."""

    def __init__(self, embedder, device: torch.device, dtype: torch.dtype):
        self.device, self.dtype = device, dtype
        metas = list(embedder._meta)
        n_types = max((int(m.type_id) for m in metas), default=-1) + 1
        kinds = np.zeros(n_types, dtype=np.int32)
        vocab = np.zeros(n_types, dtype=np.int32)
        self.tables: list[torch.Tensor | None] = [None] * n_types
        for m in metas:
            t = int(m.type_id)
            kinds[t] = _KIND_CODE.get(str(m.kind), 0)
            if kinds[t] == 1:
                w = embedder._tables[str(t)].weight
                if w.device != device or w.dtype != dtype or not w.is_contiguous():
                    w = w.detach().to(device=device, dtype=dtype).contiguous()
                self.tables[t] = w
                vocab[t] = w.shape[0]
        ptrs = np.array([0 if w is None else w.data_ptr() for w in self.tables], dtype=np.int64)
        self.kinds = torch.from_numpy(kinds).to(device)
        self.vocab = torch.from_numpy(vocab).to(device)
        self.ptrs = torch.from_numpy(ptrs).to(device)
        four = embedder.fourier
        self.freqs = four.freqs.detach().to(device=device, dtype=torch.float32).contiguous()
        self.phases = four.phases.detach().to(device=device, dtype=torch.float32).contiguous()
        self.scale = float(four.output_scale)
        self.n_types = n_types
        self.key = _layout_key(embedder)


def _layout_key(embedder):
    return tuple((k, t.weight.data_ptr(), t.weight._version) for k, t in sorted(embedder._tables.items()))


def embed_tokens(types: torch.Tensor, ids: torch.Tensor, scalars: torch.Tensor, layout: EmbedLayout,
                 hidden_dim: int) -> torch.Tensor:
    """K11 over device ``types``/``ids`` (int32 ``[L]``) and ``scalars``
    (f32 ``[L]``); returns ``embeds [L, hidden_dim]`` in the layout's dtype."""
    L = int(types.numel())
    out = torch.empty(L, hidden_dim, dtype=layout.dtype, device=layout.device)
    if L == 0:
        return out
    for name, t, dt in (("types", types, torch.int32), ("ids", ids, torch.int32), ("scalars", scalars, torch.float32)):
        if t.dtype != dt or t.device != layout.device or not t.is_contiguous() or t.numel() != L:
            raise ValueError(f"{name} must be a contiguous {dt} tensor of {L} entries on {layout.device}")
    stream = torch.cuda.current_stream(layout.device).cuda_stream
    _lib.call("mb_embed_tokens", types.data_ptr(), ids.data_ptr(), scalars.data_ptr(), L, hidden_dim,
              layout.kinds.data_ptr() if layout.n_types else None, layout.ptrs.data_ptr() if layout.n_types else None,
              layout.vocab.data_ptr() if layout.n_types else None, layout.n_types, layout.freqs.data_ptr(),
              layout.phases.data_ptr(), layout.freqs.shape[0], layout.scale, out.data_ptr(),
              int(layout.dtype == torch.float32), stream)
    from mouse_core_b200 import kernels as K

    K._count()
    return out


class TokenUploader:
    """The per-token arrays of a TokenBatch to the device in one copy: types,
    ids and scalars (int32 / f32 bit patterns) and the int64 sequence ids,
    step ids and prediction indices share one pinned staging buffer; the
    device views are sliced out of one fresh device buffer per call."""

    def __init__(self, device: torch.device):
        self.device = device
        self._host = torch.empty(0, dtype=torch.int32, pin_memory=True)
        self._event = None

    def __call__(self, tb) -> dict[str, torch.Tensor]:
        L = int(np.asarray(tb.token_types).shape[0])
        N = int(np.asarray(tb.prediction_indices).shape[0])
        o = 3 * L + (3 * L) % 2  # the int64 arrays start 8-byte aligned
        n32 = o + 2 * (2 * L + N)  # int64 arrays as pairs of int32
        if self._event is not None:
            self._event.synchronize()  # the previous copy has read the staging buffer
        if self._host.numel() < n32:
            self._host = torch.empty(max(n32, 2 * self._host.numel()), dtype=torch.int32, pin_memory=True)
        h = self._host.numpy()
        h[0:L] = tb.token_types
        h[L:2 * L] = tb.token_ids
        h[2 * L:3 * L] = np.asarray(tb.scalars, dtype=np.float32).view(np.int32)
        wide = h[o:o + 2 * (2 * L + N)].view(np.int64)
        wide[0:L] = tb.sequence_ids
        wide[L:2 * L] = tb.step_ids
        wide[2 * L:2 * L + N] = tb.prediction_indices
        d = torch.empty(n32, dtype=torch.int32, device=self.device)  # fresh: callers may keep the views
        d.copy_(self._host[:n32], non_blocking=True)
        if self._event is None:
            self._event = torch.cuda.Event()
        self._event.record()
        d64 = d[o:].view(torch.int64)
        return {"token_types": d[0:L], "token_ids": d[L:2 * L], "scalars": d[2 * L:3 * L].view(torch.float32),
                "sequence_ids": d64[0:L], "step_ids": d64[L:2 * L], "prediction_indices": d64[2 * L:2 * L + N]}


def fused_forward(embedder, token_batch):
    """``NumericEmbedder.forward`` for a CUDA embedder: ``(embeds [L, D],
    col_values, prediction_indices [N])`` with the same values, the token
    arrays uploaded once and the embedding one kernel."""
    if not hasattr(token_batch, "token_types"):
        token_batch = embedder.prepare(token_batch)
    try:
        p0 = next(embedder.parameters())
        device, dtype = p0.device, p0.dtype
    except StopIteration:
        device, dtype = embedder.fourier.freqs.device, embedder.fourier.freqs.dtype
    if device.type != "cuda":
        raise RuntimeError("the fused embedding runs on a CUDA device (B200, sm_100a) only")
    state = embedder.__dict__.setdefault("_mb_embed_state", {})
    layout = state.get("layout")
    if layout is None or layout.key != _layout_key(embedder) or layout.dtype != dtype:
        layout = state["layout"] = EmbedLayout(embedder, device, dtype)
    up = state.get("uploader")
    if up is None:
        up = state["uploader"] = TokenUploader(device)
    t = up(token_batch)
    embeds = embed_tokens(t["token_types"], t["token_ids"], t["scalars"], layout, int(embedder.hidden_dim))
    col_values = {}
    for k, v in token_batch.col_values.items():
        arr = np.asarray(v)
        src = torch.from_numpy(arr.astype(np.float32 if np.issubdtype(arr.dtype, np.floating) else np.int64))
        col_values[k] = src.to(device, non_blocking=False)
    return embeds, col_values, t["prediction_indices"]
