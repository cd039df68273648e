"""mouse_core_b200 — B200-native (sm_100a) attention hot path of mouse-core.

Drop-in pieces for ``mouse_core.models``:

* ``PagedDecodeSession`` (alias ``FlexDecodeSession``) — cached batched
  decode over ragged env batches with a paged KV cache.
* ``GrowRebuildDecoder`` — the grow-then-rebuild caller loop on that session.
* ``flex_packed_forward`` — packed segment-causal training forward whose
  attention (and its backward) run on tcgen05 kernels.
* ``Qwen3Backbone`` / ``LlamaBackbone`` / ``IdentityBackbone`` /
  ``Backbone.decode_session`` — adapters whose decode sessions are paged.
* ``resolve_cache_bounds`` / ``rebuild_starts`` / ``cache_needs_rebuild`` —
  the grow-then-rebuild policy.
* ``left_align_content`` / ``flat_to_batched_left_pad`` /
  ``flat_sequence_position_ids`` / ``flat_sequence_causal_mask`` — packing.
* ``install()`` — patch an importable ``mouse_core`` to use all of the above.

Kernels live in ``libmouse_b200.so`` (C ABI: ``include/mouse_b200.h``),
built with ``python -m mouse_core_b200.build``.
"""

from mouse_core_b200.kv_policy import (
    cache_needs_rebuild,
    rebuild_starts,
    resolve_cache_bounds,
    rows_needing_rebuild,
)
from mouse_core_b200.packing import (
    flat_sequence_causal_mask,
    flat_sequence_position_ids,
    flat_to_batched_left_pad,
    left_align_content,
)

__all__ = [
    "PagedDecodeSession",
    "GrowRebuildDecoder",
    "FlexDecodeSession",
    "flex_packed_forward",
    "Backbone",
    "Qwen3Backbone",
    "LlamaBackbone",
    "IdentityBackbone",
    "cache_needs_rebuild",
    "rebuild_starts",
    "resolve_cache_bounds",
    "rows_needing_rebuild",
    "flat_sequence_causal_mask",
    "flat_sequence_position_ids",
    "flat_to_batched_left_pad",
    "left_align_content",
    "install",
]


def __getattr__(name):
    # Lazy: the session/backbone modules import torch + transformers.
    if name in ("PagedDecodeSession", "FlexDecodeSession"):
        from mouse_core_b200 import decode

        return getattr(decode, name)
    if name == "GrowRebuildDecoder":
        from mouse_core_b200.grow_rebuild import GrowRebuildDecoder

        return GrowRebuildDecoder
    if name == "flex_packed_forward":
        from mouse_core_b200.packed import flex_packed_forward

        return flex_packed_forward
    if name in ("Backbone", "Qwen3Backbone", "LlamaBackbone", "IdentityBackbone"):
        from mouse_core_b200 import backbone

        return getattr(backbone, name)
    if name == "install":
        from mouse_core_b200.integration import install

        return install
    raise AttributeError(name)
