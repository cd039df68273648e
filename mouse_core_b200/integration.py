"""Route an importable ``mouse_core`` (the reference package) through this one.

    import mouse_core_b200
    mouse_core_b200.install()          # after `import mouse_core`

Patches, in place and reversibly (``uninstall()``):

* ``Backbone.decode_session``  (mouse_core/models/backbone/base.py:61-73)
  -> returns ``PagedDecodeSession`` (``Model.forward`` at base.py:932-934 and
  every ``Qwen3Backbone``/``LlamaBackbone`` pick it up);
* ``flex_train.flex_packed_forward`` (looked up by ``Model.forward`` at
  call time, base.py:953-960) -> the sm_100a packed forward, once available;
* ``packing.left_align_content`` and ``base._flat_to_batched_left_pad``
  (base.py:924-937) -> the loop-free versions in ``mouse_core_b200.packing``;
* ``kv_policy`` functions -> the same-semantics versions here.
"""

from __future__ import annotations

import importlib

_saved: list[tuple[object, str, object]] = []


def _patch(obj, name, value) -> None:
    _saved.append((obj, name, getattr(obj, name)))
    setattr(obj, name, value)


def install(mouse_core_module=None) -> None:
    """Patch ``mouse_core`` so its hot path runs on these kernels."""
    if _saved:
        return
    mc = mouse_core_module or importlib.import_module("mouse_core")
    del mc
    base_bb = importlib.import_module("mouse_core.models.backbone.base")
    packing = importlib.import_module("mouse_core.models.embedding.packing")
    base = importlib.import_module("mouse_core.models.base")
    kvp = importlib.import_module("mouse_core.models.kv_policy")

    from mouse_core_b200 import kv_policy as my_kvp
    from mouse_core_b200 import packing as my_packing
    from mouse_core_b200.decode import PagedDecodeSession

    def decode_session(self, batch_size: int, capacity: int):
        model = getattr(self, "model", None)
        if model is None:
            raise NotImplementedError(f"{type(self).__name__} does not support cached decoding.")
        return PagedDecodeSession(model, batch_size=batch_size, capacity=capacity)

    _patch(base_bb.Backbone, "decode_session", decode_session)
    _patch(packing, "left_align_content", my_packing.left_align_content)
    _patch(base, "_flat_to_batched_left_pad", my_packing.flat_to_batched_left_pad)
    for fn in ("resolve_cache_bounds", "rebuild_starts", "cache_needs_rebuild"):
        _patch(kvp, fn, getattr(my_kvp, fn))
    try:
        from mouse_core_b200.packed import flex_packed_forward
    except ImportError:
        flex_packed_forward = None
    if flex_packed_forward is not None:
        flex_train = importlib.import_module("mouse_core.models.backbone.flex_train")
        _patch(flex_train, "flex_packed_forward", flex_packed_forward)
    try:
        embedding = importlib.import_module("mouse_core.models.embedding.embedding")
    except ImportError:
        embedding = None
    if embedding is not None and hasattr(embedding, "NumericEmbedder"):
        from mouse_core_b200.encoder import fused_forward

        cls = embedding.NumericEmbedder
        reference_forward = cls.forward

        def forward(self, token_batch):
            # CUDA embedders take the one-kernel path; a CPU embedder is the
            # caller's own CPU model and keeps the reference's code.
            try:
                on_cuda = next(self.parameters()).device.type == "cuda"
            except StopIteration:
                on_cuda = self.fourier.freqs.device.type == "cuda"
            return fused_forward(self, token_batch) if on_cuda else reference_forward(self, token_batch)

        _patch(cls, "forward", forward)


def uninstall() -> None:
    """Undo ``install()``."""
    while _saved:
        obj, name, old = _saved.pop()
        setattr(obj, name, old)
