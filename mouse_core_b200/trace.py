"""NVTX ranges around the hot path's host calls.

The reference has no tracing. Here the decode step, the in-session prefill,
the packed attention forward and backward and the gradient all-reduce each
push a named NVTX range (``mouse_b200/<name>``), so an Nsight Systems or
Nsight Compute timeline shows where a step's kernels come from. With no tool
attached a range costs a call into the NVTX stub (well under a microsecond);
set ``MOUSE_B200_NVTX=0`` to skip even that.
"""

from __future__ import annotations

import contextlib
import os

ENABLED = os.environ.get("MOUSE_B200_NVTX", "1") != "0"

try:
    from torch.cuda import nvtx as _nvtx
except Exception:  # pragma: no cover - torch without CUDA bindings
    _nvtx = None
    ENABLED = False


@contextlib.contextmanager
def nvtx_range(name: str):
    """``with nvtx_range("decode_step"): ...`` marks the enclosed host work."""
    if not ENABLED:
        yield
        return
    _nvtx.range_push("mouse_b200/" + name)
    try:
        yield
    finally:
        _nvtx.range_pop()
