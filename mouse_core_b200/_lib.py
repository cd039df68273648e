"""ctypes binding of ``libmouse_b200.so`` (the C ABI of ``include/mouse_b200.h``).

The library is loaded from this package directory only; if it is missing the
import of any op raises — there is no fallback implementation.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libmouse_b200.so")

_c_int, _c_float, _c_size, _c_ll = ctypes.c_int, ctypes.c_float, ctypes.c_size_t, ctypes.c_longlong
_vp = ctypes.c_void_p

# name -> (restype, argtypes), in the order of include/mouse_b200.h
PROTOTYPES = {
    "mb_last_error": (ctypes.c_char_p, []),
    "mb_version": (_c_int, []),
    "mb_device_status": (_c_int, [ctypes.POINTER(_c_int), _c_int]),
    "mb_set_wait_limit": (_c_int, [ctypes.c_longlong]),
    "mb_decode_workspace_bytes": (_c_size, [_c_int, _c_int, _c_int, _c_int, _c_int]),
    "mb_decode_plan": (_c_int, [_vp, _c_int, _c_int, _c_int, _c_int, _c_int, _vp, _c_size, _vp]),
    "mb_decode_plan_shared": (_c_int, [_vp, _vp, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _c_int, _vp,
                                       _c_size, _vp]),
    "mb_decode_attention": (_c_int, [_vp, _vp, _vp, _c_int, _vp, _c_int, _vp, _vp, _c_int, _c_int, _c_int,
                                     _c_int, _c_int, _c_int, _c_float, _c_int, _c_int, _vp, _vp, _c_size, _vp]),
    "mb_decode_attention_noalloc": (_c_int, [_vp, _vp, _vp, _c_int, _vp, _c_int, _vp, _vp, _c_int, _c_int,
                                             _c_int, _c_int, _c_int, _c_int, _c_float, _c_int, _vp, _vp]),
    "mb_kv_append": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _c_float, _vp, _c_float, _c_int, _c_int,
                              _c_int, _c_int, _c_ll, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_kv_append_f32": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _c_float, _vp, _c_float, _c_int,
                                  _c_int, _c_int, _c_int, _c_ll, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_rope_table": (_c_int, [_vp, _c_int, _vp, _c_int, _c_float, _vp, _vp]),
    "mb_qkv_append": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _c_float, _vp, _c_int, _c_int, _c_int,
                               _c_int, _c_ll, _vp, _vp, _vp, _vp]),
    "mb_page_copy": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_ll, _vp]),
    "mb_decode_step_meta": (_c_int, [_c_int, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_rmsnorm": (_c_int, [_vp, _vp, _vp, _c_float, _c_int, _c_int, _vp, _vp, _vp]),
    "mb_embed_tokens": (_c_int, [_vp, _vp, _vp, _c_ll, _c_int, _vp, _vp, _vp, _c_int, _vp, _vp, _c_int,
                                 _c_float, _vp, _c_int, _vp]),
    "mb_td_loss_scratch_bytes": (_c_size, [_c_int]),
    "mb_td_loss_fwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _vp, _c_float, _c_float, _vp,
                                _c_size, _vp, _vp]),
    "mb_td_loss_bwd": (_c_int, [_vp, _vp, _c_int, _c_int, _c_float, _vp, _c_size, _vp, _vp, _vp, _vp]),
    "mb_silu_mul": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "mb_rmsnorm_f32": (_c_int, [_vp, _vp, _vp, _vp, _c_float, _c_int, _c_int, _vp, _vp, _vp]),
    "mb_silu_mul_f32": (_c_int, [_vp, _c_int, _c_int, _vp, _vp]),
    "mb_varlen_attention_fwd": (_c_int, [_vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _c_float, _vp,
                                         _vp, _vp]),
    "mb_varlen_attention_bwd": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp, _vp,
                                         _c_float, _vp, _vp, _vp, _vp, _vp]),
    "mb_segment_meta": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_varlen_bwd_pair_offsets": (_c_int, [_vp, _c_int, _vp, _vp]),
    "mb_flat_rank": (_c_int, [_vp, _c_int, _c_int, _vp, _c_int, _vp, _vp, _c_int, _vp, _vp, _vp, _vp]),
    "mb_flat_scatter": (_c_int, [_vp, _c_int, _c_int, _vp, _vp, _c_int, _c_int, _vp, _vp]),
    "mb_left_align": (_c_int, [_vp, _c_int, _c_int, _c_int, _vp, _c_int, _vp, _vp, _vp]),
    "mb_varlen_attention_bwd_stored": (_c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _c_int, _c_int, _vp,
                                                _vp, _vp, _vp, _c_int, _c_float, _vp, _vp, _vp, _vp, _vp, _c_size,
                                                _vp]),
    "mb_rmsnorm_fwd": (_c_int, [_vp, _vp, _c_float, _c_int, _c_int, _vp, _vp, _vp]),
    "mb_add_rmsnorm_fwd": (_c_int, [_vp, _vp, _vp, _c_float, _c_int, _c_int, _vp, _vp, _vp, _vp]),
    "mb_rmsnorm_bwd_add": (_c_int, [_vp, _vp, _vp, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp]),
    "mb_rmsnorm_bwd_scratch_floats": (_c_size, [_c_int, _c_int]),
    "mb_rmsnorm_bwd": (_c_int, [_vp, _vp, _vp, _vp, _c_int, _c_int, _vp, _vp, _vp, _c_size, _vp]),
    "mb_qkv_heads_fwd": (_c_int, [_vp, _c_ll, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _c_float, _c_float,
                                  _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    "mb_qkv_heads_bwd_scratch_floats": (_c_size, [_c_int, _c_int]),
    "mb_qkv_heads_bwd": (_c_int, [_vp, _vp, _vp, _vp, _c_ll, _c_int, _c_int, _c_int, _c_int, _vp, _vp, _vp, _vp,
                                  _vp, _vp, _vp, _c_ll, _vp, _vp, _vp, _c_size, _vp]),
    "mb_silu_mul_bwd": (_c_int, [_vp, _vp, _c_int, _c_int, _vp, _vp]),
}

_LIB = None


class KernelError(RuntimeError):
    """A C-ABI call of libmouse_b200 returned a non-zero status."""


def load():
    """Load the library (once) and attach prototypes."""
    global _LIB
    if _LIB is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built; run `python -m mouse_core_b200.build` (nvcc, sm_100a)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in PROTOTYPES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _LIB = lib
    return _LIB


def check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load().mb_last_error().decode(errors="replace")
        raise KernelError(f"{what} failed (status {rc}): {msg}")


def call(name: str, *args):
    """Call ``name`` and raise ``KernelError`` on a non-zero status."""
    fn = getattr(load(), name)
    rc = fn(*args)
    check(rc, name)


def device_status(clear: bool = True) -> int:
    """Device status word of the kernels (0 = healthy); synchronizes."""
    out = ctypes.c_int(0)
    check(load().mb_device_status(ctypes.byref(out), int(clear)), "mb_device_status")
    return out.value


def set_wait_limit(cycles: int | None) -> None:
    """Cycles every bounded wait of the kernels spins before it gives up
    (``None`` restores the default of about two seconds); synchronizes."""
    check(load().mb_set_wait_limit(-1 if cycles is None else int(cycles)), "mb_set_wait_limit")
