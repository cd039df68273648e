"""The C-ABI library builds for sm_100a, loads, and exports exactly what
include/mouse_b200.h declares (no GPU needed: only argument-validation paths
that return before any CUDA call are exercised)."""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from mouse_core_b200 import _lib, build

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "mouse_b200.h")


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(mb_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_header_declares_entry_points():
    names = declared_functions()
    assert "mb_decode_attention" in names and "mb_kv_append" in names
    assert set(names) == set(_lib.PROTOTYPES), "ctypes prototypes and header disagree"


def test_library_exports_every_declared_symbol(lib):
    raw = ctypes.CDLL(build.LIB)
    for name in declared_functions():
        assert hasattr(raw, name), f"{name} declared in mouse_b200.h but not exported"


def test_version_and_error_text(lib):
    assert lib.mb_version() == 100
    # head_dim 96 is rejected before any CUDA call
    rc = lib.mb_decode_attention(None, None, None, 1, None, 1, None, None, 1, 1, 2, 1, 96, 64, 1.0, 1, 0,
                                 None, None, 0, None)
    assert rc == 2  # MB_ERR_UNSUPPORTED
    assert b"head_dim" in lib.mb_last_error()
    rc = lib.mb_decode_attention(None, None, None, 1, None, 1, None, None, 1, 1, 3, 2, 64, 64, 1.0, 1, 0,
                                 None, None, 0, None)
    assert rc == 1 and b"multiple" in lib.mb_last_error()
    rc = lib.mb_kv_append(None, 4, 8, None, None, None, None, 1e-6, None, 1.0, 1, 1, 64, 0, 0, None, None, None,
                          None, None, None)
    assert rc == 1


def test_workspace_size_rules(lib):
    small = lib.mb_decode_workspace_bytes(256, 8, 2, 128, 4096)
    big = lib.mb_decode_workspace_bytes(256, 8, 2, 128, 8192)
    assert 0 < small < big
    assert lib.mb_decode_workspace_bytes(256, 8, 17, 128, 4096) == 0  # block mode needs none
    assert lib.mb_decode_workspace_bytes(256, 8, 2, 96, 4096) == 0


def test_zero_sized_calls_are_noops(lib):
    assert lib.mb_kv_append(None, 0, 0, None, None, None, None, 0.0, None, 1.0, 1, 1, 64, 0, 0, None, None, None,
                            None, None, None) == 0
    assert lib.mb_page_copy(None, None, None, None, 0, 8, None) == 0
    assert lib.mb_rmsnorm(None, None, None, 1e-6, 0, 8, None, None, None) == 0


def test_training_elementwise_argument_rules(lib):
    # dim must be a multiple of 256 (<= 2048); rejected before any CUDA call
    assert lib.mb_rmsnorm_fwd(None, None, 1e-6, 4, 1000, None, None, None) == 2
    assert b"256" in lib.mb_last_error()
    assert lib.mb_rmsnorm_fwd(None, None, 1e-6, 4, 4096, None, None, None) == 2
    assert lib.mb_rmsnorm_fwd(None, None, 1e-6, 0, 1024, None, None, None) == 0
    assert lib.mb_rmsnorm_fwd(None, None, 1e-6, 4, 1024, None, None, None) == 1
    # scratch sizing: one row of dim floats per reduction block
    n = lib.mb_rmsnorm_bwd_scratch_floats(32768, 1024)
    assert n > 0 and n % 1024 == 0
    assert lib.mb_rmsnorm_bwd_scratch_floats(0, 1024) == 0
    assert lib.mb_rmsnorm_bwd(None, None, None, None, 8, 1024, None, ctypes.c_void_p(16), ctypes.c_void_p(16),
                              1, None) == 1
    assert b"NULL" in lib.mb_last_error()
    # fused QKV heads: head_dim 64/128 only, norm weights in pairs, strides checked
    assert lib.mb_qkv_heads_fwd(None, 96 * 8, 4, 4, 2, 96, None, None, 1e-6, 1e-6, None, None, None, None, None,
                                None, None, None) == 2
    assert lib.mb_qkv_heads_fwd(None, 1024, 0, 4, 2, 128, None, None, 1e-6, 1e-6, None, None, None, None, None,
                                None, None, None) == 0
    assert lib.mb_qkv_heads_fwd(None, 1024, 4, 4, 2, 128, ctypes.c_void_p(16), None, 1e-6, 1e-6, None, None, None,
                                None, None, None, None, None) == 1
    assert b"both" in lib.mb_last_error()
    assert lib.mb_qkv_heads_bwd_scratch_floats(16384, 128) % 256 == 0
    assert lib.mb_qkv_heads_bwd_scratch_floats(16384, 96) == 0
    assert lib.mb_qkv_heads_bwd(None, None, None, None, 1024, 4, 4, 2, 128, ctypes.c_void_p(16),
                                ctypes.c_void_p(16), None, None, None, None, None, 1024, None, None, None, 0,
                                None) == 1
    assert b"dweight" in lib.mb_last_error()
    # SiLU-gated product backward
    assert lib.mb_silu_mul_bwd(None, None, 0, 3072, None, None) == 0
    assert lib.mb_silu_mul_bwd(None, None, 4, 3071, None, None) == 1


def test_stored_ds_backward_argument_rules(lib):
    p = ctypes.c_void_p(4096)  # aligned, never dereferenced: every call below returns before any CUDA call
    args = [p, p, p, p, p, p, 1000, 4, 2, 128, p, p, p, p]

    def call(n_pairs, ds, ds_bytes, L=1000):
        a = list(args)
        a[6] = L
        return lib.mb_varlen_attention_bwd_stored(*a, n_pairs, 0.1, p, p, p, p, ds, ds_bytes, None)

    assert call(8, p, 1 << 30, L=0) == 0
    assert call(8, None, 1 << 30) == 1 and b"ds_scratch" in lib.mb_last_error()
    assert call(7, p, 1 << 30) == 1 and b"n_pairs" in lib.mb_last_error()  # fewer pairs than query tiles
    assert call(36, p, 4 * 36 * 32768 - 1) == 3 and b"MB_VARLEN_BWD_DS_BYTES" in lib.mb_last_error()
    a = list(args)
    a[12] = None  # tile_lo
    assert lib.mb_varlen_attention_bwd_stored(*a, 36, 0.1, p, p, p, p, p, 1 << 30, None) == 1
    assert lib.mb_varlen_bwd_pair_offsets(None, -1, p, None) == 1
    assert lib.mb_varlen_bwd_pair_offsets(None, 5, p, None) == 1


def test_glue_argument_rules(lib):
    p = ctypes.c_void_p(4096)
    assert lib.mb_flat_rank(p, 4, 49153, p, 1, p, p, 1, p, p, p, None) == 2  # batch above the shared counters
    assert lib.mb_flat_rank(p, -1, 4, p, 1, p, p, 1, p, p, p, None) == 1
    assert lib.mb_flat_rank(p, 4, 2, None, 3, p, p, 1, p, p, p, None) == 1 and b"NULL" in lib.mb_last_error()
    assert lib.mb_flat_scatter(p, 4, 0, p, p, 2, 2, p, None) == 1
    assert lib.mb_flat_scatter(None, 0, 16, None, None, 0, 0, None, None) == 0  # nothing to write
    assert lib.mb_left_align(p, 2, 3, 16, p, 0, p, p, None) == 1  # needs a last index column
    assert lib.mb_left_align(None, 0, 3, 16, None, 1, None, None, None) == 0


def test_add_rmsnorm_argument_rules(lib):
    p = ctypes.c_void_p(4096)
    assert lib.mb_add_rmsnorm_fwd(p, p, p, 1e-6, 4, 1000, p, p, p, None) == 2  # width
    assert lib.mb_add_rmsnorm_fwd(p, None, p, 1e-6, 4, 1024, p, p, p, None) == 1
    assert lib.mb_add_rmsnorm_fwd(None, None, None, 1e-6, 0, 1024, None, None, None, None) == 0
    assert lib.mb_rmsnorm_bwd_add(p, p, p, p, None, 4, 1024, p, p, p, 1 << 20, None) == 1
    assert b"dsum" in lib.mb_last_error()


def test_qkv_append_argument_rules(lib):
    """K13 and its RoPE table reject bad shapes and pointers before any CUDA
    call; zero tokens is a no-op that needs no pointers."""
    p = ctypes.c_void_p(4096)  # aligned, never dereferenced
    odd = ctypes.c_void_p(4098)

    def qa(tokens=8, hidden=1024, hq=16, hkv=8, hd=128, x=p, w=p, rope=p, q=p, kp=None, vp=None, slot=None,
           page=0, pages=0):
        return lib.mb_qkv_append(x, tokens, hidden, w, None, rope, None, None, 1e-6, slot, hq, hkv, hd, page,
                                 pages, q, kp, vp, None)

    assert qa(tokens=0, x=None, w=None, rope=None, q=None) == 0
    assert qa(hd=96) == 2 and b"head_dim" in lib.mb_last_error()
    assert qa(hq=1, hkv=1, hd=64) == 2 and b"multiple of 128" in lib.mb_last_error()  # 3 heads of 64
    assert qa(hidden=1020) == 2 and b"hidden" in lib.mb_last_error()
    assert qa(hq=3, hkv=2) == 1 and b"multiple of kv_heads" in lib.mb_last_error()
    assert qa(rope=None) == 1 and b"NULL" in lib.mb_last_error()
    assert qa(x=odd) == 1 and b"aligned" in lib.mb_last_error()
    assert qa(kp=p, vp=p) == 1 and b"go together" in lib.mb_last_error()  # pools without slots
    assert qa(kp=p, vp=p, slot=p) == 1 and b"page_size" in lib.mb_last_error()
    assert lib.mb_rope_table(p, 4, p, 96, 1.0, p, None) == 2
    assert lib.mb_rope_table(p, 4, p, 128, 1.0, odd, None) == 1
    assert lib.mb_rope_table(None, 0, None, 128, 1.0, None, None) == 0
