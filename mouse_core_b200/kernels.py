"""Torch-facing wrappers of the C ABI: check devices, dtypes and layouts, then
pass raw pointers and torch's current CUDA stream to ``libmouse_b200.so``.

Every function raises ``TypeError``/``ValueError`` on bad arguments and
``mouse_core_b200._lib.KernelError`` if the library reports an error. Nothing
here computes on the CPU.
"""

from __future__ import annotations

import torch

from mouse_core_b200 import _lib

BF16 = torch.bfloat16

# Kernels of libmouse_b200 launched through this module (read by the bench).
launch_count = [0]


def _count(n: int = 1) -> None:
    launch_count[0] += n


def _need(t: torch.Tensor, name: str, dtype=None, contiguous=True) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if t.device.type != "cuda":
        raise ValueError(f"{name} must be on a CUDA device, got {t.device}")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def _p(t):
    return None if t is None else t.data_ptr()


def _stream(t: torch.Tensor):
    return torch.cuda.current_stream(t.device).cuda_stream


def decode_workspace_bytes(batch: int, kv_heads: int, q_rows: int, head_dim: int, max_kv_len: int) -> int:
    return int(_lib.load().mb_decode_workspace_bytes(batch, kv_heads, q_rows, head_dim, max_kv_len))


def decode_plan(kv_len: torch.Tensor, kv_heads: int, q_rows: int, head_dim: int, max_kv_len: int,
                workspace: torch.Tensor, block_table: torch.Tensor | None = None, page_size: int = 0) -> None:
    """The split-mode work list for ``kv_len``. With ``block_table`` (and the
    pool's ``page_size``) whole chunks that consecutive rows hold on the same
    pages get one shared work item (``mb_decode_plan_shared``); the queries
    must then see every cached slot (one-token decode)."""
    _need(kv_len, "kv_len", torch.int32)
    _need(workspace, "workspace", torch.uint8)
    if block_table is None:
        _lib.call("mb_decode_plan", _p(kv_len), kv_len.numel(), kv_heads, q_rows, head_dim, max_kv_len,
                  _p(workspace), workspace.numel(), _stream(kv_len))
    else:
        _need(block_table, "block_table", torch.int32)
        _lib.call("mb_decode_plan_shared", _p(kv_len), _p(block_table), block_table.shape[1], int(page_size),
                  kv_len.numel(), kv_heads, q_rows, head_dim, max_kv_len, _p(workspace), workspace.numel(),
                  _stream(kv_len))
    _count()


def decode_attention(q: torch.Tensor, k_pool: torch.Tensor, v_pool: torch.Tensor, block_table: torch.Tensor,
                     q_pos: torch.Tensor, kv_len: torch.Tensor, scale: float, max_kv_len: int,
                     out: torch.Tensor | None = None, workspace: torch.Tensor | None = None,
                     plan_ready: bool = False) -> torch.Tensor:
    """Paged GQA attention (K1).

    q ``[B, S, Hq, hd]`` bf16; pools ``[P, Hkv, page, hd]`` bf16 (one layer);
    block_table ``[B, max_pages]`` int32; q_pos ``[B, S]`` int32; kv_len
    ``[B]`` int32. Returns ``out [B, S, Hq, hd]``.
    """
    _need(q, "q", BF16)
    _need(k_pool, "k_pool", BF16)
    _need(v_pool, "v_pool", BF16)
    _need(block_table, "block_table", torch.int32)
    _need(q_pos, "q_pos", torch.int32)
    _need(kv_len, "kv_len", torch.int32)
    if q.ndim != 4 or k_pool.ndim != 4 or k_pool.shape != v_pool.shape:
        raise ValueError("q must be [B, S, Hq, hd] and the pools [P, Hkv, page, hd] of equal shape")
    B, S, Hq, hd = q.shape
    P, Hkv, page, hd2 = k_pool.shape
    if hd2 != hd:
        raise ValueError(f"head_dim mismatch: q {hd}, pool {hd2}")
    if block_table.ndim != 2 or block_table.shape[0] != B or tuple(q_pos.shape) != (B, S) or kv_len.numel() != B:
        raise ValueError("block_table [B, max_pages], q_pos [B, S] and kv_len [B] must match q")
    if out is None:
        out = torch.empty_like(q)
    else:
        _need(out, "out", BF16)
    G = Hq // Hkv
    ws_ptr, ws_n = None, 0
    split = G * S <= 16
    if split:
        need = decode_workspace_bytes(B, Hkv, G * S, hd, max_kv_len)
        if workspace is None or workspace.numel() < need:
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    if workspace is not None:  # prefill chunks use 4 bytes of it as a tile counter
        _need(workspace, "workspace", torch.uint8)
        ws_ptr, ws_n = _p(workspace), workspace.numel()
    _lib.call("mb_decode_attention", _p(q), _p(k_pool), _p(v_pool), P, _p(block_table), block_table.shape[1],
              _p(q_pos), _p(kv_len), B, S, Hq, Hkv, hd, page, float(scale), int(max_kv_len), int(plan_ready),
              _p(out), ws_ptr, ws_n, _stream(q))
    _count(2 if (split and not plan_ready) else 1)
    return out


def kv_append(qkv: torch.Tensor, pos: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int,
              inv_freq: torch.Tensor, attention_scaling: float = 1.0, q_norm_w: torch.Tensor | None = None,
              k_norm_w: torch.Tensor | None = None, eps: float = 1e-6, slot: torch.Tensor | None = None,
              k_pool: torch.Tensor | None = None, v_pool: torch.Tensor | None = None,
              q_out: torch.Tensor | None = None, k_out: torch.Tensor | None = None,
              v_out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused q/k RMSNorm + RoPE + paged append (K2). ``qkv [T, >=(Hq+2Hkv)hd]``
    bf16 (or fp32: the fp32 projection output of the fp32 residual stream)
    with unit inner stride; returns ``q_out [T, Hq, hd]`` (bf16)."""
    f32 = qkv.dtype == torch.float32
    _need(qkv, "qkv", torch.float32 if f32 else BF16, contiguous=False)
    if qkv.ndim != 2 or qkv.stride(1) != 1:
        raise ValueError("qkv must be 2-D with unit inner stride")
    _need(pos, "pos", torch.int32)
    _need(inv_freq, "inv_freq", torch.float32)
    T = qkv.shape[0]
    if pos.numel() != T:
        raise ValueError("pos must have one entry per token")
    if q_out is None:
        q_out = torch.empty(T, q_heads, head_dim, dtype=BF16, device=qkv.device)
    for name, t in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w)):
        if t is not None:
            _need(t, name, BF16)
    page_size, num_pages = 0, 0
    if k_pool is not None:
        _need(k_pool, "k_pool", BF16)
        _need(v_pool, "v_pool", BF16)
        _need(slot, "slot", torch.int32)
        num_pages, _, page_size, _ = k_pool.shape
    for name, t in (("k_out", k_out), ("v_out", v_out)):
        if t is not None:
            _need(t, name, BF16)
    _lib.call("mb_kv_append_f32" if f32 else "mb_kv_append", _p(qkv), T, qkv.stride(0), _p(pos), _p(slot),
              _p(q_norm_w), _p(k_norm_w),
              float(eps), _p(inv_freq), float(attention_scaling), q_heads, kv_heads, head_dim, page_size,
              num_pages, _p(q_out), _p(k_out), _p(v_out), _p(k_pool), _p(v_pool), _stream(qkv))
    _count()
    return q_out


def rope_table(pos: torch.Tensor, inv_freq: torch.Tensor, head_dim: int, attention_scaling: float = 1.0,
               out: torch.Tensor | None = None) -> torch.Tensor:
    """``[T, head_dim / 2, 2]`` f32: (cos, sin)(pos[t] * inv_freq[j]) *
    attention_scaling, the rotation factors of K2, for ``qkv_append``."""
    _need(pos, "pos", torch.int32)
    _need(inv_freq, "inv_freq", torch.float32)
    T = pos.numel()
    if out is None:
        out = torch.empty(T, head_dim // 2, 2, dtype=torch.float32, device=pos.device)
    _lib.call("mb_rope_table", _p(pos), T, _p(inv_freq), head_dim, float(attention_scaling), _p(out), _stream(pos))
    _count()
    return out


def qkv_append(x: torch.Tensor, w_qkv: torch.Tensor, bias: torch.Tensor | None, rope: torch.Tensor, q_heads: int,
               kv_heads: int, head_dim: int, q_norm_w: torch.Tensor | None = None,
               k_norm_w: torch.Tensor | None = None, eps: float = 1e-6, slot: torch.Tensor | None = None,
               k_pool: torch.Tensor | None = None, v_pool: torch.Tensor | None = None) -> torch.Tensor:
    """K13: ``x [T, hidden] @ w_qkv.T (+ bias)`` on tcgen05 with K2 as the
    epilogue (q/k RMSNorm, RoPE from ``rope``, bf16 q returned, k/v stored at
    ``slot`` in the pools); the same outputs as the fp32 GEMM followed by
    ``kv_append`` up to the GEMM's order of summation."""
    _need(x, "x", BF16)
    _need(w_qkv, "w_qkv", BF16)
    _need(rope, "rope", torch.float32)
    T, hidden = x.shape
    if w_qkv.shape != ((q_heads + 2 * kv_heads) * head_dim, hidden):
        raise ValueError("w_qkv must be [(q_heads + 2 kv_heads) * head_dim, hidden]")
    if rope.numel() != T * head_dim:
        raise ValueError("rope must hold head_dim / 2 (cos, sin) pairs per token")
    if bias is not None:
        _need(bias, "bias", BF16)
    for name, t in (("q_norm_w", q_norm_w), ("k_norm_w", k_norm_w)):
        if t is not None:
            _need(t, name, BF16)
    page_size, num_pages = 0, 0
    if k_pool is not None:
        _need(k_pool, "k_pool", BF16)
        _need(v_pool, "v_pool", BF16)
        _need(slot, "slot", torch.int32)
        num_pages, _, page_size, _ = k_pool.shape
    q_out = torch.empty(T, q_heads, head_dim, dtype=BF16, device=x.device)
    _lib.call("mb_qkv_append", _p(x), T, hidden, _p(w_qkv), _p(bias), _p(rope), _p(q_norm_w), _p(k_norm_w),
              float(eps), _p(slot), q_heads, kv_heads, head_dim, page_size, num_pages, _p(q_out), _p(k_pool),
              _p(v_pool), _stream(x))
    _count()
    return q_out


def page_copy(src_pool: torch.Tensor, dst_pool: torch.Tensor, src_pages: torch.Tensor,
              dst_pages: torch.Tensor) -> None:
    """``dst_pool[dst_pages[i]] = src_pool[src_pages[i]]`` (K3), one layer."""
    _need(src_pool, "src_pool", BF16)
    _need(dst_pool, "dst_pool", BF16)
    _need(src_pages, "src_pages", torch.int32)
    _need(dst_pages, "dst_pages", torch.int32)
    page_elems = src_pool[0].numel()
    _lib.call("mb_page_copy", _p(src_pool), _p(dst_pool), _p(src_pages), _p(dst_pages), src_pages.numel(),
              page_elems, _stream(src_pool))
    _count()


def decode_step_meta(block_table: torch.Tensor, q_pos: torch.Tensor, kv_len: torch.Tensor, slot: torch.Tensor,
                     page_size: int, new_page: torch.Tensor | None = None) -> None:
    """In place: one decode step's ``q_pos``, ``slot`` and ``kv_len`` (int32
    ``[B]``) from the current ``kv_len`` and ``block_table [B, max_pages]``.
    ``new_page`` holds one code per row (``None``: every row appends): -1
    append; a page id the row's token opens (written into the table first),
    with bit 30 set for a row emptied since (it restarts at length 0); -2 the
    row sits out; -3 the row was emptied and sits out."""
    for name, t in (("block_table", block_table), ("q_pos", q_pos), ("kv_len", kv_len), ("slot", slot)):
        _need(t, name, torch.int32)
    if new_page is not None:
        _need(new_page, "new_page", torch.int32)
    B, width = block_table.shape
    _lib.call("mb_decode_step_meta", B, width, int(page_size), _p(new_page), _p(block_table), _p(q_pos),
              _p(kv_len), _p(slot), _stream(kv_len))
    _count()


def decode_step_meta_args(block_table: torch.Tensor, q_pos: torch.Tensor, kv_len: torch.Tensor, slot: torch.Tensor,
                          page_size: int, new_page: torch.Tensor) -> tuple:
    """Checked argument tuple of ``decode_step_meta`` for tensors that stay in
    place across many steps; launch it with ``decode_step_meta_launch``."""
    for name, t in (("block_table", block_table), ("q_pos", q_pos), ("kv_len", kv_len), ("slot", slot),
                    ("new_page", new_page)):
        _need(t, name, torch.int32)
    B, width = block_table.shape
    if not (q_pos.numel() == kv_len.numel() == slot.numel() == new_page.numel() == B):
        raise ValueError("q_pos, kv_len, slot and new_page must have one entry per block-table row")
    return (B, width, int(page_size), new_page.data_ptr(), block_table.data_ptr(), q_pos.data_ptr(),
            kv_len.data_ptr(), slot.data_ptr())


def decode_step_meta_launch(args: tuple, use_new_page: bool, stream: int) -> None:
    """``decode_step_meta`` from a ``decode_step_meta_args`` tuple; ``new_page``
    is read only when ``use_new_page``."""
    B, width, page_size, new_page, bt, q_pos, kv_len, slot = args
    _lib.call("mb_decode_step_meta", B, width, page_size, new_page if use_new_page else None, bt, q_pos, kv_len,
              slot, stream)
    _count()


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, residual: torch.Tensor | None = None):
    """Returns ``(sum, norm)``: ``sum = x + residual`` (or ``x``), ``norm = RMSNorm(sum) * weight``."""
    _need(x, "x", BF16)
    _need(weight, "weight", BF16)
    D = x.shape[-1]
    rows = x.numel() // D
    norm = torch.empty_like(x)
    s = None
    if residual is not None:
        _need(residual, "residual", BF16)
        s = torch.empty_like(x)
    _lib.call("mb_rmsnorm", _p(x), _p(residual), _p(weight), float(eps), rows, D, _p(s), _p(norm), _stream(x))
    _count()
    return (s if s is not None else x), norm


def rmsnorm_f32(x: torch.Tensor, weight: torch.Tensor, eps: float, delta: torch.Tensor | None = None,
                sum_out: torch.Tensor | None = None):
    """fp32 residual stream: returns ``(sum, norm)`` with ``sum = x + delta``
    kept fp32 (``x`` fp32, or the bf16 embeddings entering the first layer;
    written into ``sum_out`` when given, which may be ``x``) and ``norm =
    bf16(RMSNorm(sum) * weight)``."""
    _need(x, "x", torch.float32 if x.dtype == torch.float32 else BF16)
    _need(weight, "weight", BF16)
    D = x.shape[-1]
    rows = x.numel() // D
    if delta is not None:
        _need(delta, "delta", torch.float32)
    if sum_out is None and (delta is not None or x.dtype != torch.float32):
        sum_out = torch.empty(x.shape, dtype=torch.float32, device=x.device)
    norm = torch.empty(x.shape, dtype=BF16, device=x.device)
    xf, xb = (x, None) if x.dtype == torch.float32 else (None, x)
    _lib.call("mb_rmsnorm_f32", _p(xf), _p(xb), _p(delta), _p(weight), float(eps), rows, D, _p(sum_out), _p(norm),
              _stream(x))
    _count()
    return (sum_out if sum_out is not None else x), norm


def silu_mul_f32(gate_up: torch.Tensor) -> torch.Tensor:
    """``bf16(silu(gate) * up)`` for an fp32 ``gate_up [..., 2I]``; returns ``[..., I]`` bf16."""
    _need(gate_up, "gate_up", torch.float32)
    I2 = gate_up.shape[-1]
    rows = gate_up.numel() // I2
    out = torch.empty(*gate_up.shape[:-1], I2 // 2, dtype=BF16, device=gate_up.device)
    _lib.call("mb_silu_mul_f32", _p(gate_up), rows, I2 // 2, _p(out), _stream(gate_up))
    _count()
    return out


def segment_meta(sequence_ids: torch.Tensor, tile: int = 128, with_run_end: bool = False):
    """K7: ``(position int64 [L], run_start int32 [L], tile_lo int32 [ceil(L/tile)],
    unsorted flag int32 [1])`` of a packed stream, plus ``run_end int32 [L]``
    (one past the end of each token's run) last when ``with_run_end``."""
    _need(sequence_ids, "sequence_ids", torch.int64)
    L = sequence_ids.numel()
    dev = sequence_ids.device
    pos = torch.empty(L, dtype=torch.int64, device=dev)
    rs = torch.empty(L, dtype=torch.int32, device=dev)
    tl = torch.empty((L + tile - 1) // tile, dtype=torch.int32, device=dev)
    flags = torch.zeros(1, dtype=torch.int32, device=dev)
    re = torch.empty(L, dtype=torch.int32, device=dev) if with_run_end else None
    _lib.call("mb_segment_meta", _p(sequence_ids), L, tile, _p(pos), _p(rs), _p(re), _p(tl), _p(flags),
              _stream(sequence_ids))
    _count()
    if with_run_end:
        return pos, rs, tl, flags, re
    return pos, rs, tl, flags


def varlen_attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, run_start: torch.Tensor,
                        tile_lo: torch.Tensor, scale: float):
    """K5: segment-causal GQA attention over a packed stream. q ``[L, Hq, hd]``,
    k/v ``[L, Hkv, hd]`` bf16; returns ``(out [L, Hq, hd], lse [Hq, L] f32, log2 units)``."""
    for name, t in (("q", q), ("k", k), ("v", v)):
        _need(t, name, BF16)
    _need(run_start, "run_start", torch.int32)
    _need(tile_lo, "tile_lo", torch.int32)
    L, Hq, hd = q.shape
    Hkv = k.shape[1]
    if k.shape != (L, Hkv, hd) or v.shape != k.shape:
        raise ValueError("k and v must be [L, Hkv, hd] matching q")
    out = torch.empty_like(q)
    lse_buf = torch.empty(Hq * L + 4, dtype=torch.float32, device=q.device)  # MB_VARLEN_FWD_LSE_FLOATS
    _lib.call("mb_varlen_attention_fwd", _p(q), _p(k), _p(v), L, Hq, Hkv, hd, _p(run_start), _p(tile_lo),
              float(scale), _p(out), _p(lse_buf), _stream(q))
    _count()
    return out, lse_buf[:Hq * L].view(Hq, L)


# Largest dS scratch the stored-dS backward takes before falling back to the
# recompute path (bytes); the scratch is Hq x pairs x 32 KB.
STORED_DS_MAX_BYTES = 24 << 30


def varlen_pair_offsets(tile_lo: torch.Tensor, L: int) -> torch.Tensor:
    """``pair_off int32 [ceil(L/128) + 1]`` of the stored-dS backward (the
    last entry is the number of (query tile, key tile) pairs)."""
    _need(tile_lo, "tile_lo", torch.int32)
    out = torch.empty((L + 127) // 128 + 1, dtype=torch.int32, device=tile_lo.device)
    _lib.call("mb_varlen_bwd_pair_offsets", _p(tile_lo), int(L), _p(out), _stream(tile_lo))
    _count()
    return out


def varlen_attention_bwd(q, k, v, out, dout, lse, run_start, run_end, scale, tile_lo=None, pair_off=None,
                         n_pairs=None):
    """K6: ``(dq, dk, dv)`` of ``varlen_attention_fwd`` for upstream ``dout``.
    With ``tile_lo``, ``pair_off`` and ``n_pairs`` (and a dS scratch within
    ``STORED_DS_MAX_BYTES``) dQ is one GEMM over the dS blocks the dK/dV kernel
    stores; otherwise the dQ kernel recomputes S and dP."""
    for name, t in (("q", q), ("k", k), ("v", v), ("out", out), ("dout", dout)):
        _need(t, name, BF16)
    _need(lse, "lse", torch.float32)
    _need(run_start, "run_start", torch.int32)
    _need(run_end, "run_end", torch.int32)
    L, Hq, hd = q.shape
    Hkv = k.shape[1]
    dq = torch.empty_like(q)
    dk = torch.empty_like(k)
    dv = torch.empty_like(v)
    delta = torch.empty(Hq * L + 4, dtype=torch.float32, device=q.device)  # MB_VARLEN_BWD_SCRATCH_FLOATS
    ds_bytes = Hq * int(n_pairs) * 32768 if n_pairs is not None else None  # MB_VARLEN_BWD_DS_BYTES
    if pair_off is not None and L > 0 and ds_bytes <= STORED_DS_MAX_BYTES:
        _need(tile_lo, "tile_lo", torch.int32)
        _need(pair_off, "pair_off", torch.int32)
        ds = torch.empty(ds_bytes, dtype=torch.uint8, device=q.device)
        _lib.call("mb_varlen_attention_bwd_stored", _p(q), _p(k), _p(v), _p(out), _p(dout), _p(lse), L, Hq, Hkv,
                  hd, _p(run_start), _p(run_end), _p(tile_lo), _p(pair_off), int(n_pairs), float(scale), _p(dq),
                  _p(dk), _p(dv), _p(delta), _p(ds), ds_bytes, _stream(q))
    else:
        _lib.call("mb_varlen_attention_bwd", _p(q), _p(k), _p(v), _p(out), _p(dout), _p(lse), L, Hq, Hkv, hd,
                  _p(run_start), _p(run_end), float(scale), _p(dq), _p(dk), _p(dv), _p(delta), _stream(q))
    _count(3)
    return dq, dk, dv


# ---------------------------------------------------------------- decode-step layout glue (K9)


def flat_rank(sequence_ids: torch.Tensor, prediction_indices: torch.Tensor, steps_and_offsets: torch.Tensor,
              B: int, S: int):
    """``(rank int32 [L], stats int32 [B + 2], local int64 [B, S])`` of
    ``mb_flat_rank``; ``steps_and_offsets`` is int32 ``[2, B]`` (step counts,
    then their exclusive prefix sums)."""
    _need(sequence_ids, "sequence_ids", torch.int64)
    _need(prediction_indices, "prediction_indices", torch.int64)
    _need(steps_and_offsets, "steps_and_offsets", torch.int32)
    L, dev = sequence_ids.numel(), sequence_ids.device
    rank = torch.empty(L, dtype=torch.int32, device=dev)
    stats = torch.empty(B + 2, dtype=torch.int32, device=dev)
    local = torch.empty(B, S, dtype=torch.int64, device=dev)
    _lib.call("mb_flat_rank", _p(sequence_ids), L, int(B), _p(prediction_indices), prediction_indices.numel(),
              _p(steps_and_offsets[0]), _p(steps_and_offsets[1]), int(S), _p(rank), _p(stats), _p(local),
              _stream(sequence_ids))
    _count()
    return rank, stats, local


def flat_scatter(embeds: torch.Tensor, sequence_ids: torch.Tensor, rank: torch.Tensor, B: int, max_len: int):
    """Right-padded ``[B, max_len, D]`` copy of flat ``embeds [L, D]`` at
    ``(sequence_ids[i], rank[i])`` (``mb_flat_scatter``)."""
    _need(embeds, "embeds")
    _need(sequence_ids, "sequence_ids", torch.int64)
    _need(rank, "rank", torch.int32)
    L, D = embeds.shape
    out = torch.empty(B, max_len, D, dtype=embeds.dtype, device=embeds.device)
    _lib.call("mb_flat_scatter", _p(embeds), L, D * embeds.element_size(), _p(sequence_ids), _p(rank), int(B),
              int(max_len), _p(out), _stream(embeds))
    _count()
    return out


def left_align(embeds: torch.Tensor, prediction_indices: torch.Tensor):
    """``(aligned [B, L, D], aligned_indices int64 [B, S])`` of ``mb_left_align``."""
    _need(embeds, "embeds")
    _need(prediction_indices, "prediction_indices", torch.int64)
    B, L, D = embeds.shape
    out = torch.empty_like(embeds)
    idx = torch.empty_like(prediction_indices)
    _lib.call("mb_left_align", _p(embeds), B, L, D * embeds.element_size(), _p(prediction_indices),
              prediction_indices.shape[1], _p(out), _p(idx), _stream(embeds))
    _count()
    return out, idx


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gate_up [..., 2I]``; returns ``[..., I]``."""
    _need(gate_up, "gate_up", BF16)
    I2 = gate_up.shape[-1]
    rows = gate_up.numel() // I2
    out = torch.empty(*gate_up.shape[:-1], I2 // 2, dtype=BF16, device=gate_up.device)
    _lib.call("mb_silu_mul", _p(gate_up), rows, I2 // 2, _p(out), _stream(gate_up))
    _count()
    return out


# ---------------------------------------------------------------- training layer element-wise (K4)


def _rows_view(x: torch.Tensor, name: str):
    """``(rows, row_stride)`` of a 2-D bf16 view whose last dim is contiguous."""
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with a contiguous last dimension")
    return x.shape[0], x.stride(0)


def rmsnorm_fwd(x: torch.Tensor, weight: torch.Tensor, eps: float):
    """``(y, rstd)``: ``y = weight * bf16(x * rstd)`` over the last dim; rstd f32 ``[rows]``."""
    _need(x, "x", BF16)
    _need(weight, "weight", BF16)
    D = x.shape[-1]
    rows = x.numel() // D
    y = torch.empty_like(x)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.call("mb_rmsnorm_fwd", _p(x), _p(weight), float(eps), rows, D, _p(y), _p(rstd), _stream(x))
    _count()
    return y, rstd


def add_rmsnorm_fwd(x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float):
    """``(sum, y, rstd)``: ``sum = bf16(x + residual)``, then ``rmsnorm_fwd(sum)``."""
    for name, t in (("x", x), ("residual", residual), ("weight", weight)):
        _need(t, name, BF16)
    if residual.shape != x.shape:
        raise ValueError("residual must match x")
    D = x.shape[-1]
    rows = x.numel() // D
    total = torch.empty_like(x)
    y = torch.empty_like(x)
    rstd = torch.empty(rows, dtype=torch.float32, device=x.device)
    _lib.call("mb_add_rmsnorm_fwd", _p(x), _p(residual), _p(weight), float(eps), rows, D, _p(total), _p(y), _p(rstd),
              _stream(x))
    _count()
    return total, y, rstd


def rmsnorm_bwd(dy: torch.Tensor, x: torch.Tensor, weight: torch.Tensor, rstd: torch.Tensor,
                dsum: torch.Tensor | None = None):
    """``(dx bf16, dweight f32)`` of ``rmsnorm_fwd``; with ``dsum`` (the
    gradient reaching ``x`` along a residual path) added into ``dx``."""
    for name, t in (("dy", dy), ("x", x), ("weight", weight)):
        _need(t, name, BF16)
    _need(rstd, "rstd", torch.float32)
    if dsum is not None:
        _need(dsum, "dsum", BF16)
        if dsum.shape != x.shape:
            raise ValueError("dsum must match x")
    D = x.shape[-1]
    rows = x.numel() // D
    if dy.shape != x.shape or rstd.numel() != rows:
        raise ValueError("dy must match x and rstd must hold one value per row")
    dx = torch.empty_like(x)
    dw = torch.empty(D, dtype=torch.float32, device=x.device)
    n = int(_lib.load().mb_rmsnorm_bwd_scratch_floats(rows, D))
    scratch = torch.empty(max(n, 1), dtype=torch.float32, device=x.device)
    if dsum is None:
        _lib.call("mb_rmsnorm_bwd", _p(dy), _p(x), _p(weight), _p(rstd), rows, D, _p(dx), _p(dw), _p(scratch), n,
                  _stream(x))
    else:
        _lib.call("mb_rmsnorm_bwd_add", _p(dy), _p(x), _p(weight), _p(rstd), _p(dsum), rows, D, _p(dx), _p(dw),
                  _p(scratch), n, _stream(x))
    _count(2)
    return dx, dw


def qkv_heads_fwd(qkv: torch.Tensor, q_heads: int, kv_heads: int, head_dim: int, cos: torch.Tensor,
                  sin: torch.Tensor, q_norm_weight: torch.Tensor | None = None,
                  k_norm_weight: torch.Tensor | None = None, q_eps: float = 1e-6, k_eps: float = 1e-6):
    """Attention inputs from a fused projection ``qkv [L, >= (Hq + 2 Hkv) hd]``
    (rows may be strided, last dim contiguous): q and k through the optional
    per-head RMSNorm and rotate-half RoPE (``cos``/``sin [L, hd]``), v copied.
    Returns ``(q [L,Hq,hd], k [L,Hkv,hd], v [L,Hkv,hd], q_rstd, k_rstd)``
    (the rstd tensors are None without the norm)."""
    _need(qkv, "qkv", BF16, contiguous=False)
    L, xs = _rows_view(qkv, "qkv")
    for name, t in (("cos", cos), ("sin", sin)):
        _need(t, name, BF16)
        if t.shape != (L, head_dim):
            raise ValueError(f"{name} must be [L, head_dim]")
    norm = q_norm_weight is not None
    if norm != (k_norm_weight is not None):
        raise ValueError("pass both norm weights or neither")
    if norm:
        _need(q_norm_weight, "q_norm_weight", BF16)
        _need(k_norm_weight, "k_norm_weight", BF16)
    dev = qkv.device
    q = torch.empty(L, q_heads, head_dim, dtype=BF16, device=dev)
    k = torch.empty(L, kv_heads, head_dim, dtype=BF16, device=dev)
    v = torch.empty(L, kv_heads, head_dim, dtype=BF16, device=dev)
    q_rstd = torch.empty(L * q_heads, dtype=torch.float32, device=dev) if norm else None
    k_rstd = torch.empty(L * kv_heads, dtype=torch.float32, device=dev) if norm else None
    _lib.call("mb_qkv_heads_fwd", _p(qkv), xs, L, q_heads, kv_heads, head_dim, _p(q_norm_weight),
              _p(k_norm_weight), float(q_eps), float(k_eps), _p(cos), _p(sin), _p(q), _p(k), _p(v), _p(q_rstd),
              _p(k_rstd), _stream(qkv))
    _count()
    return q, k, v, q_rstd, k_rstd


def qkv_heads_bwd(dq: torch.Tensor, dk: torch.Tensor, dv: torch.Tensor, qkv: torch.Tensor, cos: torch.Tensor,
                  sin: torch.Tensor, q_norm_weight: torch.Tensor | None = None,
                  k_norm_weight: torch.Tensor | None = None, q_rstd: torch.Tensor | None = None,
                  k_rstd: torch.Tensor | None = None, dqkv: torch.Tensor | None = None):
    """Gradient of ``qkv_heads_fwd``: fills ``dqkv`` (allocated like ``qkv``
    when None) and returns ``(dqkv, dq_norm_weight f32, dk_norm_weight f32)``
    (the weight gradients are None without the norm)."""
    for name, t in (("dq", dq), ("dk", dk), ("dv", dv)):
        _need(t, name, BF16)
    L, Hq, hd = dq.shape
    Hkv = dk.shape[1]
    if dk.shape != (L, Hkv, hd) or dv.shape != dk.shape:
        raise ValueError("dk and dv must be [L, Hkv, hd] matching dq")
    _need(qkv, "qkv", BF16, contiguous=False)
    _, xs = _rows_view(qkv, "qkv")
    if dqkv is None:
        dqkv = torch.empty(L, (Hq + 2 * Hkv) * hd, dtype=BF16, device=dq.device)
    _need(dqkv, "dqkv", BF16, contiguous=False)
    _, dxs = _rows_view(dqkv, "dqkv")
    norm = q_norm_weight is not None
    dqw = dkw = scratch = None
    n = 0
    if norm:
        _need(q_rstd, "q_rstd", torch.float32)
        _need(k_rstd, "k_rstd", torch.float32)
        dqw = torch.empty(hd, dtype=torch.float32, device=dq.device)
        dkw = torch.empty(hd, dtype=torch.float32, device=dq.device)
        n = int(_lib.load().mb_qkv_heads_bwd_scratch_floats(L, hd))
        scratch = torch.empty(max(n, 1), dtype=torch.float32, device=dq.device)
    _lib.call("mb_qkv_heads_bwd", _p(dq), _p(dk), _p(dv), _p(qkv), xs, L, Hq, Hkv, hd, _p(q_norm_weight),
              _p(k_norm_weight), _p(cos), _p(sin), _p(q_rstd), _p(k_rstd), _p(dqkv), dxs, _p(dqw), _p(dkw),
              _p(scratch), n, _stream(dq))
    _count(2 if norm else 1)
    return dqkv, dqw, dkw


def silu_mul_bwd(gate_up: torch.Tensor, dh: torch.Tensor) -> torch.Tensor:
    """``dgate_up [..., 2I]`` of ``silu_mul`` for upstream ``dh [..., I]``."""
    _need(gate_up, "gate_up", BF16)
    _need(dh, "dh", BF16)
    I2 = gate_up.shape[-1]
    rows = gate_up.numel() // I2
    if dh.numel() != rows * (I2 // 2):
        raise ValueError("dh must be [..., I] matching gate_up [..., 2I]")
    dgu = torch.empty_like(gate_up)
    _lib.call("mb_silu_mul_bwd", _p(gate_up), _p(dh), rows, I2 // 2, _p(dgu), _stream(gate_up))
    _count()
    return dgu
