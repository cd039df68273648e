"""Paged cached decoding — drop-in for mouse-core's ``FlexDecodeSession``.

Reference: ``FlexDecodeSession`` (src/mouse_core/models/backbone/flex_decode.py:
75-240). Same constructor ``(model, batch_size, capacity)``, same
``forward(*, embeds, lengths, output_hidden_states=False)`` contract, same
``B``/``lengths`` attributes and errors; every row decodes exactly as it
would alone with a private cache.

What changes is the machinery, built for B200:

* KV lives in pages of ``page_size`` tokens drawn from one pool per layer
  (``[num_pages, kv_heads, page, head_dim]`` bf16) and addressed through a
  block table, so a row that outgrows its space gets a new page instead of the
  reference's whole-cache doubling copy (flex_decode.py:140-149).
* Per layer, the decoder loop (flex_decode.py:208-234) runs five kernels of
  ``libmouse_b200`` around three cuBLAS GEMMs: fused residual-add + RMSNorm;
  QKV GEMM; K2 (q/k RMSNorm + RoPE + page append); K1 (paged split-KV GQA
  attention, replacing the FlexAttention call and the per-call BlockMask
  build); o_proj GEMM; residual-add + RMSNorm; gate/up GEMM; SiLU product;
  down GEMM.
* Per call, positions, cache slots and the changed block table are computed
  on the host (where the lengths already are) and shipped in ONE host-to-device
  copy; the split-KV work list is built once on the device and reused by every
  layer. The reference's host syncs (``.max()`` at flex_decode.py:180,
  ``nonzero`` at :195) are gone.

The session requires a CUDA bf16 model with head_dim 64 or 128; anything else
raises — there is no CPU or eager fallback.
"""

from __future__ import annotations

import copy
from typing import Any, cast

import numpy as np
import torch
import torch.nn.functional as F

from mouse_core_b200 import kernels as K
from mouse_core_b200.pages import PageTable
from mouse_core_b200.trace import nvtx_range

DEFAULT_PAGE_SIZE = 128


def _round_up(value: int, multiple: int) -> int:
    return -(-value // multiple) * multiple


# mb_decode_step_meta code flag (MB_STEP_RESTART): the row was emptied and its
# token restarts it at length 0, opening the page in the low bits at column 0.
_STEP_RESTART = 1 << 30


def rope_frequencies(rotary, config, device) -> tuple[torch.Tensor, float]:
    """RoPE inverse frequencies in fp32 as the model config defines them, and
    the cos/sin scaling.

    A transformers rotary module keeps its frequencies in an ``inv_freq``
    buffer, and casting the model to bf16 casts that buffer too: the
    frequencies keep 8 mantissa bits, so the rotation angle ``pos * f`` of a
    token at position 500 is off by up to ~1 radian at the highest frequency.
    The reference's bf16 decode inherits that (flex_decode.py:204 calls the
    module). The frequencies are a function of the config, so they are
    recomputed here in fp32 with transformers' own initialiser for the
    config's rope type (Llama-3 scaling included); rope types whose module
    updates the buffer at run time fall back to the buffer."""
    rope_type = getattr(rotary, "rope_type", "default")
    try:
        if rope_type == "default":
            fn = type(rotary).compute_default_rope_parameters
        elif rope_type in ("dynamic", "longrope"):
            fn = None
        else:
            from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS

            fn = ROPE_INIT_FUNCTIONS[rope_type]
        if fn is not None:
            inv, scaling = fn(config, device)
            return inv.to(device=device, dtype=torch.float32), float(scaling)
    except Exception:  # an unknown rotary module: use what it holds
        pass
    return (rotary.inv_freq.to(device=device, dtype=torch.float32),
            float(getattr(rotary, "attention_scaling", 1.0)))


class _LayerWeights:
    """Per-layer weights; QKV and gate/up are concatenated once per weight
    version so each runs as one GEMM."""

    def __init__(self, layer, n_heads, n_kv_heads, head_dim):
        self.layer = layer
        self.version = None
        self.refresh()

    def _sources(self):
        a = self.layer.self_attn
        m = self.layer.mlp
        return (a.q_proj.weight, a.k_proj.weight, a.v_proj.weight, m.gate_proj.weight, m.up_proj.weight)

    def refresh(self) -> None:
        ver = tuple((t.data_ptr(), t._version) for t in self._sources())
        if ver == self.version:
            return
        a = self.layer.self_attn
        m = self.layer.mlp
        with torch.no_grad():
            self.wqkv = torch.cat([a.q_proj.weight, a.k_proj.weight, a.v_proj.weight], 0).contiguous()
            bq = a.q_proj.bias
            self.bqkv = torch.cat([a.q_proj.bias, a.k_proj.bias, a.v_proj.bias]) if bq is not None else None
            self.wgu = torch.cat([m.gate_proj.weight, m.up_proj.weight], 0).contiguous()
            bg = getattr(m.gate_proj, "bias", None)
            self.bgu = torch.cat([m.gate_proj.bias, m.up_proj.bias]) if bg is not None else None
        self.version = ver
        self.in_w = self.layer.input_layernorm.weight
        self.in_eps = float(self.layer.input_layernorm.variance_epsilon)
        self.post_w = self.layer.post_attention_layernorm.weight
        self.post_eps = float(self.layer.post_attention_layernorm.variance_epsilon)
        qn = getattr(a, "q_norm", None)
        self.q_norm_w = qn.weight if qn is not None else None
        self.k_norm_w = a.k_norm.weight if qn is not None else None
        self.qk_eps = float(qn.variance_epsilon) if qn is not None else 1e-6
        self.o_proj = a.o_proj
        self.down = m.down_proj
        self.scale = float(a.scaling)


class PagedDecodeSession:
    """Incremental decoder over ``batch_size`` independently-growing sequences.

    Args:
        model: A transformers decoder stack (``Qwen3Model`` / ``LlamaModel``)
            with ``layers``, ``rotary_emb`` and ``norm``; used in place. Must
            be bf16 on a CUDA device.
        batch_size: Number of sequences decoded by this session.
        capacity: Initial per-row KV slots used to size the page pool (the
            pool grows when it runs out; rows never need a copy).
        page_size: Tokens per KV page (a multiple of 64).
        num_pages: Pool size in pages (default: enough for ``capacity`` slots
            in every row).
    """

    def __init__(self, model: torch.nn.Module, batch_size: int, capacity: int = DEFAULT_PAGE_SIZE, *,
                 page_size: int = DEFAULT_PAGE_SIZE, num_pages: int | None = None) -> None:
        hf = cast(Any, model)
        if getattr(hf.config, "use_sliding_window", False):
            raise ValueError("FlexDecodeSession does not support sliding-window attention.")
        self.model = hf
        cfg = hf.config
        self.B = int(batch_size)
        self.n_heads = int(cfg.num_attention_heads)
        self.n_kv_heads = int(cfg.num_key_value_heads)
        self.head_dim = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads)
        param = next(hf.parameters())
        self.device, self.dtype = param.device, param.dtype
        if self.device.type != "cuda":
            raise RuntimeError("mouse_core_b200 decoding runs on a CUDA device (B200, sm_100a) only; "
                               f"the model is on {self.device}")
        if self.dtype != torch.bfloat16:
            raise TypeError("mouse_core_b200 kernels compute in bfloat16; move the backbone to "
                            f"torch.bfloat16 (got {self.dtype})")
        if self.head_dim not in (64, 128):
            raise ValueError(f"head_dim must be 64 or 128 for the sm_100a kernels, got {self.head_dim}")
        if page_size <= 0 or page_size % 64:
            raise ValueError("page_size must be a positive multiple of 64")
        self.page_size = int(page_size)
        self.n_layers = len(hf.layers)
        cap = _round_up(max(int(capacity), 1), self.page_size)
        pages_per_row = cap // self.page_size
        P = int(num_pages) if num_pages is not None else max(self.B * pages_per_row, 1)
        shape = (self.n_layers, P, self.n_kv_heads, self.page_size, self.head_dim)
        # Zero-filled like the reference's cache: slots never written read as 0.
        self.k_pool = torch.zeros(shape, device=self.device, dtype=self.dtype)
        self.v_pool = torch.zeros_like(self.k_pool)
        self.pages = PageTable(self.B, P, self.page_size, pages_per_row)
        self._len = np.zeros(self.B, dtype=np.int64)
        self._bt_dev = torch.full((self.B, self.pages.max_pages), -1, dtype=torch.int32, device=self.device)
        self._workspace = torch.empty(0, dtype=torch.uint8, device=self.device)
        self._meta_dev = torch.empty(0, dtype=torch.int32, device=self.device)
        # Single-token steps (S = 1, the steady state of env stepping) replay a
        # CUDA graph of the whole layer stack after one eager warm-up call.
        self.use_graphs = True
        # Steps of at most one token per row between replays: positions,
        # slots and lengths are made on the device from the previous step's
        # lengths (K8, mb_decode_step_meta), fed only with one code per row
        # (pages opened, rows sitting out, rows emptied since); the host keeps
        # its page table and lengths in step with it.
        self.use_device_step = True
        self._device_step_ok = False  # device metadata is the one-token layout of the host's state
        # Rows emptied by reset_rows while the device path stays valid: their
        # device table rows and lengths are stale until a step restarts them
        # (or a host-path call re-sends the whole table).
        self._pending_reset = np.zeros(self.B, dtype=bool)
        self._new_page_dev = torch.full((self.B,), -1, dtype=torch.int32, device=self.device)
        self._step_args: tuple | None = None  # pointers of the captured graph's metadata views
        self._graph = None
        self._graph_key = None
        self._graph_warm = False
        # decode_step's graph: embedding gather + layer stack + norm + head.
        self._step_graph = None
        self._step_graph_key = None
        self._step_graph_warm = False
        # Keep the residual stream in fp32 between the layers (only GEMM
        # inputs, q/k/v and the pool are bf16); False restores the modules'
        # bf16 rounding at every add.
        self.residual_fp32 = True
        # Run each layer's QKV projection as K13 (the tcgen05 GEMM with K2 as
        # its epilogue, no fp32 projection written) instead of cuBLAS
        # followed by K2. Off by default: at decode sizes (256-1024 tokens,
        # hidden 1024-2048) cuBLAS + K2 measured 9.6 against 11.3 us per
        # layer, K13's 64-256 CTAs each streaming its whole K extent.
        self.fused_qkv = False
        self._step_ids = None
        self._step_out = None
        self._step_launches = 0
        self._staging = [None, None]
        self._staging_ev = [None, None]
        self._turn = 0
        self._layers = [_LayerWeights(layer, self.n_heads, self.n_kv_heads, self.head_dim) for layer in hf.layers]
        self.inv_freq, self.attention_scaling = rope_frequencies(hf.rotary_emb, cfg, self.device)
        # When a list, each attention launch appends (start, end, reps): CUDA
        # events on the launching stream around `attn_reps` repeats of the
        # launch (used for roofline timing; see _attend).
        self.attn_events: list | None = None
        self.attn_reps = 4

    def clone(self) -> "PagedDecodeSession":
        """An independent copy of this session's cache (page pools, page
        table, lengths, pending resets) that shares the model weights and
        holds no captured graph: stepping either one leaves the other as it
        was. Costs one device copy of the pools."""
        c = copy.copy(self)
        c.k_pool, c.v_pool = self.k_pool.clone(), self.v_pool.clone()
        c.pages = copy.deepcopy(self.pages)
        c._len = self._len.copy()
        c._pending_reset = self._pending_reset.copy()
        c._bt_dev = self._bt_dev.clone()
        c._meta_dev = self._meta_dev.clone()
        c._new_page_dev = self._new_page_dev.clone()
        c._workspace = torch.empty_like(self._workspace)
        c._graph = c._graph_key = c._step_graph = c._step_graph_key = c._step_args = None
        c._graph_warm = c._step_graph_warm = False
        c._step_ids = c._step_out = None
        c._staging, c._staging_ev = [None, None], [None, None]
        c.attn_events = None
        return c

    def _attend(self, q, li, scale, q_pos, kv_len, split):
        """Attention of layer ``li`` over the page pool (K1 split/block decode
        or the tcgen05 paged prefill). With ``attn_events`` set, the launch is
        then repeated ``attn_reps`` times between two CUDA events on the
        launching stream: each repeat is queued behind the previous launch,
        so the events time the kernel and not a gap while the host submits it
        (the launch reads the pools and writes a fresh output: repeats are
        idempotent)."""
        args = (q, self.k_pool[li], self.v_pool[li], self._bt_dev, q_pos, kv_len, scale, self.cap)
        o = K.decode_attention(*args, workspace=self._workspace, plan_ready=split)
        if self.attn_events is not None:
            reps = max(1, int(self.attn_reps))
            ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            ev0.record()
            for _ in range(reps):
                o = K.decode_attention(*args, workspace=self._workspace, plan_ready=split)
            ev1.record()
            self.attn_events.append((ev0, ev1, reps))
        return o

    # ------------------------------------------------------------------ state
    @property
    def lengths(self) -> torch.Tensor:
        """Tokens cached per row, ``[B]`` long on the session device."""
        return torch.from_numpy(self._len.copy()).to(self.device)

    @property
    def cap(self) -> int:
        """Slots addressable per row without widening the block table."""
        return self.pages.max_pages * self.page_size

    @property
    def block_table(self) -> torch.Tensor:
        return self._bt_dev

    def reset_rows(self, rows) -> None:
        """Empty ``rows`` (their pages return to the pool); the next call
        decodes them from position 0, as a fresh session would."""
        r = np.atleast_1d(np.asarray(rows, dtype=np.int64))
        table_synced = not self.pages.dirty
        self.pages.release_rows(r)
        self._len[r] = 0
        if self._device_step_ok and table_synced:
            self.pages.dirty = False  # only these rows differ; the next step restarts them
            self._pending_reset[r] = True
        else:
            self._device_step_ok = False

    def fork(self, src_rows, dst_rows, prefix_lengths=None) -> None:
        """Start rows ``dst_rows`` as branches of ``src_rows``: branch ``i``
        holds the first ``prefix_lengths[i]`` cached tokens of its source row
        (default: all of them) and continues decoding from there.

        The prefix's full pages are shared by reference (no copy; pages are
        refcounted and return to the pool when the last holder lets go); only
        a partially filled last page is copied (K3) so the branch can append
        to it. Destination rows are emptied first. This has no counterpart in
        the reference, whose GRPO rollouts re-run every branch uncached."""
        src = np.atleast_1d(np.asarray(src_rows, dtype=np.int64))
        dst = np.atleast_1d(np.asarray(dst_rows, dtype=np.int64))
        if src.shape != dst.shape:
            raise ValueError("src_rows and dst_rows must have the same length")
        self._device_step_ok = False
        plen = self._len[src].copy() if prefix_lengths is None else np.atleast_1d(
            np.asarray(prefix_lengths, dtype=np.int64))
        if plen.shape != src.shape or (plen < 0).any() or (plen > self._len[src]).any():
            raise ValueError("prefix_lengths must satisfy 0 <= prefix <= the source row's length")
        if len(set(dst.tolist())) != dst.size or set(dst.tolist()) & set(src.tolist()):
            raise ValueError("dst_rows must be distinct and disjoint from src_rows")
        self.pages.release_rows(dst)
        self._len[dst] = 0
        page = self.page_size
        full = plen // page
        partial = plen % page
        n_copy = int((partial > 0).sum())
        if n_copy > self.pages.free_pages:
            self._grow_pool(n_copy)
        copy_src, copy_dst = [], []
        for s_row, d_row, nf, part in zip(src, dst, full, partial):
            self.pages.share(int(d_row), int(s_row), int(nf))
            if part:
                new = int(self.pages.take_free(1)[0])
                self.pages.ensure_width(int(nf) + 1)
                self.pages.table[d_row, nf] = new
                self.pages.npages[d_row] = nf + 1
                self.pages.dirty = True
                copy_src.append(int(self.pages.table[s_row, nf]))
                copy_dst.append(new)
        if copy_src:
            cs = torch.tensor(copy_src, dtype=torch.int32, device=self.device)
            cd = torch.tensor(copy_dst, dtype=torch.int32, device=self.device)
            for li in range(self.n_layers):
                K.page_copy(self.k_pool[li], self.k_pool[li], cs, cd)
                K.page_copy(self.v_pool[li], self.v_pool[li], cs, cd)
        self._len[dst] = plen

    # ------------------------------------------------------------------ pool
    def _grow_pool(self, need_free: int) -> None:
        self._device_step_ok = False
        old = self.pages.num_pages
        new = max(2 * old, old + need_free - self.pages.free_pages)
        shape = (self.n_layers, new, self.n_kv_heads, self.page_size, self.head_dim)
        for name in ("k_pool", "v_pool"):
            src = getattr(self, name)
            dst = torch.zeros(shape, device=self.device, dtype=self.dtype)
            dst[:, :old] = src
            setattr(self, name, dst)
        self.pages.grow_pool(new)

    def _stage(self, n_int32: int) -> torch.Tensor:
        """A pinned int32 staging buffer that no in-flight copy still reads."""
        i = self._turn
        self._turn ^= 1
        buf = self._staging[i]
        ev = self._staging_ev[i]
        if ev is not None:
            ev.synchronize()
        if buf is None or buf.numel() < n_int32:
            buf = torch.empty(max(n_int32, 1024), dtype=torch.int32, pin_memory=True)
            self._staging[i] = buf
        return buf, i

    # --------------------------------------------------------------- forward
    def prepare(self, lengths, S: int):
        """Host bookkeeping of one call: allocate pages and upload positions,
        slots, lengths and (if changed) the block table in one copy.
        Returns the device views ``(q_pos [B,S], kv_len [B], slot [B*S], max_kv)``."""
        B = self.B
        n = np.asarray(lengths, dtype=np.int64).reshape(-1)
        if n.shape[0] != B:
            raise ValueError(f"lengths has {n.shape[0]} entries, session batch_size={B}.")
        if (n < 0).any() or (n > S).any():
            raise ValueError(f"lengths must satisfy 0 <= lengths[b] <= S={S}.")
        new_len = self._len + n
        add = self.pages.pages_needed(new_len)
        total = int(add.sum())
        if total > self.pages.free_pages:
            self._grow_pool(total)
        self.pages.allocate(add)

        if S == 1:
            # A decode step: one position per row, no [B, S] broadcasting.
            pos = self._len - 1 + n
            q_pos = np.maximum(pos, 0)
            slot = np.full(B, -1, dtype=np.int64)
            live = np.flatnonzero(n)
            if live.size:
                slot[live] = self.pages.slots(live, pos[live])
        else:
            col = np.arange(S, dtype=np.int64)[None, :]
            pad = (S - n)[:, None]
            pos = self._len[:, None] + col - pad
            q_pos = np.maximum(pos, 0)
            real = col >= pad
            rows = np.broadcast_to(np.arange(B)[:, None], (B, S))
            slot = np.full((B, S), -1, dtype=np.int64)
            if real.any():
                slot[real] = self.pages.slots(rows[real], pos[real])

        bt_changed = self.pages.dirty or bool(self._pending_reset.any())
        width = self.pages.max_pages
        n_meta = 2 * B * S + B + (B * width if bt_changed else 0)
        buf, i = self._stage(n_meta)
        host = buf.numpy()
        o = 0
        host[o:o + B * S] = q_pos.reshape(-1)
        o += B * S
        host[o:o + B] = new_len
        o += B
        host[o:o + B * S] = slot.reshape(-1)
        o += B * S
        if bt_changed:
            host[o:o + B * width] = self.pages.table.reshape(-1)
        if self._meta_dev.numel() < n_meta:
            self._meta_dev = torch.empty(max(n_meta, 2 * self._meta_dev.numel()), dtype=torch.int32,
                                         device=self.device)
            self._graph = None  # its captured views point at the old buffer
            self._step_graph = None
        dev = self._meta_dev
        dev[:n_meta].copy_(buf[:n_meta], non_blocking=True)
        ev = self._staging_ev[i]
        if ev is None:
            ev = self._staging_ev[i] = torch.cuda.Event()
        ev.record()
        q_pos_d = dev[:B * S].view(B, S)
        kv_len_d = dev[B * S:B * S + B]
        slot_d = dev[B * S + B:2 * B * S + B]
        if bt_changed:
            if self._bt_dev.shape[1] != width:
                self._bt_dev = torch.empty((B, width), dtype=torch.int32, device=self.device)
            self._bt_dev.copy_(dev[2 * B * S + B:n_meta].view(B, width))
            self.pages.dirty = False
            self._pending_reset[:] = False
        self._len = new_len
        self._device_step_ok = S == 1
        return q_pos_d, kv_len_d, slot_d, int(new_len.max()) if B else 0

    def _device_step(self, lengths) -> bool:
        """A step of at most one token per row whose metadata the device makes
        (K8): the host only opens the pages this step's tokens start and, when
        anything but a plain append happens, uploads one code per row. False
        (nothing changed) when the host path must run instead: a row appends
        more than one token, the device metadata is stale, or the new pages
        would not fit the pool or the block table's width."""
        B, P, pages = self.B, self.page_size, self.pages
        if not self._device_step_ok or pages.dirty:
            return False
        n = None  # every row appends one token
        if isinstance(lengths, list):
            if len(lengths) != B:
                return False
            if lengths.count(1) != B:
                if lengths.count(1) + lengths.count(0) != B:
                    return False
                n = np.asarray(lengths, dtype=np.int64)
        else:
            a = np.asarray(lengths).reshape(-1)
            if a.shape[0] != B or not bool(((a == 0) | (a == 1)).all()):
                return False
            if not bool((a == 1).all()):
                n = a.astype(np.int64)
        grows = pages.npages * P <= self._len
        opening = np.flatnonzero(grows if n is None else grows & (n == 1))
        if opening.size:
            if opening.size > pages.free_pages or int(pages.npages[opening].max()) >= pages.max_pages:
                return False
        pend = self._pending_reset
        any_pend = bool(pend.any())
        coded = opening.size > 0 or n is not None or any_pend
        if coded:
            buf, i = self._stage(B)
            host = buf.numpy()[:B]
            host.fill(-1)
            if n is not None:
                host[n == 0] = -2
                if any_pend:
                    host[pend & (n == 0)] = -3
            if opening.size:
                ids = pages.open_pages(opening)
                if any_pend:
                    ids = np.where(pend[opening], ids | _STEP_RESTART, ids)
                host[opening] = ids
            pend[:] = False
            self._new_page_dev.copy_(buf[:B], non_blocking=True)
            ev = self._staging_ev[i]
            if ev is None:
                ev = self._staging_ev[i] = torch.cuda.Event()
            ev.record()
        if self._step_args is None:
            dev = self._meta_dev
            self._step_args = K.decode_step_meta_args(self._bt_dev, dev[:B], dev[B:2 * B], dev[2 * B:3 * B], P,
                                                      self._new_page_dev)
        K.decode_step_meta_launch(self._step_args, coded, torch.cuda.current_stream().cuda_stream)
        self._len = self._len + (1 if n is None else n)
        return True

    @torch.no_grad()
    def forward(self, *, embeds: torch.Tensor, lengths, output_hidden_states: bool = False):
        """Decode one chunk per sequence (left-padded ``embeds [B, S, D]``,
        ``lengths[b]`` real trailing tokens per row). Returns hidden states
        ``[B, S, D]`` (pad positions meaningless) and, with
        ``output_hidden_states=True``, the tuple of per-layer hidden states."""
        with nvtx_range("decode_step" if embeds.shape[1] == 1 else "prefill"):
            return self._forward(embeds, lengths, output_hidden_states)

    def _forward(self, embeds, lengths, output_hidden_states):
        B, S, D = embeds.shape
        if B != self.B:
            raise ValueError(f"Session was created for batch_size={self.B}, got {B}.")
        x = embeds.to(self.device, self.dtype).reshape(B * S, D).contiguous()
        if (S == 1 and B > 0 and self.use_graphs and self.use_device_step and self._graph is not None
                and not output_hidden_states and self.attn_events is None
                and not torch.cuda.is_current_stream_capturing()):
            for lw in self._layers:
                lw.refresh()
            key = (self.k_pool.data_ptr(), self._bt_dev.data_ptr(), self._meta_dev.data_ptr(), self.cap,
                   tuple(lw.version for lw in self._layers))
            if key == self._graph_key and self._device_step(lengths):
                self._graph_x.copy_(x)
                self._graph.replay()
                K._count(self._graph_launches)
                return self._final(self._graph_out.view(B, S, D), copy=True)
        q_pos, kv_len, slot, max_kv = self.prepare(lengths, S)
        if B == 0 or S == 0:
            h = x.view(B, S, D)
            return (h, tuple(h for _ in range(self.n_layers))) if output_hidden_states else h
        graphable = (S == 1 and self.use_graphs and not output_hidden_states and self.attn_events is None
                     and not torch.cuda.is_current_stream_capturing())
        if not graphable:
            out = self._body(x, q_pos, kv_len, slot, S, output_hidden_states)
            if output_hidden_states:
                h, hiddens = out
                return self._final(h.view(B, S, D)), tuple(t.view(B, S, D).to(self.dtype) for t in hiddens)
            return self._final(out.view(B, S, D))
        for lw in self._layers:
            lw.refresh()
        key = (self.k_pool.data_ptr(), self._bt_dev.data_ptr(), self._meta_dev.data_ptr(), self.cap,
               tuple(lw.version for lw in self._layers))
        if self._graph is None or self._graph_key != key:
            if not self._graph_warm:
                # Eager warm-up: allocates the workspace and initialises cuBLAS.
                self._graph_warm = True
                return self._final(self._body(x, q_pos, kv_len, slot, 1, False).view(B, S, D))
            self._graph = None
            self._graph_x = torch.empty_like(x)
            self._graph_x.copy_(x)
            graph = torch.cuda.CUDAGraph()
            n0 = K.launch_count[0]
            with torch.cuda.graph(graph):
                self._graph_out = self._body(self._graph_x, q_pos, kv_len, slot, 1, False)
            self._graph_launches = K.launch_count[0] - n0
            K.launch_count[0] = n0
            self._graph, self._graph_key = graph, key
            self._step_args = None
        else:
            self._graph_x.copy_(x)
        self._graph.replay()
        K._count(self._graph_launches)
        return self._final(self._graph_out.view(B, S, D), copy=True)

    def _final(self, h: torch.Tensor, copy: bool = False) -> torch.Tensor:
        """The model's final norm, in the model's dtype (a fresh tensor when
        ``h`` is a graph buffer)."""
        h = self.model.norm(h)
        if h.dtype != self.dtype:
            return h.to(self.dtype)
        return h.clone() if copy else h

    def _graph_key_now(self):
        for lw in self._layers:
            lw.refresh()
        return (self.k_pool.data_ptr(), self._bt_dev.data_ptr(), self._meta_dev.data_ptr(), self.cap,
                tuple(lw.version for lw in self._layers))

    @torch.no_grad()
    def decode_step(self, ids: torch.Tensor, lengths, embed, head):
        """One step of at most one token per row, from token ids to the
        head's output, replayed as ONE CUDA graph.

        The reference's caller runs this step as separate pieces: the encoder's
        embedding gather, ``FlexDecodeSession.forward`` with S = 1, the fp32
        head (models/heads/swiglu.py:71-74) and ``get_action``'s argmax
        (models/base.py:1065-1106). Here the gather, the layer stack (K1/K2
        and the GEMMs), the final norm and ``head`` are captured together, so
        a step costs the host one device-step metadata launch (K8) and one
        graph launch.

        Args:
            ids: ``[B]`` token ids on the device (any value for rows that sit
                out); copied into the graph's input buffer.
            lengths: ``[B]`` 0/1 tokens per row (list or array).
            embed: ``embed(ids [B]) -> [B, D]`` in the backbone's dtype.
            head: ``head(h [B, D]) -> tensor`` (e.g. action values' argmax).
            Both must be device-only work (no host syncs) and the same
            callables from step to step (a new one is captured anew).

        Returns the head's output: a buffer of the graph, overwritten by the
        next step (copy it out before then). A step whose metadata the device
        cannot make (after a multi-token call, a fork or pool growth) is
        prepared on the host and replays the same graph; the first step runs
        eagerly and the second captures the graph, with the same results.
        """
        with nvtx_range("decode_step_graph"):
            return self._decode_step(ids, lengths, embed, head)

    def _decode_step(self, ids, lengths, embed, head):
        B = self.B
        if ids.shape[0] != B:
            raise ValueError(f"Session was created for batch_size={B}, got {ids.shape[0]} ids.")
        use_graph = (B > 0 and self.use_graphs and self.use_device_step and self.attn_events is None
                     and not torch.cuda.is_current_stream_capturing())
        if use_graph and self._step_graph is not None:
            key = (self._graph_key_now(), id(embed), id(head))
            if key == self._step_graph_key and self._device_step(lengths):
                self._step_ids.copy_(ids, non_blocking=True)
                self._step_graph.replay()
                K._count(self._step_launches)
                return self._step_out
        if not use_graph:
            h = self.forward(embeds=embed(ids).view(B, 1, -1), lengths=lengths)
            return head(h[:, -1])
        q_pos, kv_len, slot, _ = self.prepare(lengths, 1)
        if self._step_graph is not None and (self._graph_key_now(), id(embed), id(head)) == self._step_graph_key:
            # Host-prepared metadata landed in the buffers the graph reads.
            self._step_ids.copy_(ids, non_blocking=True)
            self._step_graph.replay()
            K._count(self._step_launches)
            return self._step_out
        if not self._step_graph_warm:
            # Eager warm-up: allocates the workspace and initialises cuBLAS.
            self._step_graph_warm = True
            x = embed(ids).to(self.device, self.dtype).reshape(B, -1).contiguous()
            h = self._body(x, q_pos, kv_len, slot, 1, False)
            return head(self.model.norm(h.view(B, 1, -1))[:, -1])
        self._step_graph = None
        self._step_ids = torch.empty_like(ids, device=self.device)
        self._step_ids.copy_(ids)
        graph = torch.cuda.CUDAGraph()
        n0 = K.launch_count[0]
        with torch.cuda.graph(graph):
            xs = embed(self._step_ids).to(self.dtype).reshape(B, -1)
            h = self._body(xs, q_pos, kv_len, slot, 1, False)
            self._step_out = head(self.model.norm(h.view(B, 1, -1))[:, -1])
        self._step_launches = K.launch_count[0] - n0
        K.launch_count[0] = n0
        self._step_graph = graph
        self._step_graph_key = (self._graph_key_now(), id(embed), id(head))
        self._step_args = None
        graph.replay()  # capturing ran nothing: this step runs now
        K._count(self._step_launches)
        return self._step_out

    def _body(self, x, q_pos, kv_len, slot, S, output_hidden_states):
        """The layer stack for flattened ``x [B*S, D]``; returns the last hidden
        state (before the final norm) and, if asked, every layer's."""
        if self.residual_fp32:
            return self._body_f32(x, q_pos, kv_len, slot, S, output_hidden_states)
        B = self.B
        Hq, Hkv, hd = self.n_heads, self.n_kv_heads, self.head_dim
        split = self._plan(kv_len, S)
        q_pos_flat = q_pos.reshape(-1)

        resid, delta = x, None
        hiddens = []
        for li, lw in enumerate(self._layers):
            lw.refresh()
            if delta is None:
                _, hn = K.rmsnorm(resid, lw.in_w, lw.in_eps)
            else:
                resid, hn = K.rmsnorm(delta, lw.in_w, lw.in_eps, residual=resid)
            qkv = F.linear(hn, lw.wqkv, lw.bqkv)
            q = K.kv_append(qkv, q_pos_flat, Hq, Hkv, hd, self.inv_freq, self.attention_scaling,
                            lw.q_norm_w, lw.k_norm_w, lw.qk_eps, slot=slot,
                            k_pool=self.k_pool[li], v_pool=self.v_pool[li])
            o = self._attend(q.view(B, S, Hq, hd), li, lw.scale, q_pos, kv_len, split)
            a = lw.o_proj(o.view(B * S, Hq * hd))
            resid, hn2 = K.rmsnorm(a, lw.post_w, lw.post_eps, residual=resid)
            delta = lw.down(K.silu_mul(F.linear(hn2, lw.wgu, lw.bgu)))
            if output_hidden_states:
                hiddens.append(resid + delta)
        h = hiddens[-1] if output_hidden_states else resid + delta
        if output_hidden_states:
            return h, hiddens
        return h

    def _plan(self, kv_len, S):
        """Split-KV work list for this call (once, shared by every layer)."""
        B, Hkv, hd = self.B, self.n_kv_heads, self.head_dim
        R = (self.n_heads // Hkv) * S
        split = R <= 16
        if split:
            need = K.decode_workspace_bytes(B, Hkv, R, hd, self.cap)
            if self._workspace.numel() < need:
                self._workspace = torch.empty(need, dtype=torch.uint8, device=self.device)
                self._graph = None
                self._step_graph = None
            # One-token steps see every cached slot, so chunks that forked
            # rows hold on the same pages can share one work item.
            K.decode_plan(kv_len, Hkv, R, hd, self.cap, self._workspace,
                          block_table=self._bt_dev if S == 1 else None, page_size=self.page_size)
        elif self._workspace.numel() < 256:  # prefill chunks keep a tile counter in it
            self._workspace = torch.empty(256, dtype=torch.uint8, device=self.device)
            self._graph = None
            self._step_graph = None
        return split

    def _fused_qkv(self, lw, tokens: int) -> bool:
        """Whether this layer's QKV projection runs as K13: asked for
        (``fused_qkv``), bf16 weights (and norms and bias), heads filling whole
        128-column tiles, at most FUSED_QKV_MAX_TOKENS tokens."""
        if not self.fused_qkv:
            return False
        n = lw.wqkv.shape[0]
        if tokens > FUSED_QKV_MAX_TOKENS or n % 128 or lw.wqkv.shape[1] % 8 or lw.wqkv.dtype != torch.bfloat16:
            return False
        return all(t is None or t.dtype == torch.bfloat16 for t in (lw.bqkv, lw.q_norm_w, lw.k_norm_w))

    def _body_f32(self, x, q_pos, kv_len, slot, S, output_hidden_states):
        """The layer stack with an fp32 residual stream: the embeddings enter
        it exactly, every residual add and every projection output stays
        fp32 (cuBLAS bf16 GEMMs with fp32 outputs), and only the GEMM inputs
        are rounded to bf16 (the normalised activations, the attention output,
        the SiLU product) together with the q/k/v the attention kernel and the
        bf16 page pool take. The reference's bf16 modules round the stream at
        every add and every op output instead; against the fp32 forward this
        path's greedy actions agree more often (measured on the decode
        benchmark's model shape). Returns fp32 hidden states."""
        B = self.B
        Hq, Hkv, hd = self.n_heads, self.n_kv_heads, self.head_dim
        split = self._plan(kv_len, S)
        q_pos_flat = q_pos.reshape(-1)
        resid, delta = None, None
        hiddens = []
        rope = None
        for li, lw in enumerate(self._layers):
            lw.refresh()
            if resid is None:
                resid, hn = K.rmsnorm_f32(x, lw.in_w, lw.in_eps)
            else:
                resid, hn = K.rmsnorm_f32(resid, lw.in_w, lw.in_eps, delta=delta, sum_out=resid)
            if self._fused_qkv(lw, B * S):
                # K13: the QKV GEMM with K2 as its epilogue; one RoPE table
                # for the step's tokens serves every layer.
                if rope is None:
                    rope = K.rope_table(q_pos_flat, self.inv_freq, hd, self.attention_scaling)
                q = K.qkv_append(hn, lw.wqkv, lw.bqkv, rope, Hq, Hkv, hd, lw.q_norm_w, lw.k_norm_w, lw.qk_eps,
                                 slot=slot, k_pool=self.k_pool[li], v_pool=self.v_pool[li])
            else:
                qkv = _mm_f32(hn, lw.wqkv, lw.bqkv)
                q = K.kv_append(qkv, q_pos_flat, Hq, Hkv, hd, self.inv_freq, self.attention_scaling,
                                lw.q_norm_w, lw.k_norm_w, lw.qk_eps, slot=slot,
                                k_pool=self.k_pool[li], v_pool=self.v_pool[li])
            o = self._attend(q.view(B, S, Hq, hd), li, lw.scale, q_pos, kv_len, split)
            a = _mm_f32(o.view(B * S, Hq * hd), lw.o_proj.weight, lw.o_proj.bias)
            resid, hn2 = K.rmsnorm_f32(resid, lw.post_w, lw.post_eps, delta=a, sum_out=resid)
            delta = _mm_f32(K.silu_mul_f32(_mm_f32(hn2, lw.wgu, lw.bgu)), lw.down.weight, lw.down.bias)
            if output_hidden_states:
                hiddens.append(resid + delta)
        h = hiddens[-1] if output_hidden_states else resid + delta
        if output_hidden_states:
            return h, hiddens
        return h


# Largest token count of one forward whose QKV projection runs as K13 (the
# GEMM with K2 as its epilogue) when the session asks for it: every decode
# step and short chunk; longer prefill chunks keep cuBLAS followed by K2.
FUSED_QKV_MAX_TOKENS = 8192


def _mm_f32(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ b)`` of bf16 operands with an fp32 result (cuBLAS accumulates
    in fp32 either way; the output is just not rounded to bf16)."""
    y = torch.mm(x, w.t(), out_dtype=torch.float32)
    return y if b is None else y + b.float()


# The reference's name, so callers and tests written against it keep working.
FlexDecodeSession = PagedDecodeSession
