"""Packed segment-causal forward — drop-in for mouse-core's ``flex_packed_forward``.

Reference: ``flex_packed_forward`` (src/mouse_core/models/backbone/
flex_train.py:51-157). Same keyword signature, same ``ValueError``s, same
result: a decoder pass over one flat stream ``embeds [L, D]`` where token ``i``
attends token ``j`` iff ``j <= i`` and ``sequence_ids[i] == sequence_ids[j]``,
with RoPE positions restarting at every run of ``sequence_ids``; autograd
reaches ``embeds`` and every weight.

B200 machinery instead of the reference's BlockMask + compiled
FlexAttention:

* K7 (``mb_segment_meta``) computes the position ids (bit-exact with the
  reference's cummax formula), each token's run start/end and each 128-token
  query tile's first visible key, in one pass; no ``[L, L]`` mask exists.
* The attention core is the tcgen05 kernel pair K5 (forward, saves the log2
  softmax denominator) / K6 (backward: deterministic dK/dV and dQ kernels)
  behind ``torch.autograd.Function``.
* K4 element-wise kernels replace the layer's eager bf16 glue: RMSNorm
  forward/backward (input, post-attention and final norms), the per-head
  q/k RMSNorm + RoPE read straight out of one fused QKV projection (and its
  gradient written straight back into the fused QKV gradient), and the
  SiLU-gated product over one fused gate|up projection. The projections are
  cuBLAS GEMMs over the concatenated weights. A model whose shapes the K4
  kernels are not built for (hidden size not a multiple of 256 up to 2048,
  biased projections, an activation other than SiLU) keeps those pieces on
  its own transformers modules.

Ids that are not sorted (one id owning several runs) are made contiguous by a
stable sort before the attention call and scattered back after it, which
keeps the reference's id-equality mask; positions still restart per run.
"""

from __future__ import annotations

from typing import Any, cast

import numpy as np
import torch

from mouse_core_b200 import kernels as K
from mouse_core_b200.trace import nvtx_range


class _SegmentAttention(torch.autograd.Function):
    """out = segment-causal GQA attention of ``q [L,Hq,hd]`` over ``k, v [L,Hkv,hd]``."""

    @staticmethod
    def forward(ctx, q, k, v, run_start, run_end, tile_lo, scale, pair_off, n_pairs):
        q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
        with nvtx_range("packed_attention_fwd"):
            out, lse = K.varlen_attention_fwd(q, k, v, run_start, tile_lo, scale)
        ctx.save_for_backward(q, k, v, out, lse, run_start, run_end, tile_lo)
        ctx.scale = scale
        ctx.pair_off, ctx.n_pairs = pair_off, n_pairs
        return out

    @staticmethod
    def backward(ctx, dout):
        q, k, v, out, lse, run_start, run_end, tile_lo = ctx.saved_tensors
        with nvtx_range("packed_attention_bwd"):
            dq, dk, dv = K.varlen_attention_bwd(q, k, v, out, dout.contiguous(), lse, run_start, run_end, ctx.scale,
                                                tile_lo=tile_lo, pair_off=ctx.pair_off, n_pairs=ctx.n_pairs)
        return dq, dk, dv, None, None, None, None, None, None


def segment_attention(q, k, v, run_start, run_end, tile_lo, scale, pair_off=None, n_pairs=None):
    """Autograd-aware K5/K6 attention (``q [L,Hq,hd]``, ``k, v [L,Hkv,hd]``, bf16).
    With ``pair_off``/``n_pairs`` (``SegmentLayout``) the backward stores dS
    instead of recomputing it for dQ."""
    return _SegmentAttention.apply(q, k, v, run_start, run_end, tile_lo, scale, pair_off, n_pairs)


def pair_count(sequence_ids: np.ndarray) -> int:
    """Number of (128-query tile, 128-key tile) pairs the segment-causal
    attention visits over ``sequence_ids`` whose every id is one contiguous
    run: query tile ``i`` visits key tiles ``run_start(128 i) // 128 .. i``."""
    ids = np.asarray(sequence_ids).reshape(-1)
    L = ids.shape[0]
    if L == 0:
        return 0
    T = (L + 127) // 128
    starts = np.flatnonzero(np.r_[True, ids[1:] != ids[:-1]])
    first = np.arange(T, dtype=np.int64) * 128
    rs = starts[np.searchsorted(starts, first, side="right") - 1]
    return int((np.arange(T, dtype=np.int64) - rs // 128 + 1).sum())


class SegmentLayout:
    """Per-stream metadata shared by every layer of one packed forward."""

    def __init__(self, sequence_ids: torch.Tensor, device: torch.device):
        seq = sequence_ids.to(device=device, dtype=torch.long).contiguous()
        self.L = seq.shape[0]
        pos, rs, tl, flags, re = K.segment_meta(seq, tile=128, with_run_end=True)
        self.position_ids = pos
        if sequence_ids.device.type == "cpu":
            unsorted = bool((sequence_ids[1:] < sequence_ids[:-1]).any()) if self.L > 1 else False
        else:
            unsorted = bool(flags.item())
        self.perm = None
        self.inv = None
        if unsorted:
            # Make every id one run: stable sort keeps each id's token order.
            self.perm = torch.sort(seq, stable=True).indices
            self.inv = torch.empty_like(self.perm)
            self.inv[self.perm] = torch.arange(self.L, device=device)
            _, rs, tl, _, re = K.segment_meta(seq[self.perm].contiguous(), tile=128, with_run_end=True)
        self.run_start, self.run_end, self.tile_lo = rs, re, tl
        # (query tile, key tile) pairs of the stored-dS backward: counted on
        # the host from host ids, else read back once per layout.
        self.pair_off = K.varlen_pair_offsets(tl, self.L)
        if sequence_ids.device.type == "cpu":
            ids = sequence_ids.numpy()
            self.n_pairs = pair_count(np.sort(ids, kind="stable") if unsorted else ids)
        else:
            self.n_pairs = int(self.pair_off[-1].item())

    def attend(self, q, k, v, scale):
        if self.perm is None:
            return segment_attention(q, k, v, self.run_start, self.run_end, self.tile_lo, scale, self.pair_off,
                                     self.n_pairs)
        o = segment_attention(q[self.perm], k[self.perm], v[self.perm], self.run_start, self.run_end,
                              self.tile_lo, scale, self.pair_off, self.n_pairs)
        return o[self.inv]


def _rotate_half(x):
    half = x.shape[-1] // 2
    return torch.cat((-x[..., half:], x[..., :half]), dim=-1)


class _RMSNorm(torch.autograd.Function):
    """``weight * bf16(x * rsqrt(mean(x^2) + eps))`` over the last dim (K4)."""

    @staticmethod
    def forward(ctx, x, weight, eps):
        x = x.contiguous()
        y, rstd = K.rmsnorm_fwd(x, weight, eps)
        ctx.save_for_backward(x, weight, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, weight, rstd = ctx.saved_tensors
        dx, dw = K.rmsnorm_bwd(dy.contiguous(), x, weight, rstd)
        return dx, dw.to(weight.dtype), None


class _AddRMSNorm(torch.autograd.Function):
    """``(s, y)``: ``s = bf16(x + residual)`` (the decoder layer's residual
    add) and ``y = RMSNorm(s)`` in one pass (K4); the backward adds the
    gradient reaching ``s`` along the residual path into the norm's input
    gradient in the same pass."""

    @staticmethod
    def forward(ctx, x, residual, weight, eps):
        ctx.set_materialize_grads(False)
        total, y, rstd = K.add_rmsnorm_fwd(x.contiguous(), residual.contiguous(), weight, eps)
        ctx.save_for_backward(total, weight, rstd)
        return total, y

    @staticmethod
    def backward(ctx, dtotal, dy):
        total, weight, rstd = ctx.saved_tensors
        if dy is None:
            return dtotal, dtotal, None, None
        dx, dw = K.rmsnorm_bwd(dy.contiguous(), total, weight, rstd,
                               None if dtotal is None else dtotal.contiguous())
        return dx, dx, dw.to(weight.dtype), None


class _QKVHeads(torch.autograd.Function):
    """Split a fused QKV projection ``[L, (Hq + 2 Hkv) hd]`` into attention
    inputs in one pass: q and k through the per-head RMSNorm (when the model
    has one) and rotate-half RoPE, v as is (K4)."""

    @staticmethod
    def forward(ctx, qkv, q_w, k_w, cos, sin, q_eps, k_eps, Hq, Hkv, hd):
        q, k, v, q_rstd, k_rstd = K.qkv_heads_fwd(qkv, Hq, Hkv, hd, cos, sin, q_w, k_w, q_eps, k_eps)
        ctx.save_for_backward(qkv, q_w, k_w, cos, sin, q_rstd, k_rstd)
        return q, k, v

    @staticmethod
    def backward(ctx, dq, dk, dv):
        qkv, q_w, k_w, cos, sin, q_rstd, k_rstd = ctx.saved_tensors
        dqkv, dqw, dkw = K.qkv_heads_bwd(dq.contiguous(), dk.contiguous(), dv.contiguous(), qkv, cos, sin, q_w,
                                         k_w, q_rstd, k_rstd)
        return (dqkv, None if dqw is None else dqw.to(q_w.dtype), None if dkw is None else dkw.to(k_w.dtype),
                None, None, None, None, None, None, None)


class _SiluMul(torch.autograd.Function):
    """``bf16(silu(gate)) * up`` over a fused ``gate|up`` projection ``[L, 2I]`` (K4)."""

    @staticmethod
    def forward(ctx, gate_up):
        gate_up = gate_up.contiguous()
        ctx.save_for_backward(gate_up)
        return K.silu_mul(gate_up)

    @staticmethod
    def backward(ctx, dh):
        (gate_up,) = ctx.saved_tensors
        return K.silu_mul_bwd(gate_up, dh.contiguous())


class _CatLinear(torch.autograd.Function):
    """``x @ cat(weights)^T`` with the concatenated weight built once per
    weight version (the rows of one step share it) instead of on every
    forward; the backward splits dW back onto the separate weights."""

    @staticmethod
    def forward(ctx, x, w_cat, *weights):
        ctx.save_for_backward(x, w_cat)
        ctx.rows = [w.shape[0] for w in weights]
        return torch.nn.functional.linear(x, w_cat)

    @staticmethod
    def backward(ctx, dy):
        x, w_cat = ctx.saved_tensors
        dy2 = dy.reshape(-1, dy.shape[-1])
        dx = (dy2 @ w_cat).view(x.shape) if ctx.needs_input_grad[0] else None
        dw = dy2.t() @ x.reshape(-1, x.shape[-1])
        return (dx, None, *torch.split(dw, ctx.rows, dim=0))


def _cat_linear(owner, key, x, weights):
    """``linear(x, cat(weights))`` through _CatLinear, the concatenation
    cached on ``owner`` under ``key`` and rebuilt when a weight's storage or
    version changes (an optimizer step updates them in place)."""
    cache = owner.__dict__.setdefault("_mb_cat_cache", {})
    tag = tuple((w.data_ptr(), w._version, w.dtype, tuple(w.shape)) for w in weights)
    hit = cache.get(key)
    if hit is None or hit[0] != tag:
        with torch.no_grad():
            hit = (tag, torch.cat([w.detach() for w in weights], dim=0))
        cache[key] = hit
    return _CatLinear.apply(x, hit[1], *weights)


def _k4_norm(module, x) -> bool:
    D = x.shape[-1]
    return hasattr(module, "variance_epsilon") and D % 256 == 0 and D <= 2048


def _norm(module, x):
    """The model's RMSNorm through K4 when its width is supported (an
    ``nn.Identity`` final norm, as the backbones install, stays as is)."""
    if _k4_norm(module, x):
        return _RMSNorm.apply(x, module.weight, float(module.variance_epsilon))
    return module(x)


def _add_norm(module, residual, delta):
    """``(h, norm(h))`` for ``h = residual + delta``: one K4 pass when the
    norm is a supported RMSNorm, else the add and the module."""
    if _k4_norm(module, residual):
        return _AddRMSNorm.apply(delta, residual, module.weight, float(module.variance_epsilon))
    h = residual + delta
    return h, _norm(module, h)


def _fused_attention_inputs(attn):
    """True when the attention block has bias-free q/k/v projections."""
    return all(getattr(attn, n).bias is None for n in ("q_proj", "k_proj", "v_proj"))


def _fused_mlp(mlp, cfg):
    return (getattr(cfg, "hidden_act", "silu") == "silu" and mlp.gate_proj.bias is None
            and mlp.up_proj.bias is None)


def flex_packed_forward(*, model: torch.nn.Module, embeds: torch.Tensor, sequence_ids: torch.Tensor,
                        output_hidden_states: bool = False):
    """Full pass over a flat packed sequence ``embeds [L, D]``.

    Attention is causal within positions that share ``sequence_ids``; RoPE
    positions restart at each new run of ``sequence_ids``. Returns ``[L, D]``
    (and the tuple of per-layer hidden states when ``output_hidden_states``).
    """
    if embeds.ndim != 2:
        raise ValueError(f"embeds must be [L, D], got shape {tuple(embeds.shape)}")
    L, _D = embeds.shape
    if sequence_ids.shape != (L,):
        raise ValueError("sequence_ids must have shape [L]")
    hf = cast(Any, model)
    param = next(hf.parameters())
    device, dtype = param.device, param.dtype
    if device.type != "cuda":
        raise RuntimeError(f"mouse_core_b200 packed attention runs on a CUDA device (B200) only; model is on {device}")
    if dtype != torch.bfloat16:
        raise TypeError("mouse_core_b200 kernels compute in bfloat16; move the backbone to torch.bfloat16 "
                        f"(got {dtype})")
    cfg = hf.config
    n_heads = int(cfg.num_attention_heads)
    n_kv = int(cfg.num_key_value_heads)
    hd = int(getattr(cfg, "head_dim", None) or cfg.hidden_size // n_heads)
    if hd not in (64, 128):
        raise ValueError(f"head_dim must be 64 or 128 for the sm_100a kernels, got {hd}")

    x = embeds.to(device=device, dtype=dtype)
    if L == 0:
        h = hf.norm(x)
        return (h, tuple(x for _ in hf.layers)) if output_hidden_states else h
    layout = SegmentLayout(sequence_ids, device)
    cos, sin = hf.rotary_emb(x.unsqueeze(0), layout.position_ids.unsqueeze(0))
    cos, sin = cos[0].contiguous(), sin[0].contiguous()  # [L, hd]

    h = x
    hiddens = []
    pending = None  # the last MLP output, not yet added to h (fused into the next norm)
    for layer in hf.layers:
        if pending is None:
            hn = _norm(layer.input_layernorm, h)
        else:
            h, hn = _add_norm(layer.input_layernorm, h, pending)
        residual = h
        attn = layer.self_attn
        q_norm = getattr(attn, "q_norm", None)
        if _fused_attention_inputs(attn):
            qkv = _cat_linear(attn, "qkv", hn, (attn.q_proj.weight, attn.k_proj.weight, attn.v_proj.weight))
            if q_norm is not None:
                q, k, v = _QKVHeads.apply(qkv, q_norm.weight, attn.k_norm.weight, cos, sin,
                                          float(q_norm.variance_epsilon), float(attn.k_norm.variance_epsilon),
                                          n_heads, n_kv, hd)
            else:
                q, k, v = _QKVHeads.apply(qkv, None, None, cos, sin, 0.0, 0.0, n_heads, n_kv, hd)
        else:
            q = attn.q_proj(hn).view(L, n_heads, hd)
            k = attn.k_proj(hn).view(L, n_kv, hd)
            if q_norm is not None:
                q = q_norm(q)
                k = attn.k_norm(k)
            v = attn.v_proj(hn).view(L, n_kv, hd)
            c, s_ = cos.unsqueeze(1), sin.unsqueeze(1)
            q = q * c + _rotate_half(q) * s_
            k = k * c + _rotate_half(k) * s_
        o = layout.attend(q, k, v, float(attn.scaling))
        mlp = layer.mlp
        h, hn = _add_norm(layer.post_attention_layernorm, residual, attn.o_proj(o.reshape(L, n_heads * hd)))
        if _fused_mlp(mlp, cfg):
            gate_up = _cat_linear(mlp, "gate_up", hn, (mlp.gate_proj.weight, mlp.up_proj.weight))
            pending = mlp.down_proj(_SiluMul.apply(gate_up))
        else:
            pending = mlp(hn)
        if output_hidden_states:
            h = h + pending
            pending = None
            hiddens.append(h)
    if pending is None:
        h = _norm(hf.norm, h)
    else:
        h = _add_norm(hf.norm, h, pending)[1]
    if output_hidden_states:
        return h, tuple(hiddens)
    return h
