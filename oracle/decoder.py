"""Float64 restatement of the decoder-layer loops on the hot path.

Test infrastructure (see ``oracle/__init__.py``).

``DecodeSessionOracle.forward`` restates ``FlexDecodeSession.forward``
(backbone/flex_decode.py:153-240) and ``packed_forward`` restates
``flex_packed_forward`` (backbone/flex_train.py:51-157). The per-layer pieces
restate the transformers modules those loops call (installed transformers
5.5.0): RMSNorm with float32-style variance (qwen3/modeling_qwen3.py:50-67),
rotate-half RoPE (llama/modeling_llama.py apply_rotary_pos_emb), SiLU-gated
MLP, GQA ``q_head // group`` head sharing and ``scaling = head_dim ** -0.5``.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.attention import cached_decode_attention, packed_attention_fwd
from oracle.policy import decode_positions, position_ids


def rms_norm(x, w, eps):
    var = np.mean(x * x, axis=-1, keepdims=True)
    y = x / np.sqrt(var + eps)
    return y * w if w is not None else y


def rope(x, pos, inv_freq, attention_scaling=1.0):
    """Rotate-half RoPE of ``x [..., T, H, hd]`` at integer positions
    ``pos [..., T]`` with ``inv_freq [hd/2]``."""
    freqs = np.asarray(pos, dtype=np.float64)[..., None] * np.asarray(inv_freq, dtype=np.float64)
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos = (np.cos(emb) * attention_scaling)[..., None, :]
    sin = (np.sin(emb) * attention_scaling)[..., None, :]
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return x * cos + rot * sin


def silu(x):
    return x / (1.0 + np.exp(-x))


@dataclass
class DecoderConfig:
    num_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    eps: float
    qk_norm: bool
    inv_freq: np.ndarray
    attention_scaling: float = 1.0


class DecoderOracle:
    """Weights of a Qwen3/Llama decoder stack as float64 arrays.

    ``weights`` maps the transformers state-dict names of the stack
    (``layers.{i}.self_attn.q_proj.weight`` …) to arrays.
    """

    def __init__(self, weights, cfg: DecoderConfig):
        self.w = {k: np.asarray(v, dtype=np.float64) for k, v in weights.items()}
        self.cfg = cfg
        self.scale = cfg.head_dim ** -0.5

    def _lin(self, x, name):
        y = x @ self.w[name + ".weight"].T
        b = self.w.get(name + ".bias")
        return y + b if b is not None else y

    def qkv(self, li, h, pos):
        """Projections + q/k norm + RoPE of layer ``li`` for ``h [..., T, D]``."""
        c = self.cfg
        p = f"layers.{li}."
        hn = rms_norm(h, self.w[p + "input_layernorm.weight"], c.eps)
        lead = hn.shape[:-1]
        q = self._lin(hn, p + "self_attn.q_proj").reshape(*lead, c.n_heads, c.head_dim)
        k = self._lin(hn, p + "self_attn.k_proj").reshape(*lead, c.n_kv_heads, c.head_dim)
        v = self._lin(hn, p + "self_attn.v_proj").reshape(*lead, c.n_kv_heads, c.head_dim)
        if c.qk_norm:
            q = rms_norm(q, self.w[p + "self_attn.q_norm.weight"], c.eps)
            k = rms_norm(k, self.w[p + "self_attn.k_norm.weight"], c.eps)
        q = rope(q, pos, c.inv_freq, c.attention_scaling)
        k = rope(k, pos, c.inv_freq, c.attention_scaling)
        return q, k, v

    def post_attention(self, li, h, o):
        p = f"layers.{li}."
        lead = o.shape[:-2]
        h = h + self._lin(o.reshape(*lead, -1), p + "self_attn.o_proj")
        hn = rms_norm(h, self.w[p + "post_attention_layernorm.weight"], self.cfg.eps)
        g = self._lin(hn, p + "mlp.gate_proj")
        u = self._lin(hn, p + "mlp.up_proj")
        return h + self._lin(silu(g) * u, p + "mlp.down_proj")


class DecodeSessionOracle:
    """Restates ``FlexDecodeSession`` (flex_decode.py:75-240) with per-row
    caches kept as growing arrays in logical slot order."""

    def __init__(self, decoder: DecoderOracle, batch_size: int):
        self.dec = decoder
        self.B = batch_size
        c = decoder.cfg
        self.lengths = np.zeros(batch_size, dtype=np.int64)
        self.k = [[np.zeros((0, c.n_kv_heads, c.head_dim)) for _ in range(batch_size)]
                  for _ in range(c.num_layers)]
        self.v = [[np.zeros((0, c.n_kv_heads, c.head_dim)) for _ in range(batch_size)]
                  for _ in range(c.num_layers)]

    def forward(self, embeds, lengths, output_hidden_states=False):
        x = np.asarray(embeds, dtype=np.float64)
        B, S, _ = x.shape
        if B != self.B:
            raise ValueError(f"Session was created for batch_size={self.B}, got {B}.")
        n = np.asarray(lengths, dtype=np.int64)
        q_pos, real = decode_positions(self.lengths, n, S)
        h = x
        hiddens = []
        for li in range(self.dec.cfg.num_layers):
            q, k, v = self.dec.qkv(li, h, q_pos)
            for b in range(B):
                cols = np.nonzero(real[b])[0]
                if cols.size:
                    # Real columns are contiguous and land at slots lengths[b]..
                    self.k[li][b] = np.concatenate([self.k[li][b], k[b, cols]], axis=0)
                    self.v[li][b] = np.concatenate([self.v[li][b], v[b, cols]], axis=0)
            o = cached_decode_attention(q, self.k[li], self.v[li], q_pos, self.dec.scale)
            h = self.dec.post_attention(li, h, o)
            hiddens.append(h)
        self.lengths = self.lengths + n
        if output_hidden_states:
            return h, tuple(hiddens)
        return h


def packed_forward(decoder: DecoderOracle, embeds, sequence_ids, output_hidden_states=False):
    """Restates ``flex_packed_forward`` (flex_train.py:51-157) for
    ``embeds [L, D]``; the final norm is the identity, as in mouse-core's
    backbones (qwen3.py:111, llama.py ``norm = nn.Identity()``)."""
    h = np.asarray(embeds, dtype=np.float64)
    pos = position_ids(sequence_ids)
    hiddens = []
    for li in range(decoder.cfg.num_layers):
        q, k, v = decoder.qkv(li, h, pos)
        o, _ = packed_attention_fwd(q, k, v, sequence_ids, decoder.scale)
        h = decoder.post_attention(li, h, o)
        hiddens.append(h)
    if output_hidden_states:
        return h, tuple(hiddens)
    return h


def config_from_hf(hf_config, inv_freq, attention_scaling=1.0):
    """Build a ``DecoderConfig`` from a transformers config object."""
    qk_norm = "qwen3" in str(getattr(hf_config, "model_type", "")).lower()
    hd = getattr(hf_config, "head_dim", None) or hf_config.hidden_size // hf_config.num_attention_heads
    return DecoderConfig(
        num_layers=int(hf_config.num_hidden_layers),
        n_heads=int(hf_config.num_attention_heads),
        n_kv_heads=int(hf_config.num_key_value_heads),
        head_dim=int(hd),
        eps=float(hf_config.rms_norm_eps),
        qk_norm=qk_norm,
        inv_freq=np.asarray(inv_freq, dtype=np.float64),
        attention_scaling=float(attention_scaling),
    )


class GrowRebuildOracle:
    """Restates the caller loop that drives the grow-then-rebuild policy:
    ``_act_from_contexts`` in ``run_eval`` (examples/02_train_offline.ipynb,
    cell 11) over ``DecodeSessionOracle``, with the policy functions of
    ``oracle.policy`` (kv_policy.py:14-72).

    Batch mode (``per_row=False``) is the reference's loop: when
    ``cache_needs_rebuild`` (or a forced rebuild) fires, the session is dropped
    and a new one prefills ``history[b, rebuild_starts[b]:ends[b]]`` for every
    row (models/base.py:932-934 makes the new session); otherwise each row
    appends ``history[b, cached_ends[b]:ends[b]]``. Per-row mode runs that same
    loop independently for every row (a batch of one env each).

    ``step`` returns ``(out [B, S, D], fed [B])`` laid out like the session's
    left-padded output: row ``b``'s ``fed[b]`` new tokens in its last columns.
    """

    def __init__(self, decoder: DecoderOracle, batch_size: int, table, max_cache: int, start_cache=None,
                 per_row: bool = False):
        from oracle.policy import resolve_cache_bounds

        self.dec = decoder
        self.B = batch_size
        self.table = np.asarray(table, dtype=np.float64)
        self.max_cache, self.start_cache = resolve_cache_bounds(max_cache, start_cache)
        self.per_row = per_row
        if per_row:
            self.rows = [GrowRebuildOracle(decoder, 1, table, max_cache, start_cache) for _ in range(batch_size)]
        self.session = None
        self.cached_starts = np.zeros(batch_size, dtype=np.int64)
        self.cached_ends = np.zeros(batch_size, dtype=np.int64)

    def step(self, history, ends, context_start=0, rebuild=False):
        from oracle.policy import cache_needs_rebuild, rebuild_starts

        hist = np.asarray(history)
        ends = np.asarray(ends, dtype=np.int64)
        ctx = np.broadcast_to(np.asarray(context_start, dtype=np.int64), ends.shape)
        if self.per_row:
            forced = np.zeros(self.B, dtype=bool)
            if rebuild is True:
                forced[:] = True
            elif rebuild is not False and rebuild is not None:
                r = np.asarray(rebuild)
                if r.dtype == bool:
                    forced |= r
                else:
                    forced[r] = True
            parts = [row.step(hist[b:b + 1], ends[b:b + 1], ctx[b:b + 1], bool(forced[b]))
                     for b, row in enumerate(self.rows)]
            fed = np.array([int(p[1][0]) for p in parts], dtype=np.int64)
            S = max(int(fed.max()), 1)
            out = np.zeros((self.B, S, self.table.shape[1]))
            for b, (o, n) in enumerate(parts):
                if n[0]:
                    out[b, S - n[0]:] = o[0, o.shape[1] - n[0]:]
            return out, fed
        need = (rebuild is True or (rebuild is not False and rebuild is not None and np.asarray(rebuild).any())
                or cache_needs_rebuild(has_cache=self.session is not None, cached_starts=self.cached_starts,
                                       cached_ends=self.cached_ends, ends=ends, context_start=ctx,
                                       max_cache=self.max_cache, batch_complete=True))
        if need:
            starts = rebuild_starts(ends=ends, context_start=ctx, start_cache=self.start_cache,
                                    max_cache=self.max_cache)
            self.session = DecodeSessionOracle(self.dec, self.B)
            self.cached_starts = starts
        else:
            starts = self.cached_ends
        fed = ends - starts
        S = max(int(fed.max()), 1)
        emb = np.zeros((self.B, S, self.table.shape[1]))
        for b in range(self.B):
            n = int(fed[b])
            if n:
                emb[b, S - n:] = self.table[hist[b, starts[b]:ends[b]]]
        out = self.session.forward(emb, fed)
        self.cached_ends = ends.copy()
        return out, fed
