"""Float64 restatements of the two attention kernels on the hot path.

Test infrastructure (see ``oracle/__init__.py``).

* ``cached_decode_attention`` restates the FlexAttention call of
  ``FlexDecodeSession.forward`` (backbone/flex_decode.py:226-229) with its
  mask ``kv_idx <= q_pos[b, q]`` (flex_decode.py:129-134) over a per-row
  cache in logical slot order.
* ``packed_attention_fwd`` / ``packed_attention_bwd`` restate the packed
  training attention (backbone/flex_train.py:98-102,147 on CUDA; the dense
  SDPA mask of models/base.py:1204-1223 on CPU): ``kv <= q`` and
  ``sequence_ids[q] == sequence_ids[kv]``, GQA with ``q_head // group``.
  The backward is the analytic gradient of softmax attention.
"""

from __future__ import annotations

import numpy as np


def cached_decode_attention(q, k_rows, v_rows, q_pos, scale):
    """Attention of left-padded queries against per-row caches.

    Args:
        q: ``[B, S, Hq, hd]`` queries (post-RoPE).
        k_rows, v_rows: length-``B`` lists of ``[n_b, Hkv, hd]`` arrays: row
            ``b``'s cache in logical slot order (slot ``i`` = token ``i``).
        q_pos: ``[B, S]`` int, each query attends slots ``0..q_pos``.
            Slots at or beyond ``n_b`` read as zero, as the reference's
            zero-initialised cache does (flex_decode.py:109-113).
        scale: softmax scale (``head_dim ** -0.5``).

    Returns ``[B, S, Hq, hd]`` float64.
    """
    q = np.asarray(q, dtype=np.float64)
    B, S, Hq, hd = q.shape
    out = np.zeros((B, S, Hq, hd), dtype=np.float64)
    for b in range(B):
        kb = np.asarray(k_rows[b], dtype=np.float64)
        vb = np.asarray(v_rows[b], dtype=np.float64)
        Hkv = kb.shape[1] if kb.ndim == 3 else 1
        if kb.ndim != 3:
            kb = kb.reshape(0, Hkv, hd)
            vb = vb.reshape(0, Hkv, hd)
        group = Hq // max(Hkv, 1)
        for s in range(S):
            n_keys = int(q_pos[b, s]) + 1
            keys = np.zeros((n_keys, kb.shape[1], hd))
            vals = np.zeros((n_keys, kb.shape[1], hd))
            m = min(n_keys, kb.shape[0])
            keys[:m] = kb[:m]
            vals[:m] = vb[:m]
            for h in range(Hq):
                kh = h // group
                sc = keys[:, kh, :] @ q[b, s, h] * scale
                sc -= sc.max()
                p = np.exp(sc)
                p /= p.sum()
                out[b, s, h] = p @ vals[:, kh, :]
    return out


def _segments(sequence_ids):
    seq = np.asarray(sequence_ids).reshape(-1)
    for sid in np.unique(seq):
        yield np.nonzero(seq == sid)[0]


def packed_attention_fwd(q, k, v, sequence_ids, scale):
    """Segment-causal GQA attention over one packed stream.

    Args:
        q ``[L, Hq, hd]``, k/v ``[L, Hkv, hd]``, sequence_ids ``[L]``.

    Returns ``(out [L, Hq, hd], lse [Hq, L])`` in float64, ``lse`` the natural
    log of the softmax denominator of the scaled scores.
    """
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    L, Hq, hd = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    out = np.zeros_like(q)
    lse = np.zeros((Hq, L))
    for idx in _segments(sequence_ids):
        n = idx.shape[0]
        causal = np.tril(np.ones((n, n), dtype=bool))
        for h in range(Hq):
            kh = h // group
            s = (q[idx, h] @ k[idx, kh].T) * scale
            s = np.where(causal, s, -np.inf)
            mx = s.max(axis=1, keepdims=True)
            p = np.exp(s - mx)
            den = p.sum(axis=1, keepdims=True)
            out[idx, h] = (p / den) @ v[idx, kh]
            lse[h, idx] = (mx + np.log(den))[:, 0]
    return out, lse


def packed_attention_bwd(q, k, v, sequence_ids, scale, dout):
    """Gradients ``(dq, dk, dv)`` of ``packed_attention_fwd`` w.r.t. q, k, v
    for upstream gradient ``dout [L, Hq, hd]`` (float64). ``dk``/``dv`` sum
    the contributions of the ``group`` query heads sharing a KV head."""
    q = np.asarray(q, dtype=np.float64)
    k = np.asarray(k, dtype=np.float64)
    v = np.asarray(v, dtype=np.float64)
    do = np.asarray(dout, dtype=np.float64)
    L, Hq, hd = q.shape
    Hkv = k.shape[1]
    group = Hq // Hkv
    dq = np.zeros_like(q)
    dk = np.zeros_like(k)
    dv = np.zeros_like(v)
    for idx in _segments(sequence_ids):
        n = idx.shape[0]
        causal = np.tril(np.ones((n, n), dtype=bool))
        for h in range(Hq):
            kh = h // group
            s = (q[idx, h] @ k[idx, kh].T) * scale
            s = np.where(causal, s, -np.inf)
            p = np.exp(s - s.max(axis=1, keepdims=True))
            p /= p.sum(axis=1, keepdims=True)
            o = p @ v[idx, kh]
            dov = do[idx, h]
            dv[idx, kh] += p.T @ dov
            dp = dov @ v[idx, kh].T
            delta = (dov * o).sum(axis=1, keepdims=True)
            ds = p * (dp - delta)
            dq[idx, h] += (ds @ k[idx, kh]) * scale
            dk[idx, kh] += (ds.T @ q[idx, h]) * scale
    return dq, dk, dv
