"""Float64 restatement of the token embedding on the hot path's input side.

Test infrastructure (see ``oracle/__init__.py``).

``embed_tokens`` restates ``NumericEmbedder.forward``
(src/mouse_core/models/embedding/embedding.py:293-326): the output starts at
zero; every token whose type has an embedding table (discrete, learnable and
image modalities) takes row ``token_ids[t]`` of that table; every token of a
Fourier modality (rff / continuous) takes the static Fourier features of
``StaticFourierFeatures.forward`` (models/embedding/encoding.py:67-86):
``output_scale * cos(x * freqs[bank] + phases[bank])`` with ``bank =
token_ids[t]``.
"""

from __future__ import annotations

import numpy as np


def embed_tokens(token_types, token_ids, scalars, tables, fourier_types, freqs, phases, output_scale, hidden_dim):
    """``tables`` maps a type id to its ``[vocab, D]`` rows; ``fourier_types``
    lists the Fourier type ids. Returns ``[L, D]`` float64."""
    types = np.asarray(token_types, dtype=np.int64)
    ids = np.asarray(token_ids, dtype=np.int64)
    x = np.asarray(scalars, dtype=np.float64)
    out = np.zeros((types.shape[0], hidden_dim))
    for tid, table in tables.items():
        mask = types == int(tid)
        out[mask] = np.asarray(table, dtype=np.float64)[ids[mask]]
    w = np.asarray(freqs, dtype=np.float64)
    b = np.asarray(phases, dtype=np.float64)
    for tid in fourier_types:
        mask = types == int(tid)
        out[mask] = float(output_scale) * np.cos(x[mask, None] * w[ids[mask]] + b[ids[mask]])
    return out
