"""K11 token embedding against the reference's NumericEmbedder outputs and
the oracle: one pinned upload of the TokenBatch, one kernel over the stream.

Table rows are copied exactly; Fourier features are computed in fp32 and
rounded once (the fp32 path matches the reference to 1e-5, the bf16 path the
float64 oracle to one bf16 rounding of the output)."""

from __future__ import annotations

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import encoder as oenc
from tests.golden_io import load

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from mouse_core_b200 import build

    build.build()
    return torch.device("cuda")


class _Fourier(torch.nn.Module):
    def __init__(self, rec):
        super().__init__()
        for name in ("freqs", "phases", "output_scale"):
            self.register_buffer(name, torch.from_numpy(np.asarray(rec[f"w:fourier.{name}"])))


class _Embedder(torch.nn.Module):
    """The layout of the reference's NumericEmbedder, loaded from the fixture."""

    def __init__(self, rec):
        super().__init__()
        self.hidden_dim = int(rec["hidden_dim"])
        self._meta = [SimpleNamespace(type_id=int(t), kind=str(k)) for t, k in zip(rec["meta_type_id"], rec["meta_kind"])]
        self._tables = torch.nn.ModuleDict()
        for m in self._meta:
            if m.kind != "fourier":
                w = torch.from_numpy(rec[f"w:_tables.{m.type_id}.weight"])
                self._tables[str(m.type_id)] = torch.nn.Embedding.from_pretrained(w, freeze=False)
        self.fourier = _Fourier(rec)


def _batch(rec, ci):
    names = ("token_types", "token_ids", "scalars", "sequence_ids", "step_ids", "prediction_indices")
    tb = SimpleNamespace(**{n: rec[f"c{ci}_{n}"] for n in names})
    tb.B = int(rec[f"c{ci}_B"])
    tb.col_values = {"sequence_id": rec[f"c{ci}_sequence_id"]}
    return tb


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_fused_embedding_matches_reference(dtype):
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200.encoder import fused_forward

    rec = load("embedding.npz")
    emb = _Embedder(rec).to(device=dev, dtype=dtype)
    tables = {m.type_id: rec[f"w:_tables.{m.type_id}.weight"] for m in emb._meta if m.kind != "fourier"}
    if dtype == torch.bfloat16:
        tables = {t: torch.from_numpy(w).bfloat16().float().numpy() for t, w in tables.items()}
    fourier = [m.type_id for m in emb._meta if m.kind == "fourier"]
    # The Fourier banks are the module's buffers as they are (a bf16 module
    # holds bf16-rounded frequencies, as the reference's bf16 path does).
    fb = {n: np.asarray(rec[f"w:fourier.{n}"], dtype=np.float64) for n in ("freqs", "phases", "output_scale")}
    if dtype == torch.bfloat16:
        fb = {n: torch.from_numpy(np.asarray(v, dtype=np.float32)).bfloat16().double().numpy() for n, v in fb.items()}
    for ci in range(2):
        tb = _batch(rec, ci)
        embeds, col, pred = fused_forward(emb, tb)
        got = embeds.float().cpu().numpy()
        assert embeds.dtype == dtype and embeds.shape == rec[f"c{ci}_embeds"].shape
        assert torch.equal(pred.cpu(), torch.from_numpy(rec[f"c{ci}_pred"]))
        assert torch.equal(col["sequence_id"].cpu(), torch.from_numpy(rec[f"c{ci}_sequence_id"]))
        ref = oenc.embed_tokens(tb.token_types, tb.token_ids, tb.scalars, tables, fourier, fb["freqs"],
                                fb["phases"], float(fb["output_scale"]), emb.hidden_dim)
        is_table = np.isin(tb.token_types, list(tables))
        assert np.array_equal(got[is_table], ref[is_table])  # table rows are copied bit for bit
        if dtype == torch.float32:
            assert np.abs(got - rec[f"c{ci}_embeds"]).max() < 1e-5
        else:
            assert np.abs(got - ref).max() <= 2.0 ** -8 * max(1.0, np.abs(ref).max())
    assert _lib.device_status() == 0


def test_fused_embedding_flags_an_id_outside_its_table():
    """An id past its table leaves that token zero and reports status 7 (the
    reference's masked gather would index out of range)."""
    dev = _dev()
    from mouse_core_b200 import _lib
    from mouse_core_b200.encoder import fused_forward

    rec = load("embedding.npz")
    emb = _Embedder(rec).to(dev)
    tb = _batch(rec, 0)
    tb.token_ids = tb.token_ids.copy()
    bad = int(np.flatnonzero(tb.token_types == 0)[0])  # an obs token (vocab 16)
    tb.token_ids[bad] = 16
    _lib.device_status()
    embeds, _, _ = fused_forward(emb, tb)
    assert _lib.device_status() == 7
    assert float(embeds[bad].abs().max()) == 0.0
