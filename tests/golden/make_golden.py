"""Generate the golden fixtures in this folder by running the reference itself.

Run in a container where the reference source tree is available::

    python tests/golden/make_golden.py --reference <reference checkout>/src [--only grow_rebuild ...]

It imports micahr234/mouse-core v0.4.0 from that tree (with a stand-in
``tensordict`` module and package metadata written to a temp dir, because the
reference imports ``tensordict`` and reads its own dist-info at import time)
and records, for seeded inputs, what the reference's own hot-path functions
return:

* ``index_maps.npz``   ``_flat_sequence_position_ids`` (models/base.py:1226),
                       ``_flat_sequence_causal_mask`` (base.py:1204),
                       ``left_align_content`` (embedding/packing.py:8),
                       ``_flat_to_batched_left_pad`` (base.py:1163).
* ``kv_policy.json``   ``resolve_cache_bounds`` / ``rebuild_starts`` /
                       ``cache_needs_rebuild`` (models/kv_policy.py:14-72).
* ``packed_attn_small.npz``  reference CPU training attention (SDPA with the
                       dense segment mask, base.py:962-969) fwd + bwd, fp32.
* ``packed_attn_cfg1.npz``   the same at the 2048-token, 4/2-head, hd-64
                       shape; inputs are regenerated from the stored seeds,
                       outputs stored as sums and a seeded sample of entries.
* ``decode_<arch>.npz``  ``FlexDecodeSession`` (backbone/flex_decode.py) run
                       on CPU fp32 over a ragged call schedule, for a tiny
                       Qwen3 and a tiny Llama backbone (weights stored,
                       fp16-representable so they store exactly).
* ``packed_fwd_qwen3.npz`` ``flex_packed_forward``'s CPU twin (the HF stack
                       with the dense mask + per-run position ids).
* ``grow_rebuild_qwen3.npz`` the caller loop that drives the grow-then-rebuild
                       policy (kv_policy.py + ``FlexDecodeSession``) over a
                       40-call ragged schedule with task ends and a small
                       ``max_cache``: whole-batch rebuilds, and each env
                       run alone (the per-row semantics).
* ``embedding.npz``    ``NumericEmbedder`` (models/embedding/embedding.py):
                       ``prepare`` and ``forward`` on ragged transition rows
                       with discrete, rff, continuous (optional) and learnable
                       modalities.

The fixtures are small; nothing at test time reads the reference.
"""

from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from tests.golden_io import grow_rebuild_schedule  # noqa: E402  (the schedule the GPU tests replay)


def _install_shims(tmp: Path) -> None:
    td = tmp / "tensordict"
    td.mkdir(parents=True, exist_ok=True)
    (td / "__init__.py").write_text(
        "import torch\n"
        "class TensorDict(dict):\n"
        "    def __init__(self, source=None, batch_size=None, device=None, **kw):\n"
        "        super().__init__(source or {})\n"
        "        self.batch_size = torch.Size(batch_size if batch_size is not None else [])\n"
        "        self.device = device\n"
    )
    meta = tmp / "mouse_core-0.4.0.dist-info"
    meta.mkdir(parents=True, exist_ok=True)
    (meta / "METADATA").write_text("Metadata-Version: 2.1\nName: mouse-core\nVersion: 0.4.0\n")
    sys.path.insert(0, str(tmp))


def cfg1_segments(seed: int = 0, L: int = 2048, lo: int = 16, hi: int = 512):
    """Segment lengths of the 2048-token packed-attention workload:
    ``rng.integers(lo, hi + 1)`` until the sum reaches ``L``, last truncated."""
    rng = np.random.default_rng(seed)
    segs = []
    total = 0
    while total < L:
        s = int(rng.integers(lo, hi + 1))
        s = min(s, L - total)
        segs.append(s)
        total += s
    return segs


def cfg1_inputs(seed: int, L: int, Hq: int, Hkv: int, hd: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    q = torch.randn(L, Hq, hd, generator=g)
    k = torch.randn(L, Hkv, hd, generator=g)
    v = torch.randn(L, Hkv, hd, generator=g)
    do = torch.randn(L, Hq, hd, generator=g)
    return q, k, v, do


def _sdpa_packed(q, k, v, seq, do):
    """Reference CPU path: SDPA with the reference's dense additive mask."""
    import torch
    import torch.nn.functional as F
    from mouse_core.models.base import _flat_sequence_causal_mask

    q = q.clone().requires_grad_(True)
    k = k.clone().requires_grad_(True)
    v = v.clone().requires_grad_(True)
    mask = _flat_sequence_causal_mask(dtype=torch.float32, sequence_ids=seq)
    o = F.scaled_dot_product_attention(
        q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
        attn_mask=mask, enable_gqa=True,
    )[0].transpose(0, 1)
    o.backward(do)
    return o.detach(), q.grad, k.grad, v.grad


def make_index_maps(out: dict) -> None:
    import torch
    from mouse_core.models.base import (
        _flat_sequence_causal_mask, _flat_sequence_position_ids, _flat_to_batched_left_pad,
    )
    from mouse_core.models.embedding.packing import left_align_content

    rng = np.random.default_rng(0)
    cases = {"known": np.array([0, 0, 0, 1, 1, 2]), "noncontig": np.array([0, 0, 1, 1, 0, 0, 2, 1])}
    for L in (0, 1, 7, 128, 257, 1000):
        seq = np.zeros(L, dtype=np.int64)
        sid = 0
        for i in range(L):
            if i > 0 and rng.random() < 0.15:
                sid += 1
            seq[i] = sid
        cases[f"rand{L}"] = seq
    for name, seq in cases.items():
        t = torch.tensor(seq, dtype=torch.long)
        out[f"pos_{name}_in"] = seq
        out[f"pos_{name}_out"] = _flat_sequence_position_ids(sequence_ids=t).numpy()
        if seq.shape[0] <= 128:
            m = _flat_sequence_causal_mask(dtype=torch.float32, sequence_ids=t)
            out[f"mask_{name}_allow"] = (m[0, 0] == 0).numpy()

    # left_align_content over random right-padded rows.
    for c in range(4):
        B, L, D = 3 + c, 6 + c, 2
        emb = rng.standard_normal((B, L, D)).astype(np.float32)
        S = 3
        idx = np.zeros((B, S), dtype=np.int64)
        for b in range(B):
            n = int(rng.integers(0, S + 1))
            rl = int(rng.integers(n, L + 1)) if n else 0
            if n:
                cols = np.sort(rng.choice(np.arange(rl), size=n, replace=False))
                cols[-1] = rl - 1
                idx[b, S - n:] = cols
        a, ai = left_align_content(torch.tensor(emb), torch.tensor(idx))
        out[f"la{c}_emb"], out[f"la{c}_idx"] = emb, idx
        out[f"la{c}_out"], out[f"la{c}_outidx"] = a.numpy(), ai.numpy()

    # _flat_to_batched_left_pad over random ragged flat batches.
    for c in range(4):
        B = 2 + c
        steps = rng.integers(0, 4, size=B)
        steps[0] = max(1, steps[0])
        tps = 1 + (c % 3)  # tokens per step
        seq, pidx = [], []
        for b in range(B):
            for s in range(int(steps[b])):
                for t in range(tps):
                    seq.append(b)
                pidx.append(len(seq) - 1)
        seq = np.array(seq, dtype=np.int64)
        pidx = np.array(pidx, dtype=np.int64)
        D = 3
        emb = rng.standard_normal((seq.shape[0], D)).astype(np.float32)
        S = int(steps.max())
        o, tl, li = _flat_to_batched_left_pad(
            torch.tensor(emb), torch.tensor(seq), torch.tensor(pidx), B, S, steps.tolist())
        out[f"fb{c}_emb"], out[f"fb{c}_seq"], out[f"fb{c}_pidx"] = emb, seq, pidx
        out[f"fb{c}_steps"] = steps.astype(np.int64)
        out[f"fb{c}_out"], out[f"fb{c}_tl"], out[f"fb{c}_local"] = o.numpy(), np.array(tl), li.numpy()


def make_kv_policy() -> dict:
    from mouse_core.models.kv_policy import cache_needs_rebuild, rebuild_starts, resolve_cache_bounds

    rng = np.random.default_rng(1)
    res = {"bounds": [], "starts": [], "rebuild": []}
    for mx, st in [(512, None), (512, 512), (1, None), (1, 5), (2, None), (8192, 1024),
                   (16384, None), (0, None), (7, 100), (100, 0)]:
        res["bounds"].append([mx, st, list(resolve_cache_bounds(mx, st))])
    for _ in range(40):
        B = int(rng.integers(1, 6))
        ends = rng.integers(0, 3000, size=B)
        ctx = rng.integers(0, 1500, size=B) if rng.random() < 0.5 else int(rng.integers(0, 100))
        st = int(rng.integers(1, 1200))
        mx = int(rng.integers(1, 2000))
        got = rebuild_starts(ends=ends, context_start=ctx, start_cache=st, max_cache=mx)
        res["starts"].append([ends.tolist(), ctx if isinstance(ctx, int) else ctx.tolist(), st, mx, got.tolist()])
    for _ in range(80):
        B = int(rng.integers(1, 5))
        cs = rng.integers(0, 500, size=B)
        ce = cs + rng.integers(0, 600, size=B)
        ends = ce + rng.integers(-2, 30, size=B)
        ctx = np.where(rng.random(B) < 0.1, cs + 1, np.minimum(cs, rng.integers(0, 500, size=B)))
        mx = int(rng.integers(100, 700))
        has = bool(rng.random() < 0.9)
        comp = bool(rng.random() < 0.9)
        if rng.random() < 0.05:
            ends = np.concatenate([ends, [5]])
        got = cache_needs_rebuild(has_cache=has, cached_starts=cs, cached_ends=ce, ends=ends,
                                  context_start=ctx, max_cache=mx, batch_complete=comp)
        res["rebuild"].append([has, cs.tolist(), ce.tolist(), ends.tolist(), ctx.tolist(), mx, comp, bool(got)])
    return res


def make_packed_attention() -> None:
    import torch

    # Small case: full tensors, with a non-contiguous repeated id.
    torch.manual_seed(0)
    segs = [37, 5, 64, 1, 50, 35]
    seq = np.concatenate([np.full(s, i) for i, s in enumerate(segs)]).astype(np.int64)
    seq[-20:] = 1  # a second run of id 1: attends back to the first run
    L, Hq, Hkv, hd = seq.shape[0], 4, 2, 64
    q, k, v, do = cfg1_inputs(7, L, Hq, Hkv, hd)
    o, dq, dk, dv = _sdpa_packed(q, k, v, torch.tensor(seq), do)
    np.savez_compressed(HERE / "packed_attn_small.npz", seq=seq, q=q.numpy(), k=k.numpy(),
                        v=v.numpy(), do=do.numpy(), out=o.numpy(), dq=dq.numpy(),
                        dk=dk.numpy(), dv=dv.numpy())

    # cfg1: 2048 tokens, seed 0 segments, 4/2 heads, hd 64.
    segs = cfg1_segments(0)
    seq = np.concatenate([np.full(s, i) for i, s in enumerate(segs)]).astype(np.int64)
    L = seq.shape[0]
    q, k, v, do = cfg1_inputs(0, L, 4, 2, 64)
    o, dq, dk, dv = _sdpa_packed(q, k, v, torch.tensor(seq), do)
    rng = np.random.default_rng(123)
    rec = {"segs": np.array(segs), "seed": np.array(0)}
    for name, t in (("out", o), ("dq", dq), ("dk", dk), ("dv", dv)):
        a = t.numpy().astype(np.float64)
        flat = a.reshape(-1)
        idx = rng.choice(flat.shape[0], size=4096, replace=False)
        rec[f"{name}_sum"] = np.array(flat.sum())
        rec[f"{name}_abssum"] = np.array(np.abs(flat).sum())
        rec[f"{name}_idx"] = idx
        rec[f"{name}_val"] = flat[idx].astype(np.float32)
    np.savez_compressed(HERE / "packed_attn_cfg1.npz", **rec)


def _round_fp16_(module) -> None:
    import torch

    with torch.no_grad():
        for p in module.parameters():
            p.copy_(p.half().float())


def _weights(model) -> dict:
    return {k: v.detach().numpy().astype(np.float16) for k, v in model.state_dict().items()
            if "rotary_emb" not in k}


def make_decode(arch: str) -> None:
    import torch
    from mouse_core.models.backbone import LlamaBackbone, Qwen3Backbone
    from mouse_core.models.backbone.flex_decode import FlexDecodeSession

    torch.manual_seed(11 if arch == "qwen3" else 12)
    if arch == "qwen3":
        bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    else:
        bb = LlamaBackbone(hidden_dim=128, num_layers=2, num_heads=2, num_key_value_heads=1)
    model = bb.model.eval()
    _round_fp16_(model)
    # Random (non-unit) norm weights so the q/k norm and layer norms are exercised.
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_((1.0 + 0.25 * torch.randn_like(p)).half().float())
    D = model.config.hidden_size
    B = 3
    schedule = [[3, 0, 2], [1, 2, 0], [2, 3, 1], [0, 1, 4], [1, 1, 1], [5, 0, 2]]
    sess = FlexDecodeSession(model, batch_size=B, capacity=4)  # small capacity: forces _grow
    rec = {"schedule": np.array(schedule), "inv_freq": model.rotary_emb.inv_freq.numpy(),
           "attention_scaling": np.array(float(model.rotary_emb.attention_scaling)),
           "eps": np.array(float(model.config.rms_norm_eps)),
           "n_heads": np.array(model.config.num_attention_heads),
           "n_kv_heads": np.array(model.config.num_key_value_heads),
           "head_dim": np.array(int(getattr(model.config, "head_dim", D // model.config.num_attention_heads))),
           "num_layers": np.array(model.config.num_hidden_layers),
           "qk_norm": np.array(arch == "qwen3")}
    for key, val in _weights(model).items():
        rec["w:" + key] = val
    g = torch.Generator().manual_seed(5)
    for ci, lens in enumerate(schedule):
        S = max(max(lens), 1)
        emb = torch.randn(B, S, D, generator=g)
        emb = emb.half().float()
        with torch.no_grad():
            h, layers = sess.forward(embeds=emb, lengths=list(lens), output_hidden_states=True)
        rec[f"c{ci}_emb"] = emb.numpy()
        rec[f"c{ci}_out"] = h.numpy()
        rec[f"c{ci}_layer0"] = layers[0].numpy()
    rec["final_lengths"] = sess.lengths.numpy()
    np.savez_compressed(HERE / f"decode_{arch}.npz", **rec)


class _RefGrowRebuildLoop:
    """The reference's caller loop (``_act_from_contexts`` in ``run_eval``,
    examples/02_train_offline.ipynb cell 11) with its own kv_policy functions
    and ``FlexDecodeSession``; the session is dropped and re-made on every
    rebuild, as ``Model.forward`` does with ``cache=None`` (base.py:932-934)."""

    def __init__(self, model, B, table, max_cache, start_cache):
        from mouse_core.models.kv_policy import resolve_cache_bounds

        self.model, self.B, self.table = model, B, table
        self.max_cache, self.start_cache = resolve_cache_bounds(max_cache, start_cache)
        self.session = None
        self.cached_starts = np.zeros(B, dtype=np.int64)
        self.cached_ends = np.zeros(B, dtype=np.int64)

    def step(self, hist, ends, ctx, rebuild):
        import torch
        from mouse_core.models.backbone.flex_decode import FlexDecodeSession
        from mouse_core.models.kv_policy import cache_needs_rebuild, rebuild_starts

        need = rebuild or cache_needs_rebuild(
            has_cache=self.session is not None, cached_starts=self.cached_starts, cached_ends=self.cached_ends,
            ends=ends, context_start=ctx, max_cache=self.max_cache, batch_complete=True)
        if need:
            starts = rebuild_starts(ends=ends, context_start=ctx, start_cache=self.start_cache,
                                    max_cache=self.max_cache)
            self.cached_starts = starts
        else:
            starts = self.cached_ends
        fed = ends - starts
        S = max(int(fed.max()), 1)
        emb = torch.zeros(self.B, S, self.table.shape[1])
        for b in range(self.B):
            n = int(fed[b])
            if n:
                emb[b, S - n:] = self.table[torch.from_numpy(hist[b, starts[b]:ends[b]])]
        if need:
            self.session = FlexDecodeSession(self.model, batch_size=self.B, capacity=S)
        with torch.no_grad():
            out = self.session.forward(embeds=emb, lengths=fed.tolist())
        self.cached_ends = ends.copy()
        return out.numpy(), fed


def make_grow_rebuild() -> None:
    """The reference's caller loop over a 40-call schedule with a tiny
    ``max_cache`` so rebuilds are frequent: batch mode (every rebuild
    re-windows the whole batch) and, for the per-row semantics, the same loop
    run on each env alone (a batch of one)."""
    import torch
    from mouse_core.models.backbone import Qwen3Backbone

    torch.manual_seed(31)
    bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    model = bb.model.eval()
    _round_fp16_(model)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if "norm" in name:
                p.copy_((1.0 + 0.25 * torch.randn_like(p)).half().float())
    B, calls, vocab, max_cache, start_cache = 4, 40, 48, 24, 10
    g = torch.Generator().manual_seed(9)
    table = torch.randn(vocab, 64, generator=g).half().float()
    rec = {"inv_freq": model.rotary_emb.inv_freq.numpy(), "eps": np.array(float(model.config.rms_norm_eps)),
           "n_heads": np.array(2), "n_kv_heads": np.array(1), "head_dim": np.array(64), "num_layers": np.array(2),
           "qk_norm": np.array(True), "table": table.numpy(), "max_cache": np.array(max_cache),
           "start_cache": np.array(start_cache), "calls": np.array(calls), "B": np.array(B)}
    for key, val in _weights(model).items():
        rec["w:" + key] = val
    batch = _RefGrowRebuildLoop(model, B, table, max_cache, start_cache)
    alone = [_RefGrowRebuildLoop(model, 1, table, max_cache, start_cache) for _ in range(B)]
    for ci, (hist, ends, ctx, ended) in enumerate(grow_rebuild_schedule(4, B, calls, vocab)):
        out, fed = batch.step(hist, ends, ctx, bool(ended.any()))
        rec[f"c{ci}_hist"], rec[f"c{ci}_ends"], rec[f"c{ci}_ctx"], rec[f"c{ci}_ended"] = hist, ends, ctx, ended
        rec[f"c{ci}_out"], rec[f"c{ci}_fed"] = out, fed
        for b in range(B):
            o, f = alone[b].step(hist[b:b + 1], ends[b:b + 1], ctx[b:b + 1], bool(ended[b]))
            rec[f"c{ci}_row{b}_out"], rec[f"c{ci}_row{b}_fed"] = o, f
    np.savez_compressed(HERE / "grow_rebuild_qwen3.npz", **rec)


EMBED_MODALITIES = [
    {"type": "discrete", "field": "obs", "vocab_size": 16},
    {"type": "discrete", "field": "action", "vocab_size": 4},
    {"type": "rff", "field": "reward"},
    {"type": "continuous", "field": "pos", "dim": 3, "required": False},
    {"type": "learnable", "tokens": 2},
]


def make_embedding() -> None:
    """The reference's NumericEmbedder (prepare + forward, fp32) on ragged
    batches of transition rows, one of them with an optional field missing."""
    import torch
    from mouse_core.models.embedding.embedding import NumericEmbedder

    torch.manual_seed(41)
    emb = NumericEmbedder(hidden_dim=64, modalities=EMBED_MODALITIES, fourier_min=0.01, fourier_max=10.0)
    rng = np.random.default_rng(42)
    rec = {"hidden_dim": np.array(64)}
    for key, val in emb.state_dict().items():
        rec["w:" + key] = val.numpy()
    rec["meta_type_id"] = np.array([m.type_id for m in emb._meta])
    rec["meta_kind"] = np.array([m.kind for m in emb._meta])
    for ci, steps in enumerate([[4, 0, 2], [1, 3, 5, 2]]):
        batch = []
        for n in steps:
            rows = []
            for _ in range(n):
                row = {"obs": int(rng.integers(0, 16)), "action": int(rng.integers(0, 4)),
                       "reward": float(rng.normal())}
                if rng.random() < 0.7:
                    row["pos"] = rng.normal(size=3).astype(np.float32) * 3.0
                rows.append(row)
            batch.append(rows)
        tb = emb.prepare(batch)
        with torch.no_grad():
            embeds, _, pred = emb(tb)
        for name in ("token_types", "token_ids", "scalars", "sequence_ids", "step_ids", "prediction_indices"):
            rec[f"c{ci}_{name}"] = np.asarray(getattr(tb, name))
        rec[f"c{ci}_B"] = np.array(tb.B)
        rec[f"c{ci}_sequence_id"] = np.asarray(tb.col_values["sequence_id"])
        rec[f"c{ci}_embeds"] = embeds.numpy()
        rec[f"c{ci}_pred"] = pred.numpy()
    np.savez_compressed(HERE / "embedding.npz", **rec)


def make_packed_forward() -> None:
    import torch
    from mouse_core.models.backbone import Qwen3Backbone
    from mouse_core.models.base import _flat_sequence_causal_mask, _flat_sequence_position_ids

    torch.manual_seed(21)
    bb = Qwen3Backbone(hidden_dim=64, num_layers=2, num_heads=2, num_key_value_heads=1, head_dim=64)
    model = bb.model.eval()
    _round_fp16_(model)
    seq = np.array([0] * 9 + [1] * 30 + [2] * 4 + [3] * 21, dtype=np.int64)
    L = seq.shape[0]
    g = torch.Generator().manual_seed(3)
    emb = torch.randn(L, 64, generator=g).half().float()
    st = torch.tensor(seq)
    with torch.no_grad():
        mask = _flat_sequence_causal_mask(dtype=torch.float32, sequence_ids=st)
        pos = _flat_sequence_position_ids(sequence_ids=st)
        h = bb(emb[None], attention_mask=mask, position_ids=pos)[0]
    rec = {"seq": seq, "emb": emb.numpy(), "out": h.numpy(), "inv_freq": model.rotary_emb.inv_freq.numpy(),
           "eps": np.array(float(model.config.rms_norm_eps))}
    for key, val in _weights(model).items():
        rec["w:" + key] = val
    np.savez_compressed(HERE / "packed_fwd_qwen3.npz", **rec)


FIXTURES = ("index_maps", "kv_policy", "packed_attention", "decode", "packed_forward", "grow_rebuild", "embedding")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MOUSE_CORE_REFERENCE_SRC"),
                    help="the reference's src/ directory (or set MOUSE_CORE_REFERENCE_SRC)")
    ap.add_argument("--only", nargs="*", choices=FIXTURES, default=list(FIXTURES),
                    help="regenerate only these fixtures")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <reference src dir> or set MOUSE_CORE_REFERENCE_SRC")
    tmp = Path(tempfile.mkdtemp(prefix="mouse_ref_shim_"))
    _install_shims(tmp)
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch

    torch.set_num_threads(min(8, os.cpu_count() or 1))
    if "index_maps" in args.only:
        maps: dict = {}
        make_index_maps(maps)
        np.savez_compressed(HERE / "index_maps.npz", **maps)
    if "kv_policy" in args.only:
        (HERE / "kv_policy.json").write_text(json.dumps(make_kv_policy()))
    if "packed_attention" in args.only:
        make_packed_attention()
    if "decode" in args.only:
        make_decode("qwen3")
        make_decode("llama")
    if "packed_forward" in args.only:
        make_packed_forward()
    if "grow_rebuild" in args.only:
        make_grow_rebuild()
    if "embedding" in args.only:
        make_embedding()
    print("golden fixtures written to", HERE)


if __name__ == "__main__":
    main()
