"""Packed DQN training step on the GPU: the bf16 tcgen05 path against the
reference's dense-mask SDPA training path run in fp32 (plain PyTorch) on the
same weights and rows."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda", 0)


def _rows(dev, lens_per_row, seed=3):
    from mouse_core_b200.train import PackedRow

    rng = np.random.default_rng(seed)
    rows = []
    for lens in lens_per_row:
        n = sum(lens)
        seq = np.concatenate([np.full(s, i) for i, s in enumerate(lens)])
        rows.append(PackedRow(
            token_ids=torch.from_numpy(rng.integers(0, 1024, size=n)).to(dev),
            sequence_ids=torch.from_numpy(seq).long().to(dev),
            action=torch.from_numpy(rng.integers(0, 4, size=n)).to(dev),
            reward=torch.from_numpy(rng.integers(0, 2, size=n).astype(np.float32)).to(dev),
            done=torch.from_numpy((rng.random(n) < 0.05).astype(np.int64)).to(dev),
            q_target=torch.from_numpy(rng.random((n, 4), dtype=np.float32)).to(dev)))
    return rows


def _models(dev):
    from mouse_core_b200.backbone import Qwen3Backbone
    from mouse_core_b200.train import ActionValueHead

    torch.manual_seed(0)
    bb = Qwen3Backbone(hidden_dim=256, num_layers=2, num_heads=4, num_key_value_heads=2, head_dim=128)
    emb = torch.nn.Embedding(1024, 256)
    head = ActionValueHead(256, 4)
    with torch.no_grad():
        for name, prm in bb.model.named_parameters():
            if "norm" not in name:
                prm.mul_(4.0)  # non-trivial attention at init
            prm.copy_(prm.bfloat16().float())
        emb.weight.copy_(emb.weight.bfloat16().float())
    return bb, emb, head


def _dense_loss(bb, emb, head, rows, total):
    from mouse_core_b200.packing import flat_sequence_causal_mask, flat_sequence_position_ids
    from mouse_core_b200.train import td_loss

    acc = 0.0
    for r in rows:
        mask = flat_sequence_causal_mask(sequence_ids=r.sequence_ids, dtype=torch.float32)
        pos = flat_sequence_position_ids(r.sequence_ids)
        h = bb(emb(r.token_ids)[None], attention_mask=mask, position_ids=pos)[0]
        loss = td_loss(head(h), r.q_target, r.action, r.reward, r.done, r.sequence_ids)
        (loss / total).backward()
        acc += float(loss)
    return acc


def _rel(a, b):
    return float((a.float() - b.float()).norm() / (b.float().norm() + 1e-12))


def test_trainer_step_matches_fp32_dense_path():
    dev = _dev()
    from mouse_core_b200.train import PackedDQNTrainer

    bb, emb, head = _models(dev)
    ref = [copy.deepcopy(m).to(dev) for m in (bb, emb, head)]
    bb = bb.to(device=dev, dtype=torch.bfloat16)
    emb = emb.to(device=dev, dtype=torch.bfloat16)
    head = head.to(dev)
    rows = _rows(dev, [[300, 45, 400, 1, 90], [512, 260]])

    opt = torch.optim.SGD(list(emb.parameters()) + list(bb.model.parameters()) + list(head.parameters()), lr=0.0)
    trainer = PackedDQNTrainer(emb, bb.model, head, opt)
    loss = float(trainer.step(rows, total_rows=2))
    ref_loss = _dense_loss(*ref, rows, 2)
    assert abs(loss - ref_loss) <= 2e-2 * max(1.0, abs(ref_loss))

    ours = dict(bb.model.named_parameters())
    checked = 0
    for name, p in ref[0].model.named_parameters():
        if p.grad is None or p.grad.norm() == 0:
            continue
        assert _rel(ours[name].grad, p.grad) < 5e-2, name
        checked += 1
    assert checked > 10
    assert _rel(emb.weight.grad, ref[1].weight.grad) < 5e-2
    for (n, a), b in zip(head.named_parameters(), ref[2].parameters()):
        assert _rel(a.grad, b.grad) < 5e-2, n


def test_trainer_step_updates_and_reduces_loss():
    dev = _dev()
    from mouse_core_b200.train import PackedDQNTrainer

    bb, emb, head = _models(dev)
    bb = bb.to(device=dev, dtype=torch.bfloat16)
    emb = emb.to(device=dev, dtype=torch.bfloat16)
    head = head.to(dev)
    rows = _rows(dev, [[200, 300, 12]], seed=5)
    params = list(emb.parameters()) + list(bb.model.parameters()) + list(head.parameters())
    opt = torch.optim.AdamW(params, lr=1e-3)
    trainer = PackedDQNTrainer(emb, bb.model, head, opt)
    before = head.out.weight.detach().clone()
    losses = [float(trainer.step(rows, total_rows=1)) for _ in range(8)]
    assert not torch.equal(before, head.out.weight)
    assert losses[-1] < losses[0]


def _reference_td(q, q_target, action, reward, done, seq, gammas, cql_weight, cql_eps):
    """DqnObjective.__call__ (objectives/dqn.py:116-213) restated in torch fp64."""
    valid = seq[1:] == seq[:-1]
    curr = q[:-1]
    a = action[1:]
    g = torch.tensor(gammas, dtype=q.dtype, device=q.device)[done[1:]]
    qv = curr.gather(-1, a.unsqueeze(-1)).squeeze(-1)
    target = reward[1:].to(q.dtype) + g * q_target[1:].amax(-1)
    loss = (qv - target.detach()) ** 2
    if cql_weight > 0:
        scale = (target.abs() + cql_eps).detach()
        loss = loss + cql_weight * scale * (torch.logsumexp(curr, -1) - qv)
    m = curr.amax(-1).detach()[valid]
    return loss[valid].mean(), torch.stack([valid.sum().to(q.dtype), m.mean(), m.std(), m.min(), m.max()])


@pytest.mark.parametrize("cql_weight", [0.0, 0.5])
def test_fused_td_loss_matches_the_objective(cql_weight):
    """K12's loss, metrics and gradient against DqnObjective's formulas (fp64),
    over a packed stream with several sequences and every done code."""
    dev = _dev()
    from mouse_core_b200.train import td_loss_fused

    g = torch.Generator().manual_seed(4)
    N, A = 5000, 4
    q = torch.randn(N, A, generator=g).to(dev).requires_grad_(True)
    qt = torch.rand(N, A, generator=g).to(dev)
    action = torch.randint(0, A, (N,), generator=g).to(dev)
    reward = torch.randn(N, generator=g).to(dev)
    done = torch.randint(0, 5, (N,), generator=g).to(dev)
    seq = torch.sort(torch.randint(0, 37, (N,), generator=g)).values.to(dev)
    gammas = (0.99, 0.5, 0.9, 0.0, 0.25)
    loss, metrics = td_loss_fused(q, qt, action, reward, done, seq, gammas, cql_weight, 1.0)
    loss.backward()
    q64 = q.detach().double().requires_grad_(True)
    ref_loss, ref_metrics = _reference_td(q64, qt.double(), action, reward, done, seq, gammas, cql_weight, 1.0)
    ref_loss.backward()
    assert abs(loss.item() - ref_loss.item()) <= 1e-5 * max(1.0, abs(ref_loss.item()))
    assert torch.allclose(metrics.double(), ref_metrics, rtol=1e-5, atol=1e-5)
    assert torch.allclose(q.grad.double(), q64.grad, rtol=1e-4, atol=1e-8)
    from mouse_core_b200 import _lib

    assert _lib.device_status() == 0
