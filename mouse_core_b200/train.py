"""Data-parallel packed training step: one gradient all-reduce per step.

The reference trains on one device: ``Model.forward(TokenBatch)`` routes the
packed stream through ``flex_packed_forward`` (models/base.py:948-981), the
heads produce per-step Q values and ``DqnObjective`` (objectives/dqn.py:
116-213) computes the TD loss, followed by ``loss.backward()`` and
``optimizer.step()``. Here the packed rows of a step are split across ranks
(one process per GPU); each rank runs forward/backward on its rows through
the tcgen05 attention, the summed gradients cross NVLink in ONE all-reduce
of a flat fp32 buffer (NCCL), and every rank applies the same optimizer
update. Nothing else is communicated.

``td_loss`` restates the reference's TD loss for the synthetic workload, with
the target network's output supplied as an input tensor.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.distributed as dist


def td_loss(q: torch.Tensor, q_target: torch.Tensor, action: torch.Tensor, reward: torch.Tensor,
            done: torch.Tensor, sequence_id: torch.Tensor, gammas=(0.99, 0.0, 0.99, 0.0, 0.0)) -> torch.Tensor:
    """One-step TD loss over a flat ``[N]`` step stream (objectives/dqn.py:116-213).

    The transition out of step ``i`` is described by the fields stored at
    ``i + 1`` (action taken, reward, done code), pairs crossing a
    ``sequence_id`` boundary are dropped, the discount is ``gammas[done]``:
    ``loss = mean((Q(s_i, a_{i+1}) - (r_{i+1} + g * max_a Q_target(s_{i+1})))^2)``.
    """
    N = q.shape[0]
    if N < 2:
        raise ValueError("Not enough valid q values in data.")
    valid = sequence_id[1:] == sequence_id[:-1]
    g = torch.tensor(gammas, dtype=q.dtype, device=q.device)[done[1:]]
    q_sa = q[:-1].gather(-1, action[1:].unsqueeze(-1)).squeeze(-1)
    target = (reward[1:] + g * q_target[1:].amax(-1)).detach()
    err = (q_sa - target) ** 2
    return err[valid].mean()


class GradientAllReduce:
    """Sum the gradients of ``params`` across ranks with one collective.

    Gradients are packed into one persistent fp32 buffer, all-reduced once
    (sum), scaled by ``scale`` and written back. With a single rank it only
    applies the scale, in place, and never allocates the buffer.
    """

    def __init__(self, params, group=None):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.device = self.params[0].device if self.params else torch.device("cpu")
        self._flat = None

    @property
    def flat(self) -> torch.Tensor:
        """The fp32 exchange buffer, allocated on first use (multi-rank only)."""
        if self._flat is None:
            n = sum(p.numel() for p in self.params)
            self._flat = torch.zeros(n, dtype=torch.float32, device=self.device)
        return self._flat

    def __call__(self, scale: float = 1.0) -> None:
        world = dist.get_world_size(self.group) if dist.is_available() and dist.is_initialized() else 1
        if world == 1:
            # nothing to exchange: scale in place, no round trip through the buffer
            if scale != 1.0:
                grads = [p.grad for p in self.params if p.grad is not None]
                if grads:
                    torch._foreach_mul_(grads, scale)
            return
        o = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None:
                self.flat[o:o + n].zero_()
            else:
                self.flat[o:o + n].copy_(p.grad.reshape(-1))
            o += n
        if world > 1:
            dist.all_reduce(self.flat, op=dist.ReduceOp.SUM, group=self.group)
        if scale != 1.0:
            self.flat.mul_(scale)
        o = 0
        for p in self.params:
            n = p.numel()
            if p.grad is None:
                p.grad = torch.empty_like(p)
            p.grad.copy_(self.flat[o:o + n].view_as(p.grad))
            o += n


class ActionValueHead(torch.nn.Module):
    """fp32 per-action value head: RMSNorm(eps 1e-5) -> SwiGLU(D -> hidden)
    -> Linear(hidden -> actions), the two-layer ``DiscreteActionValueHead``
    online network (models/heads/dqn.py:11-47, heads/swiglu.py:13-74)."""

    def __init__(self, in_features: int, actions: int = 4, hidden: int | None = None):
        super().__init__()
        hidden = hidden or in_features
        self.norm = torch.nn.RMSNorm(in_features, eps=1e-5)
        self.up = torch.nn.Linear(in_features, 2 * hidden)
        self.out = torch.nn.Linear(hidden, actions)

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        a, b = self.up(self.norm(h)).chunk(2, dim=-1)
        return self.out(torch.nn.functional.silu(a) * b)


@dataclass
class PackedRow:
    """One packed training row: ``token_ids``, ``sequence_ids``, ``action``,
    ``done`` (int64 ``[L]``), ``reward`` (f32 ``[L]``), ``q_target`` (f32 ``[L, A]``)."""

    token_ids: torch.Tensor
    sequence_ids: torch.Tensor
    action: torch.Tensor
    reward: torch.Tensor
    done: torch.Tensor
    q_target: torch.Tensor


class PackedDQNTrainer:
    """Data-parallel DQN step over packed rows with the tcgen05 attention.

    ``embedding`` maps token ids to ``[L, D]``, ``backbone_model`` is the
    transformers stack (bf16, CUDA), ``head`` maps hidden states (fp32) to
    ``[L, A]`` action values. ``step(rows, total_rows)`` runs this rank's rows
    (forward + backward, gradients accumulated and pre-divided by the global
    row count), one all-reduce, then the optimizer update.
    """

    def __init__(self, embedding, backbone_model, head, optimizer, group=None):
        from mouse_core_b200.packed import flex_packed_forward

        self._forward = flex_packed_forward
        self.embedding, self.model, self.head, self.opt = embedding, backbone_model, head, optimizer
        params = list(embedding.parameters()) + list(backbone_model.parameters()) + list(head.parameters())
        self.reduce = GradientAllReduce(params, group)

    def step(self, rows, total_rows: int) -> torch.Tensor:
        """One optimizer step; returns this rank's summed row losses as a
        device scalar (no host sync)."""
        self.opt.zero_grad(set_to_none=True)
        loss_sum = torch.zeros((), device=self.reduce.device)
        for row in rows:
            emb = self.embedding(row.token_ids)
            h = self._forward(model=self.model, embeds=emb, sequence_ids=row.sequence_ids)
            q = self.head(h.float())
            loss = td_loss(q, row.q_target, row.action, row.reward, row.done, row.sequence_ids)
            (loss / total_rows).backward()
            loss_sum = loss_sum + loss.detach()
        self.reduce()
        self.opt.step()
        return loss_sum
