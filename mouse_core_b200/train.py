"""Data-parallel packed training step: one gradient all-reduce per step.

The reference trains on one device: ``Model.forward(TokenBatch)`` routes the
packed stream through ``flex_packed_forward`` (models/base.py:948-981), the
heads produce per-step Q values and ``DqnObjective`` (objectives/dqn.py:
116-213) computes the TD loss, followed by ``loss.backward()`` and
``optimizer.step()``. Here the packed rows of a step are split across ranks
(one process per GPU); each rank runs forward/backward on its rows through
the tcgen05 attention, the summed gradients cross NVLink in ONE logical
all-reduce (NCCL, fp32), cut into buckets launched from backward hooks so it
overlaps the last row's backward, and every rank applies the same optimizer
update. Nothing else is communicated.

``td_loss`` restates the reference's TD loss for the synthetic workload, with
the target network's output supplied as an input tensor.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from mouse_core_b200.trace import nvtx_range


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


class _FusedTDLoss(torch.autograd.Function):
    """K12 forward (loss + metrics, no host sync) and backward (d loss / d q)."""

    @staticmethod
    def forward(ctx, q, q_target, action, reward, done, sequence_id, gammas, cql_weight, cql_eps):
        from mouse_core_b200 import _lib

        q = q.contiguous().float()
        N, A = q.shape
        lib = _lib.load()
        scratch = torch.zeros(int(lib.mb_td_loss_scratch_bytes(N)), dtype=torch.uint8, device=q.device)
        out = torch.empty(6, dtype=torch.float32, device=q.device)
        g = (ctypes.c_float * 5)(*[float(x) for x in gammas])  # host array, alive through the call
        _lib.call("mb_td_loss_fwd", q.data_ptr(), q_target.contiguous().float().data_ptr(),
                  action.contiguous().data_ptr(), reward.contiguous().float().data_ptr(), done.contiguous().data_ptr(),
                  None if sequence_id is None else sequence_id.contiguous().data_ptr(), N, A,
                  ctypes.cast(g, ctypes.c_void_p), float(cql_weight),
                  float(cql_eps), scratch.data_ptr(), scratch.numel(), out.data_ptr(),
                  torch.cuda.current_stream(q.device).cuda_stream)
        ctx.save_for_backward(q, action.contiguous(), out)
        ctx.scratch, ctx.cql_weight = scratch, float(cql_weight)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        from mouse_core_b200 import _lib

        q, action, out = ctx.saved_tensors
        N, A = q.shape
        dq = torch.empty_like(q)
        g = grad_out.contiguous().float()
        _lib.call("mb_td_loss_bwd", q.data_ptr(), action.data_ptr(), N, A, ctx.cql_weight, ctx.scratch.data_ptr(),
                  ctx.scratch.numel(), out.data_ptr(), g.data_ptr(), dq.data_ptr(),
                  torch.cuda.current_stream(q.device).cuda_stream)
        return dq, None, None, None, None, None, None, None, None


def td_loss_fused(q: torch.Tensor, q_target: torch.Tensor, action: torch.Tensor, reward: torch.Tensor,
                  done: torch.Tensor, sequence_id: torch.Tensor | None, gammas=(0.99, 0.0, 0.99, 0.0, 0.0),
                  cql_weight: float = 0.0, cql_eps: float = 1.0):
    """``td_loss`` (plus ``DqnObjective``'s optional CQL term and its metrics)
    as one CUDA kernel forward and one backward: returns ``(loss, metrics)``
    with ``metrics`` a device tensor ``[valid pairs, q_values_mean,
    q_values_std, q_values_min, q_values_max]`` read back only if the caller
    asks (the reference syncs to build its dict). Gradients flow to ``q``."""
    if q.ndim != 2:
        raise ValueError(f"DQN expects action_value shape [N, A], got {tuple(q.shape)}.")
    if q.shape[0] < 2:
        raise ValueError("Not enough valid q values in data.")
    if q.device.type != "cuda":
        raise RuntimeError("the fused TD loss runs on a CUDA device (B200, sm_100a) only")
    out = _FusedTDLoss.apply(q, q_target.detach(), action, reward, done, sequence_id, tuple(gammas), cql_weight,
                             cql_eps)
    return out[0], out[1:].detach()


class GradientAllReduce:
    """Sum the gradients of ``params`` across ranks: one logical all-reduce
    per step, cut into buckets that go out while the backward still runs.

    Parameters are grouped into fp32 buckets of about ``bucket_bytes``, last
    registered first (the order the backward finishes them). A hook on every
    parameter (``register_post_accumulate_grad_hook``) counts its bucket's
    final gradients once the reducer is armed; a full bucket is copied into its
    buffer and all-reduced asynchronously (NCCL on its own stream, after the
    gradient kernels of the current stream). Buckets always launch in index
    order, so every rank issues the same collectives in the same order even
    if its hooks fire in another one; ``__call__`` launches whatever the hooks
    did not (parameters without a gradient count as zeros), waits, scales and
    writes the sums back into ``.grad``.

    Use: ``arm()`` right before a step's last backward (earlier backwards of
    the step only accumulate), then ``__call__(scale)`` after it. Without
    ``arm()`` the call reduces every bucket itself (no overlap). With one rank
    nothing is exchanged or allocated: the call only scales.
    """

    def __init__(self, params, group=None, bucket_bytes: int = 64 << 20):
        self.params = [p for p in params if p.requires_grad]
        self.group = group
        self.device = self.params[0].device if self.params else torch.device("cpu")
        self.world = dist.get_world_size(group) if dist.is_available() and dist.is_initialized() else 1
        self.buckets: list[list[int]] = []
        cur, size = [], 0
        for i in reversed(range(len(self.params))):
            cur.append(i)
            size += self.params[i].numel() * 4
            if size >= bucket_bytes:
                self.buckets.append(cur)
                cur, size = [], 0
        if cur:
            self.buckets.append(cur)
        self._bucket_of = {i: b for b, idx in enumerate(self.buckets) for i in idx}
        self._flat: list[torch.Tensor | None] = [None] * len(self.buckets)
        self._works: list = [None] * len(self.buckets)
        self._pending = [len(b) for b in self.buckets]
        self._next = 0
        self._armed = False
        self._hooks = []
        if self.world > 1:
            for i, p in enumerate(self.params):
                self._hooks.append(p.register_post_accumulate_grad_hook(self._hook(i)))

    def _hook(self, i: int):
        def on_grad(_param):
            if not self._armed:
                return
            b = self._bucket_of[i]
            self._pending[b] -= 1
            while self._next < len(self.buckets) and self._pending[self._next] == 0:
                self._launch(self._next)
                self._next += 1
        return on_grad

    def _buffer(self, b: int) -> torch.Tensor:
        if self._flat[b] is None:
            n = sum(self.params[i].numel() for i in self.buckets[b])
            self._flat[b] = torch.zeros(n, dtype=torch.float32, device=self.device)
        return self._flat[b]

    def _launch(self, b: int) -> None:
        flat = self._buffer(b)
        grads = [self.params[i].grad for i in self.buckets[b]]
        if all(g is not None for g in grads):
            torch.cat([g.reshape(-1) for g in grads], out=flat)
        else:
            o = 0
            for i, g in zip(self.buckets[b], grads):
                n = self.params[i].numel()
                if g is None:
                    flat[o:o + n].zero_()
                else:
                    flat[o:o + n].copy_(g.reshape(-1))
                o += n
        with nvtx_range(f"grad_allreduce_bucket{b}"):
            self._works[b] = dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=self.group, async_op=True)

    @property
    def flat(self) -> torch.Tensor:
        """All buckets' exchange buffers as one tensor (a copy; for inspection)."""
        return torch.cat([self._buffer(b) for b in range(len(self.buckets))]) if self.buckets else torch.zeros(0)

    def arm(self) -> None:
        """The next backward is the step's last: launch buckets as they fill."""
        if self.world > 1:
            self._pending = [len(b) for b in self.buckets]
            self._next = 0
            self._armed = True

    def __call__(self, scale: float = 1.0) -> None:
        if self.world == 1:
            # nothing to exchange: scale in place, no round trip through a buffer
            if scale != 1.0:
                grads = [p.grad for p in self.params if p.grad is not None]
                if grads:
                    torch._foreach_mul_(grads, scale)
            return
        with nvtx_range("grad_allreduce_wait"):
            self._finish(scale)

    def _finish(self, scale: float) -> None:
        self._armed = False
        while self._next < len(self.buckets):  # the buckets the hooks did not launch
            self._launch(self._next)
            self._next += 1
        for b, work in enumerate(self._works):
            work.wait()
            flat = self._flat[b]
            if scale != 1.0:
                flat.mul_(scale)
            idx = self.buckets[b]
            for i in idx:
                if self.params[i].grad is None:
                    self.params[i].grad = torch.empty_like(self.params[i])
            sizes = [self.params[i].numel() for i in idx]
            grads = [self.params[i].grad for i in idx]
            torch._foreach_copy_(grads, [t.view_as(g) for t, g in zip(flat.split(sizes), grads)])
        self._works = [None] * len(self.buckets)
        self._next = 0
        self._pending = [len(b) for b in self.buckets]


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
        for r, row in enumerate(rows):
            emb = self.embedding(row.token_ids)
            h = self._forward(model=self.model, embeds=emb, sequence_ids=row.sequence_ids)
            q = self.head(h.float())
            loss, _ = td_loss_fused(q, row.q_target, row.action, row.reward, row.done, row.sequence_ids)
            if r == len(rows) - 1:
                self.reduce.arm()  # gradients become final during this backward
            (loss / total_rows).backward()
            loss_sum = loss_sum + loss.detach()
        self.reduce()
        self.opt.step()
        return loss_sum
