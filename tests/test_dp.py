"""Host logic of data-parallel training on CPU (gloo, world size 2): one
all-reduce of the flat gradient buffer reproduces the single-process
gradient of the full batch, and the TD loss follows the reference's
transition rules."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mouse_core_b200.train import GradientAllReduce, td_loss


def _tiny(seed=0):
    torch.manual_seed(seed)
    return torch.nn.Sequential(torch.nn.Linear(6, 8), torch.nn.Tanh(), torch.nn.Linear(8, 4))


def _batches(seed=1, rows=4):
    g = torch.Generator().manual_seed(seed)
    return [torch.randn(10, 6, generator=g) for _ in range(rows)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out, armed, bucket_bytes):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        model = _tiny()
        rows = _batches()
        mine = rows[rank::world]
        reduce = GradientAllReduce(model.parameters(), bucket_bytes=bucket_bytes)
        for step in range(2):  # the reducer is reused across steps
            model.zero_grad(set_to_none=True)
            for i, x in enumerate(mine):
                if armed and i == len(mine) - 1:
                    reduce.arm()  # buckets go out from the last backward's hooks
                (model(x).pow(2).mean() / len(rows)).backward()
            reduce()
        out[rank] = [p.grad.clone() for p in model.parameters()]
        out[f"buckets{rank}"] = len(reduce.buckets)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("armed,bucket_bytes", [(False, 64 << 20), (True, 64 << 20), (True, 100)])
def test_one_allreduce_matches_single_process_gradient(armed, bucket_bytes):
    """One logical all-reduce per step, in one bucket or (100-byte buckets)
    two, launched by __call__ or from the backward hooks."""
    model = _tiny()
    rows = _batches()
    for x in rows:
        (model(x).pow(2).mean() / len(rows)).backward()
    ref = [p.grad.clone() for p in model.parameters()]
    manager = mp.Manager()
    out = manager.dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out, armed, bucket_bytes)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(2):
        for a, b in zip(out[rank], ref):
            assert torch.allclose(a, b, atol=1e-6)
    assert out["buckets0"] == (2 if bucket_bytes == 100 else 1)


def _dead_peer_worker(rank, port, out):
    """Rank 1 stops before the step's all-reduce (it never joins it and exits
    later); rank 0 must get an error from the process group's timeout instead
    of waiting forever."""
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=timedelta(seconds=3))
    model = _tiny()
    (model(_batches()[rank]).pow(2).mean()).backward()
    if rank == 1:
        time.sleep(8)  # gone from the step: no collective
        out[rank] = "left"
        return
    t0 = time.monotonic()
    try:
        GradientAllReduce(model.parameters())()
        out[rank] = "no error"
    except Exception as e:  # the process group reports the missing peer
        out[rank] = f"error after {time.monotonic() - t0:.1f}s: {type(e).__name__}"


def test_dead_peer_ends_the_allreduce_with_an_error():
    manager = mp.Manager()
    out = manager.dict()
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dead_peer_worker, args=(r, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        for p in procs:
            p.join(timeout=90)
    finally:
        for p in procs:
            if p.is_alive():
                p.kill()
    assert out.get(1) == "left"
    msg = out.get(0, "no result (hung)")
    assert msg.startswith("error after"), msg
    assert float(msg.split()[2].rstrip("s:")) < 30, msg


def test_single_rank_reduce_only_scales():
    model = _tiny()
    model(torch.ones(2, 6)).sum().backward()
    before = [p.grad.clone() for p in model.parameters()]
    GradientAllReduce(model.parameters())(scale=0.5)
    for a, b in zip(model.parameters(), before):
        assert torch.allclose(a.grad, b * 0.5)


def test_td_loss_follows_reference_transition_rules():
    q = torch.tensor([[1.0, 2.0], [3.0, 4.0], [5.0, 6.0], [7.0, 8.0]], requires_grad=True)
    qt = torch.tensor([[0.5, 0.1], [0.2, 0.9], [1.0, 0.0], [0.3, 0.4]])
    action = torch.tensor([0, 1, 0, 1])
    reward = torch.tensor([0.0, 1.0, 2.0, 3.0])
    done = torch.tensor([0, 0, 1, 0])
    seq = torch.tensor([0, 0, 0, 1])  # pair (2, 3) crosses sequences
    loss = td_loss(q, qt, action, reward, done, seq, gammas=(0.9, 0.0, 0.5, 0.0, 0.0))
    # pair 0: Q(s0, a=1)=2, target = 1 + 0.9 * max(0.2, 0.9) = 1.81
    # pair 1: Q(s1, a=0)=3, target = 2 + 0.0 * 1.0 = 2.0 (done code 1 -> gamma 0)
    expect = ((2 - 1.81) ** 2 + (3 - 2.0) ** 2) / 2
    assert abs(loss.item() - expect) < 1e-6
    with pytest.raises(ValueError):
        td_loss(q[:1], qt[:1], action[:1], reward[:1], done[:1], seq[:1])
