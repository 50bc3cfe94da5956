"""Data-parallel step logic on CPU with two gloo ranks.

Each rank computes the gradient of its half of a batch; after the flat
all-reduce both ranks hold the gradient of the mean loss over the whole batch
(what one process computes on the full batch), and the replicas stay
identical after an optimizer step.
"""

from __future__ import annotations

import os

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(6, 5), torch.nn.Tanh(), torch.nn.Linear(5, 3))


def _batch():
    g = torch.Generator().manual_seed(1)
    return torch.randn(8, 6, generator=g), torch.randn(8, 3, generator=g)


def _worker(rank, world, port, out, bucket_bytes=None):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from dabsn_b200.data_parallel import FlatGradAllReduce

        model = _model()
        if rank == 1:  # a different start: the broadcast must replicate rank 0
            with torch.no_grad():
                for p in model.parameters():
                    p.add_(1.0)
        # a parameter the loss does not use: its bucket is launched by
        # all_reduce() itself, not by a hook
        unused = torch.nn.Parameter(torch.zeros(3))
        dp = FlatGradAllReduce(list(model.parameters()) + [unused], "cpu",
                               bucket_bytes=bucket_bytes)
        if bucket_bytes is not None:
            assert len(dp.buckets) > 1
        opt = torch.optim.SGD(model.parameters(), lr=0.1)
        x, y = _batch()
        xs, ys = x.chunk(world)[rank], y.chunk(world)[rank]
        for _ in range(2):
            dp.zero()
            torch.nn.functional.mse_loss(model(xs), ys).backward()
            dp.all_reduce()
            grads = [p.grad.clone() for p in model.parameters()]
            opt.step()
        out[rank] = ([g.numpy() for g in grads], [p.detach().numpy().copy() for p in model.parameters()])
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("bucket_bytes", [None, 64])
def test_flat_all_reduce_matches_full_batch(bucket_bytes):
    import socket

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    manager = mp.Manager()
    out = manager.dict()
    mp.spawn(_worker, args=(2, port, out, bucket_bytes), nprocs=2, join=True)
    # single process, full batch, same two steps
    model = _model()
    opt = torch.optim.SGD(model.parameters(), lr=0.1)
    x, y = _batch()
    for _ in range(2):
        opt.zero_grad()
        torch.nn.functional.mse_loss(model(x), y).backward()
        grads = [p.grad.clone() for p in model.parameters()]
        opt.step()
    for rank in (0, 1):
        g_r, p_r = out[rank]
        for a, e in zip(g_r, grads):
            assert torch.allclose(torch.from_numpy(a), e, atol=1e-6, rtol=1e-5)
        for a, e in zip(p_r, model.parameters()):
            assert torch.allclose(torch.from_numpy(a), e.detach(), atol=1e-6, rtol=1e-5)
