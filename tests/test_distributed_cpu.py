"""Host-side data parallelism on CPU ranks (gloo, world size 2).

1. Gradient all-reduce: averaging per-shard gradients equals the
   single-process gradient of the mean loss over the whole batch.
2. Failure detection: a rank that exits without joining the collective
   makes the survivor's all-reduce fail with an error within the process
   group timeout (no hang).
"""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from manifold_b200.distributed import allreduce_gradients, shard_rows


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _model():
    torch.manual_seed(0)
    return torch.nn.Sequential(torch.nn.Linear(8, 16), torch.nn.Tanh(), torch.nn.Linear(16, 3))


def _data():
    g = torch.Generator().manual_seed(1)
    return torch.randn(10, 8, generator=g), torch.randn(10, 3, generator=g)


def _worker_allreduce(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    m = _model()
    x, y = _data()
    xs, ys = shard_rows(x, rank, world), shard_rows(y, rank, world)
    loss = ((m(xs) - ys) ** 2).sum() / x.shape[0] * world  # per-shard share of the global mean
    loss.backward()
    allreduce_gradients(list(m.parameters()), bucket_bytes=256)
    out[rank] = [p.grad.clone() for p in m.parameters()]
    dist.destroy_process_group()


def test_gradient_allreduce_matches_single_process():
    world = 2
    out = mp.Manager().dict()
    mp.spawn(_worker_allreduce, args=(world, _port(), out), nprocs=world, join=True)
    m = _model()
    x, y = _data()
    (((m(x) - y) ** 2).sum() / x.shape[0]).backward()
    ref = [p.grad for p in m.parameters()]
    for rank in range(world):
        for a, b in zip(out[rank], ref):
            torch.testing.assert_close(a, b, rtol=1e-5, atol=1e-6)


def _worker_dead_peer(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        os._exit(0)  # leaves between steps, never joins the collective
    try:
        t = torch.ones(4)
        dist.all_reduce(t)
        out[rank] = "no error"
    except Exception as e:  # noqa: BLE001 - any error is the expected outcome
        out[rank] = "error: " + type(e).__name__


def test_dead_rank_surfaces_as_collective_error():
    world = 2
    out = mp.Manager().dict()
    ctx = mp.spawn(_worker_dead_peer, args=(world, _port(), out), nprocs=world, join=False)
    ctx.processes[0].join(60)
    assert not ctx.processes[0].is_alive(), "survivor hung instead of timing out"
    for p in ctx.processes:
        p.join(5)
    assert out.get(0, "").startswith("error"), out.get(0)


def test_shard_rows_covers_batch():
    t = torch.arange(10)
    parts = [shard_rows(t, r, 3) for r in range(3)]
    assert torch.equal(torch.cat(parts), t)
    assert [len(p) for p in parts] == [4, 4, 2]
