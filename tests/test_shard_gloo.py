"""Multi-rank host logic on CPU: view / row-band sharding covers every unit
exactly once, and the flat gradient bucket all-reduces across gloo ranks."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from vorotracing_b200.shard import GradBucket, row_band_shard, view_shard


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shards_partition(world):
    views = sorted(v for r in range(world) for v in view_shard(64, r, world))
    assert views == list(range(64))
    rows = np.sort(np.concatenate([row_band_shard(1080, r, world) for r in range(world)]))
    np.testing.assert_array_equal(rows, np.arange(1080))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    b = GradBucket(5, 12, "cpu")
    for i, t in enumerate(b.views()):
        t.fill_(float(rank + 1) * (i + 1))
    b.allreduce_()
    tot = sum(r + 1 for r in range(world))
    ok = all(torch.all(t == tot * (i + 1)).item() for i, t in enumerate(b.views()))
    b.allreduce_(average=True)
    ok = ok and torch.allclose(b.points, torch.full_like(b.points, tot * world / world))
    q.put((rank, ok))
    dist.destroy_process_group()


def test_grad_bucket_allreduce_gloo():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert all(ok for _, ok in res), res


def test_bucket_layout():
    b = GradBucket(7, 48, "cpu")
    assert b.flat.numel() == 7 * (3 + 1 + 96)
    assert b.points.data_ptr() == b.flat.data_ptr()
    assert b.nbytes == b.flat.numel() * 4
