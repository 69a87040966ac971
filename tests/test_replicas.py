"""The N>1 replica path on CPU: world_size-2 gloo ranks, no GPU.

Each rank processes its round-robin share with a stand-in per-image function,
the shares are gathered and must cover every image exactly once in order, and
the timing reduction must return the slowest rank's value.
"""

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from lama_b200.replicas import chunks, max_over_ranks, shard


def test_shard_and_chunks():
    assert shard(10, 0, 4) == [0, 4, 8]
    assert shard(10, 3, 4) == [3, 7]
    assert sorted(sum((shard(256, r, 8) for r in range(8)), [])) == list(range(256))
    assert chunks(70, 32) == [(0, 32), (32, 32), (64, 6)]
    with pytest.raises(ValueError):
        shard(4, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        mine = shard(37, rank, world)
        done = []
        for s, c in chunks(len(mine), 5):
            done += [mine[s + i] * 10 for i in range(c)]  # stand-in for one engine call per chunk
        gathered = [None] * world
        dist.all_gather_object(gathered, done)
        slowest = max_over_ranks(1.5 + rank, world)
        q.put((rank, gathered, slowest))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_cover_every_image_once():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, slowest in results:
        flat = sorted(v for part in gathered for v in part)
        assert flat == [i * 10 for i in range(37)]
        assert slowest == 2.5
