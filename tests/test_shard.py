"""The multi-GPU split of fold windows and the max over ranks, on CPU (gloo, world size 2)."""

import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from taco_b200 import shard


def test_deal_covers_every_window_once():
    for n, world in [(512 * 8, 8), (10, 3), (1, 4), (0, 2)]:
        parts = [shard.deal(n, world, r) for r in range(world)]
        got = np.sort(np.concatenate(parts)) if n else np.zeros(0, np.int64)
        assert np.array_equal(got, np.arange(n))
        sizes = [p.size for p in parts]
        assert max(sizes) - min(sizes) <= 1
    order = shard.gather_order(10, 3)
    assert sorted(order.tolist()) == list(range(10))
    with pytest.raises(ValueError):
        shard.deal(4, 2, 2)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = shard.deal(16, world, rank)
        # Rank r reports a device time of 1 + r and a wall time of 10 - r.
        got = shard.max_over_ranks([1.0 + rank, 10.0 - rank])
        q.put((rank, mine.tolist(), got))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_with_two_gloo_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict()
    for _ in range(world):
        rank, mine, got = q.get(timeout=120)
        res[rank] = (mine, got)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert res[0][0] == list(range(0, 16, 2)) and res[1][0] == list(range(1, 16, 2))
    for r in range(world):
        assert res[r][1] == [2.0, 10.0]
