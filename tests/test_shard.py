"""Batch sharding: the partition rule and a world-size-2 gloo run on CPU."""

import os

import numpy as np
import pytest
import torch.multiprocessing as mp

from yufmusicgen_b200.shard import gather_sharded, shard_range


@pytest.mark.parametrize("total,world", [(256, 1), (256, 2), (256, 8), (7, 3), (2, 8), (0, 4)])
def test_shard_range_partitions_exactly(total, world):
    seen = []
    for r in range(world):
        s, n = shard_range(total, world, r)
        assert n >= 0
        seen.extend(range(s, s + n))
    assert seen == list(range(total))


def test_shard_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        total = 10
        s, n = shard_range(total, world, rank)
        # each rank "decodes" its own sequences: here a deterministic per-sequence value
        local = [(i, float(np.sin(i))) for i in range(s, s + n)]
        merged = gather_sharded(local, world)
        q.put((rank, merged))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_shard_and_gather():
    import socket

    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        port = sk.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = [(i, float(np.sin(i))) for i in range(10)]
    assert res[0] == want and res[1] == want
