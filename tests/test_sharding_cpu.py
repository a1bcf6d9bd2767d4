"""Multi-process host logic on CPU: world-size-2 gloo ranks (no GPU).

Covers the round-robin sequence sharding of the serving configuration and the
max-over-ranks reduction bench.py applies to device-timed intervals.
"""
import os
import socket

import pytest


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    from smallmind_b200 import sharding
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        mine = sharding.shard_sequences(256, world, rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, mine)
        t_max = sharding.max_over_ranks(10.0 + 5.0 * rank)
        n_sum = sharding.sum_over_ranks(len(mine))
        out.put((rank, gathered, t_max, n_sum))
    finally:
        dist.destroy_process_group()


def test_shard_sequences_single_process():
    from smallmind_b200 import sharding
    assert sharding.shard_sequences(5, 2, 0) == [0, 2, 4]
    assert sharding.shard_sequences(5, 2, 1) == [1, 3]
    assert sharding.shard_sequences(0, 4, 3) == []
    with pytest.raises(ValueError):
        sharding.shard_sequences(4, 2, 2)
    assert sharding.max_over_ranks(3.5) == 3.5  # no process group: identity


def test_gloo_world2_sharding_and_max():
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, gathered, t_max, n_sum in res:
        assert t_max == 15.0  # the slower rank sets the job time
        assert n_sum == 256
        flat = sorted(i for part in gathered for i in part)
        assert flat == list(range(256))  # disjoint and complete
        assert all(len(part) == 128 for part in gathered)
