"""Host-side sharding and the gather of configs 3 and 4, as world-size-2
gloo process groups on CPU."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from llm_mojo_b200.shard import gather_blocks, shard_range


def test_shard_range_covers_every_unit_once():
    for world in (1, 2, 4, 8):
        seen = []
        for r in range(world):
            b, e = shard_range(256, world, r)
            seen.extend(range(b, e))
        assert seen == list(range(256))


def test_shard_range_rejects_uneven_splits():
    with pytest.raises(ValueError):
        shard_range(10, 4, 0)
    with pytest.raises(ValueError):
        shard_range(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        n, steps = 8, 5
        b, e = shard_range(n, world, rank)
        # each rank "generates" ids that identify the unit and step
        local = torch.tensor([[u * 100 + t for t in range(steps)] for u in range(b, e)], dtype=torch.int32)
        out = gather_blocks(local, world)
        q.put((rank, out.numpy()))
    finally:
        dist.destroy_process_group()


def test_gather_blocks_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=60) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.array([[u * 100 + t for t in range(5)] for u in range(8)], dtype=np.int32)
    assert np.array_equal(got[0], want) and np.array_equal(got[1], want)


def test_schedule_scores_every_token_once():
    from llm_mojo_b200.evaluate import schedule

    n = 65536
    seen = []
    for begin, end, r0, r1 in schedule(n):
        seen.extend(begin + r + 1 for r in range(r0, r1))
    assert seen == list(range(1, n)) and len(schedule(n)) == 127
