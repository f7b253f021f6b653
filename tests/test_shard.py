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


def _fake_window_stats(begin, r0, r1):
    """Deterministic per-row statistics of a window (score_rows' layout
    [6, rows]) as functions of the scored token's index."""
    idx = torch.arange(begin + r0 + 1, begin + r1 + 1, dtype=torch.float64)
    return torch.stack([torch.log1p(idx), torch.log1p(idx) * 0.9, (idx % 3 == 0).double(), 1.0 / idx,
                        torch.sin(idx) ** 2 + (idx == 40000).double() * 7.0, torch.cos(idx) ** 2])


def _eval_worker(rank, world, port, q):
    import torch.distributed as dist

    from llm_mojo_b200.evaluate import accumulate, reduce_totals, report_totals, schedule

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from llm_mojo_b200.evaluate import rank_windows

        totals = {name: torch.zeros(7, dtype=torch.float64) for name in ("int4-g32-a16", "bf16")}
        for k, (begin, end, r0, r1) in enumerate(rank_windows(schedule(65536), world, rank)):
            for j, t in enumerate(totals.values()):
                accumulate(t, _fake_window_stats(begin, r0, r1) * (1 + j), r1 - r0)
        reduce_totals(totals, world)
        q.put((rank, {n: t.numpy().copy() for n, t in totals.items()}, report_totals(totals, 50257, True)))
    finally:
        dist.destroy_process_group()


def test_config4_totals_reduce_over_two_gloo_ranks():
    """The perplexity harness's windows split round-robin over two ranks and
    the one all-reduce of the totals (sums, and the max of the largest logit
    difference) give every rank the totals a single process accumulates."""
    from llm_mojo_b200.evaluate import accumulate, report_totals, schedule

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_eval_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = {r: (t, rep) for r, t, rep in (q.get(timeout=120) for _ in procs)}
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = {name: torch.zeros(7, dtype=torch.float64) for name in ("int4-g32-a16", "bf16")}
    for begin, end, r0, r1 in schedule(65536):
        for j, t in enumerate(want.values()):
            accumulate(t, _fake_window_stats(begin, r0, r1) * (1 + j), r1 - r0)
    for r in (0, 1):
        totals, rep = got[r]
        for name, w in want.items():
            w = w.numpy()
            assert totals[name][6] == w[6] == 65535  # every token after the first, once
            assert totals[name][5] == w[5]  # the max is exact
            np.testing.assert_allclose(totals[name][:5], w[:5], rtol=1e-12)
        assert rep.keys() == report_totals(want, 50257, True).keys()
    assert all(np.array_equal(got[0][0][n], got[1][0][n]) for n in want)
