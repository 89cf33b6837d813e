"""The data-parallel host logic of bench.py on CPU: two gloo ranks split a pool of sequences without overlap and
agree on the slowest rank's time."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import dp


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
        ids = list(dp.shard(2048, rank, world))
        t = dp.max_over_ranks(1.5 + rank, dist)
        q.put((rank, ids[0], ids[-1], len(ids), t, dp.rank_seed(1234, rank)))
    finally:
        dist.destroy_process_group()


def test_shard_covers_without_overlap():
    for n, w in [(2048, 8), (10, 3), (1, 2)]:
        got = [i for r in range(w) for i in dp.shard(n, r, w)]
        assert got == list(range(n))
    with pytest.raises(ValueError):
        dp.shard(4, 2, 2)


def test_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, a0, b0, n0, t0, s0), (r1, a1, b1, n1, t1, s1) = res
    assert (a0, b0, n0) == (0, 1023, 1024) and (a1, b1, n1) == (1024, 2047, 1024)
    assert t0 == t1 == 2.5  # the slowest rank's time
    assert s0 != s1
