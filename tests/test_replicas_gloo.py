"""Replica plumbing across processes on CPU (gloo, world_size 2).

The packed tick has no data-path collective: each GPU runs its own replica and
requests are sharded round-robin. The process group only lines ranks up and
takes the maximum of their timings, which is what bench.py reports. These
tests run two CPU ranks with the same helpers bench.py uses.
"""

import os
import socket

import pytest
import torch.multiprocessing as mp

from helios_b200 import replicas


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, size: int, port: int, queue) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(size), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    try:
        assert replicas.init("gloo", timeout_s=30)
        r, n, local = replicas.world()
        requests = list(range(11))
        mine = replicas.shard(requests, r, n)
        replicas.barrier()
        slowest = replicas.max_over_ranks(1.0 + r)
        total = replicas.sum_over_ranks(float(len(mine)))
        gathered = replicas.gather_objects({"rank": r, "ttft": [0.1 * r, 0.2 * r]})
        assert gathered == [{"rank": k, "ttft": [0.1 * k, 0.2 * k]} for k in range(n)]
        queue.put((r, mine, slowest, total))
    finally:
        replicas.shutdown()


def test_two_rank_sharding_and_max_timing():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(rank, 2, port, queue)) for rank in range(2)]
    for p in procs:
        p.start()
    results = sorted(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    (r0, shard0, max0, tot0), (r1, shard1, max1, tot1) = results
    assert shard0 == [0, 2, 4, 6, 8, 10] and shard1 == [1, 3, 5, 7, 9]
    assert sorted(shard0 + shard1) == list(range(11))  # every request on exactly one replica
    assert max0 == max1 == 2.0
    assert tot0 == tot1 == 11.0


def test_single_process_needs_no_group():
    assert replicas.world()[1] == 1 or os.environ.get("WORLD_SIZE")
    assert not replicas.init("gloo") if "WORLD_SIZE" not in os.environ else True
    assert replicas.max_over_ranks(3.5) == 3.5
    assert replicas.gather_objects({"x": 1}) == [{"x": 1}]
    assert replicas.shard([1, 2, 3], 0, 1) == [1, 2, 3]
