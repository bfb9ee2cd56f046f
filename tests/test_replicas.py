"""Host-side multi-GPU plumbing: request dispatch and max-over-ranks timing,
exercised with two gloo ranks on the CPU."""

from __future__ import annotations

import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from asrback_b200.replicas import ReplicaDispatcher, max_over_ranks


def test_dispatcher_balances_by_outstanding_work():
    d = ReplicaDispatcher(3)
    assert [d.assign(10) for _ in range(3)] == [0, 1, 2]
    assert d.assign(1) == 0  # all at 10: lowest index
    d.complete(1, 10)
    assert d.assign(5) == 1  # replica 1 is now empty
    assert d.load(0) == 11 and d.load(1) == 5 and d.load(2) == 10


def test_dispatcher_rejects_bad_bookkeeping():
    d = ReplicaDispatcher(2)
    with pytest.raises(ValueError):
        d.complete(0, 1.0)
    with pytest.raises(ValueError):
        ReplicaDispatcher(0)
    with pytest.raises(ValueError):
        d.assign(-1)


def test_dispatcher_many_threads():
    import threading

    d = ReplicaDispatcher(4)
    assigned = []

    def work():
        for _ in range(250):
            r = d.assign(1.0)
            assigned.append(r)
            d.complete(r, 1.0)

    threads = [threading.Thread(target=work) for _ in range(8)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert len(assigned) == 2000
    assert all(d.load(r) == 0.0 for r in range(4))


def test_max_over_ranks_without_a_group_is_identity():
    assert max_over_ranks(3.5) == 3.5


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, results) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # Each rank "measured" its own device time; the job is as slow as the slowest.
        results[rank] = max_over_ranks(10.0 + 5.0 * rank)
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_with_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert dict(results) == {0: 15.0, 1: 15.0}
