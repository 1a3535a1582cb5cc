"""Data-parallel host logic on CPU: bucket planning, and the bucketed all-reduce driven by
leaf-ready events across two ``gloo`` ranks (world size 2, 127.0.0.1)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest


def test_plan_buckets_tiles_the_buffer():
    from tensorgrad_b200.distributed import plan_buckets

    sizes = [10, 3, 7, 20, 1, 5]
    offsets = [0, 12, 16, 24, 44, 48]  # 4-element aligned slots
    buckets = plan_buckets(sizes, offsets, 4, 48)  # 12 elements per bucket
    assert [m for _, _, m in buckets] == [[0, 1], [2, 3], [4, 5]]
    assert buckets[0][0] == 0 and buckets[-1][1] == 53
    for (_, stop, _), (start, _, _) in zip(buckets, buckets[1:]):
        assert stop == start


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, out: dict) -> None:
    import torch
    import torch.distributed as dist

    from tensorgrad_b200.distributed import BucketedAllReduce

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sizes = [6, 2, 9, 4, 4]
        offsets = [0, 8, 12, 24, 28]
        flat = torch.full((32,), float(rank + 1))
        ids = [100 + i for i in range(len(sizes))]
        red = BucketedAllReduce([(flat, ids, offsets, sizes)], bucket_bytes=40)
        for step in range(2):
            flat.fill_(float(rank + 1) * (step + 1))
            # The backward walk finalises the last parameters first.
            for pid in reversed(ids):
                red.ready(pid)
            red.finish()
            out[(rank, step)] = (flat.numpy().copy(), list(red.last_order))
    finally:
        dist.destroy_process_group()


def _worker(rank, world, port, queue):
    out: dict = {}
    _rank_main(rank, world, port, out)
    queue.put(out)


def test_bucketed_all_reduce_two_gloo_ranks():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results: dict = {}
    for _ in procs:
        results.update(queue.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for step in range(2):
        mean = 1.5 * (step + 1)  # ranks hold 1 and 2 (times step + 1): the average
        for rank in range(2):
            buf, order = results[(rank, step)]
            np.testing.assert_allclose(buf, mean)
            # Buckets complete from the end of the buffer; both ranks launch in one order.
            assert order == sorted(order, reverse=True)
        assert results[(0, step)][1] == results[(1, step)][1]


def test_unready_buckets_are_launched_by_finish_in_order():
    import torch

    from tensorgrad_b200.distributed import BucketedAllReduce

    flat = torch.ones(32)
    red = BucketedAllReduce([(flat, [1, 2, 3, 4], [0, 8, 16, 24], [8, 8, 8, 8])],
                            bucket_bytes=32)
    red.ready(4)          # bucket 3 complete
    red.ready(2)          # bucket 1 complete
    red.finish()          # 0 and 2 never got their gradients: launched in bucket order
    assert red.last_order == [3, 1, 0, 2]
    assert red.pending == red.members and not any(red.launched)


# ------------------------------------------------------------------ fault injection (host)
def _fault_rank(rank: int, world: int, port: int, fault: str, queue) -> None:
    """One gloo rank of a two-step exchange; rank 1's communicator injects ``fault`` into
    bucket 1 of step 1. Reports what each step did, then leaves without tearing the group
    down (after a failed collective the group cannot be trusted to shut down cleanly)."""
    import torch
    import torch.distributed as dist

    from tensorgrad_b200 import distributed
    from tensorgrad_b200.distributed import (
        BucketedAllReduce, CollectiveError, FaultyCommunicator, ProcessGroupCommunicator,
    )

    import datetime

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    # A short group timeout bounds every gloo operation, also the ones a fault leaves waiting.
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=5))
    comm = ProcessGroupCommunicator()
    if rank == 1 and fault != "leave":
        comm = FaultyCommunicator(comm, {(1, 1): fault}, delay_s=0.3)
    flat = torch.zeros(32)
    red = BucketedAllReduce([(flat, [1, 2, 3, 4], [0, 8, 16, 24], [8, 8, 8, 8])],
                            bucket_bytes=32, comm=comm, deadline_s=3.0, verify=True)
    report = []
    for step in range(2):
        flat.copy_(torch.arange(32, dtype=torch.float32) * (rank + 1) + step)
        if fault == "leave" and step == 1:
            if rank == 1:  # stops between steps, with nothing in flight
                distributed.leave_job()
                report.append(("left", None))
                break
            # Sequenced so that the announcement lands before this rank's next launch.
            dist.distributed_c10d._get_default_store().wait([distributed._LEFT.format(1)])
        try:
            red.finish()
            report.append(("ok", flat.numpy().copy()))
        except CollectiveError as exc:
            report.append((type(exc).__name__, None))
            break
    queue.put((rank, report))
    queue.close()
    queue.join_thread()  # the report is handed over before the hard exit
    os._exit(0)


def _run_fault(fault: str) -> dict:
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fault_rank, args=(r, 2, port, fault, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    return results


def test_dropped_bucket_times_out_on_every_rank():
    results = _run_fault("drop")
    expected_first = (np.arange(32) * 1.5).astype(np.float32)  # mean of ranks 1x and 2x
    for rank in (0, 1):
        first, second = results[rank]
        assert first[0] == "ok"
        np.testing.assert_allclose(first[1], expected_first)
        assert second[0] == "CollectiveTimeout"


def test_delayed_bucket_still_reduces_correctly():
    results = _run_fault("delay")
    for rank in (0, 1):
        assert [kind for kind, _ in results[rank]] == ["ok", "ok"]
        np.testing.assert_allclose(results[rank][1][1], np.arange(32) * 1.5 + 1.0)


def test_corrupted_bucket_is_caught_by_verification():
    results = _run_fault("corrupt")
    for rank in (0, 1):
        first, second = results[rank]
        assert first[0] == "ok"
        assert second[0] == "CollectiveMismatch"


def test_departed_rank_is_seen_before_the_next_launch():
    results = _run_fault("leave")
    assert [kind for kind, _ in results[1]] == ["ok", "left"]
    first, second = results[0]
    assert first[0] == "ok"
    np.testing.assert_allclose(first[1], (np.arange(32) * 1.5).astype(np.float32))
    assert second[0] == "CollectiveError"  # raised by the peer check, not a deadline
