"""Failure detection across ranks, on CPU (gloo, world size 2): a rank that leaves between steps is found on the host,
and an exchange that a rank never joins ends with an error instead of a wait for ever. The failures are made on the
host (a rank that returns early); nothing here touches a GPU.

  * Leaves before marking step 1: the other rank's Liveness.require(1) names it within the deadline, before any
    exchange of step 1 is queued.
  * Marks step 1, then leaves without joining its exchange: the other rank's all-gather fails (the peer's connection
    closes, or the process group's 5 s timeout runs out) and the sums' exchange reports CairnError(ERR_TIMEOUT).
"""

from __future__ import annotations

import os
import time
from datetime import timedelta

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cairn_b200 import CairnError, shard
from cairn_b200._lib import ERR_TIMEOUT


def _worker(rank: int, world: int, port: int, q, mode: str):
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=timedelta(seconds=30))
    dist.init_process_group("gloo", store=store, rank=rank, world_size=world, timeout=timedelta(seconds=5))
    live = shard.Liveness(store, rank, world)
    events = []
    try:
        for step in range(3):
            if rank == 1 and step == 1 and mode == "leave":
                break  # leaves between steps: nothing of step 1 was marked or queued
            live.mark(step)
            if rank == 1 and step == 1 and mode == "skip_exchange":
                break  # arrived at step 1, then leaves without joining its exchange
            t0 = time.perf_counter()
            try:
                live.require(step, timeout_s=3.0)
                part = torch.tensor([float(rank + 1), 0.0, 24.0], dtype=torch.float64)  # (hi, lo, flags)
                flat = torch.empty(world * 3, dtype=torch.float64)
                shard._all_gather(flat, part, None, "exchange")
                events.append(("sum", step, shard.combine_f32_parts(flat.view(world, 3))))
            except CairnError as e:
                events.append(("error", step, e.status, str(e), time.perf_counter() - t0))
                break
        q.put((rank, events))
    finally:
        dist.destroy_process_group()


def _run(mode: str):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + (os.getpid() + len(mode)) % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, mode)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return results


def test_a_rank_that_leaves_between_steps_is_named_before_the_next_exchange():
    results = _run("leave")
    assert results[1] == [("sum", 0, 3.0)]
    first, second = results[0]
    assert first == ("sum", 0, 3.0)
    kind, step, status, message, waited = second
    assert (kind, step, status) == ("error", 1, ERR_TIMEOUT)
    assert "[1]" in message and waited < 20


def test_an_exchange_a_rank_never_joins_ends_with_an_error():
    results = _run("skip_exchange")
    assert results[1] == [("sum", 0, 3.0)]
    first, second = results[0]
    assert first == ("sum", 0, 3.0)
    kind, step, status, message, waited = second
    assert (kind, step, status) == ("error", 1, ERR_TIMEOUT)
    assert "did not join the exchange" in message and waited < 30
