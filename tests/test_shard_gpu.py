"""The sharded forms on 2 GPUs (one process per GPU, NCCL): the row-block GEMM against the single-GPU product and its
all-gather into the whole product, the range-sharded f32 sum against the oracle's exact sum of all terms (bit for
bit) and the u64 checked sum against n (n - 1) / 2; and a rank that leaves between steps, which the other rank's
Liveness names from the store before it queues anything of the next step. Skipped with fewer than 2 GPUs; NVLS is
off (NCCL_NVLS_ENABLE=0), every rank's collectives run in the same order, and a rank leaves only between steps, with
nothing of its own in flight."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _start(target, world: int, *args):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, *args, q)) for r in range(world)]
    for p in procs:
        p.start()
    return procs, q


def _finish(procs, q, timeout: float = 240):
    """Every rank's result, then every process joined; a process still alive after the timeout is terminated."""
    results = dict(q.get(timeout=timeout) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
            p.join(timeout=10)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    return results


def _init(rank: int, world: int, port: int, seconds: int):
    import datetime

    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    store = dist.TCPStore("127.0.0.1", port, world, is_master=rank == 0, timeout=datetime.timedelta(seconds=60))
    dist.init_process_group("nccl", store=store, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=seconds), device_id=dev)
    return dev, store


def _worker(rank: int, world: int, port: int, q):
    import torch.distributed as dist

    import cairn_b200
    from cairn_b200 import shard

    dev, _ = _init(rank, world, port, 60)
    try:
        rng = np.random.default_rng(5)
        n = 3_000_017
        x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-40, 40, n)).astype(np.float32)
        lo, hi = shard.range_of(n, world, rank)
        total = shard.sharded_sum_f32(torch.from_numpy(x[lo:hi]).to(dev))
        u = torch.arange(*shard.range_of(1 << 24, world, rank), device=dev, dtype=torch.int64).view(torch.uint64)
        usum = shard.sharded_sum_u64(u)
        m, k, nn = 1024, 512, 768
        g = torch.Generator(device=dev).manual_seed(0)
        a = torch.randn(m, k, device=dev, generator=g).bfloat16()
        b = torch.randn(k, nn, device=dev, generator=g).bfloat16()
        r0, r1 = shard.row_block(m, world, rank)
        block = shard.sharded_gemm(a[r0:r1].contiguous(), b)
        whole = cairn_b200.gemm(a, b)
        gathered = shard.sharded_gemm(a[r0:r1].contiguous(), b, gather=True, m=m)
        m2 = 1001  # uneven blocks: padded, gathered, the padding dropped
        q0, q1 = shard.row_block(m2, world, rank)
        whole2 = cairn_b200.gemm(a[:m2].contiguous(), b)
        gathered2 = shard.sharded_gemm(a[q0:q1].contiguous(), b, gather=True, m=m2)
        cairn_b200.stream_status()
        q.put((rank, (total, usum, bool(torch.equal(block, whole[r0:r1])), bool(torch.equal(gathered, whole)),
                      bool(torch.equal(gathered2, whole2)))))
    finally:
        dist.destroy_process_group()


def test_two_ranks_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from oracle import restated

    procs, q = _start(_worker, 2, 29700 + os.getpid() % 500)
    results = _finish(procs, q)
    rng = np.random.default_rng(5)
    n = 3_000_017
    x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-40, 40, n)).astype(np.float32)
    want = restated.sum_f32(x).view(np.uint32)
    for rank, (total, usum, same, gathered, gathered_uneven) in results.items():
        assert np.float32(total).view(np.uint32) == want, rank
        assert usum == (1 << 24) * ((1 << 24) - 1) // 2
        assert same, "a row block differs from the same rows of the whole product"
        assert gathered and gathered_uneven, "the gathered product differs from the whole product"


def _leaving_worker(rank: int, world: int, port: int, q):
    import time

    import torch.distributed as dist

    from cairn_b200 import CairnError, shard

    dev, store = _init(rank, world, port, 20)
    live = shard.Liveness(store, rank, world)
    events = []
    try:
        x = torch.ones(1 << 20, device=dev)
        for step in range(3):
            if rank == 1 and step == 1:
                torch.cuda.synchronize()  # nothing of this rank's in flight: it leaves between steps
                break
            live.mark(step)
            t0 = time.perf_counter()
            try:
                live.require(step, timeout_s=3.0)
            except CairnError as e:
                events.append(("missing", step, e.status, str(e), time.perf_counter() - t0))
                break
            events.append(("sum", step, shard.sharded_sum_f32(x)))
        torch.cuda.synchronize()
        q.put((rank, events))
    finally:
        dist.destroy_process_group()


def test_a_rank_that_leaves_between_steps_is_named_on_the_host_before_the_next_launch():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from cairn_b200._lib import ERR_TIMEOUT

    procs, q = _start(_leaving_worker, 2, 29200 + os.getpid() % 500)
    results = _finish(procs, q, timeout=180)
    assert results[1] == [("sum", 0, float(2 << 20))]
    first, second = results[0]
    assert first == ("sum", 0, float(2 << 20))
    kind, step, status, message, waited = second
    assert (kind, step, status) == ("missing", 1, ERR_TIMEOUT)
    assert "[1]" in message and waited < 20
