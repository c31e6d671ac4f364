"""The sharded forms on 2 GPUs (one process per GPU, NCCL): the row-block GEMM against the single-GPU product, the
range-sharded f32 sum against the oracle's exact sum of all terms (bit for bit) and the u64 checked sum against
n (n - 1) / 2. Skipped with fewer than 2 GPUs; NVLS is off (NCCL_NVLS_ENABLE=0) and every rank's collectives run
in the same order."""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _worker(rank: int, world: int, port: int, q):
    import datetime

    import torch.distributed as dist

    import cairn_b200
    from cairn_b200 import shard

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
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
        cairn_b200.stream_status()
        same = bool(torch.equal(block, whole[r0:r1]))
        q.put((rank, total, usum, same))
    finally:
        dist.destroy_process_group()


def test_two_ranks_on_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp

    from oracle import restated

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29700 + os.getpid() % 500
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [q.get(timeout=5) for _ in procs]
    rng = np.random.default_rng(5)
    n = 3_000_017
    x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-40, 40, n)).astype(np.float32)
    want = restated.sum_f32(x).view(np.uint32)
    for rank, total, usum, same in results:
        assert np.float32(total).view(np.uint32) == want, rank
        assert usum == (1 << 24) * ((1 << 24) - 1) // 2
        assert same, "a row block differs from the same rows of the whole product"
