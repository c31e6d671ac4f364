"""The multi-GPU host logic at world size 2 on CPU (gloo): the range and row-block partitions, the exact combination
of ranks' f32 sum parts through an all-gather and the library's host combine, and the rank-order fold of u64 parts
with its overflow rule. Each rank's part is formed here exactly from its terms (the device forms it on a GPU); the
combined total must equal the oracle's exact sum of all terms, bit for bit. The row all-gather (gather_rows) of
even and uneven row blocks gives every rank the whole matrix."""

from __future__ import annotations

import os
from fractions import Fraction

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cairn_b200 import shard


def _exact_part(x: np.ndarray) -> list[float]:
    """(hi, lo, flags) for finite terms: hi + lo is the exact total when it fits a double-double."""
    total = sum((Fraction(float(t)) for t in x), Fraction(0))
    hi = float(total)
    lo = float(total - Fraction(hi))
    flags = 16.0 + (8.0 if any(np.asarray([t], np.float32).view(np.uint32)[0] != 0x80000000 for t in x) else 0.0)
    return [hi, lo, flags]


def _worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(7)
        n = 20_003
        x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-30, 30, n)).astype(np.float32)
        lo, hi = shard.range_of(n, world, rank)
        part = torch.tensor(_exact_part(x[lo:hi]), dtype=torch.float64)
        flat = torch.empty(world * 3, dtype=torch.float64)
        dist.all_gather_into_tensor(flat, part)
        total = shard.combine_f32_parts(flat.view(world, 3))
        u = np.arange(1_000_000, dtype=np.uint64)
        ulo, uhi = shard.range_of(u.size, world, rank)
        cell = torch.tensor([int(u[ulo:uhi].sum())], dtype=torch.int64)
        cells = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(cells, cell)
        folded = shard.fold_u64([int(c.item()) for c in cells], [0] * world)
        q.put((rank, float(total), folded))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_combine_to_the_exact_whole():
    from oracle import restated

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [q.get(timeout=5) for _ in procs]
    rng = np.random.default_rng(7)
    n = 20_003
    x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-30, 30, n)).astype(np.float32)
    want = float(restated.sum_f32(x))
    for rank, total, folded in results:
        assert np.float32(total).view(np.uint32) == np.float32(want).view(np.uint32), rank
        assert folded == (499_999_500_000, False)


@pytest.mark.parametrize("n,world", [(0, 2), (1, 2), (7, 3), (1 << 30, 8), (65536, 8)])
def test_partitions_cover_every_index_once(n, world):
    bounds = [shard.range_of(n, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == n
    assert all(bounds[r][1] == bounds[r + 1][0] for r in range(world - 1))
    sizes = [h - lo for lo, h in bounds]
    assert max(sizes) - min(sizes) <= 1
    assert shard.row_block(65536, 8, 3) == (24576, 32768)


def test_the_u64_fold_flags_exactly_the_totals_that_do_not_fit():
    top = 2**64 - 1
    assert shard.fold_u64([top, 0], [0, 0]) == (top, False)
    assert shard.fold_u64([top, 1], [0, 0]) == (0, True)
    assert shard.fold_u64([5, 6], [1, 0]) == (11, True)  # a rank's own part overflowed
    assert shard.fold_u64([2**63, 2**63 - 1], [0, 0]) == (top, False)


def test_an_empty_rank_keeps_the_sign_of_an_all_negative_zero_sum():
    parts = torch.tensor([[-0.0, -0.0, 16.0], [0.0, 0.0, 0.0]], dtype=torch.float64)  # rank 1 has no terms
    assert np.float32(shard.combine_f32_parts(parts)).view(np.uint32) == 0x80000000
    parts = torch.tensor([[0.0, 0.0, 0.0], [0.0, 0.0, 0.0]], dtype=torch.float64)  # no terms anywhere
    assert np.float32(shard.combine_f32_parts(parts)).view(np.uint32) == 0
    parts = torch.tensor([[1.0, 0.0, 24.0], [float("inf"), 0.0, 26.0]], dtype=torch.float64)
    assert shard.combine_f32_parts(parts) == float("inf")


def _gather_worker(rank: int, world: int, port: int, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = []
        for m in (12, 13, 2):  # equal blocks, then blocks of 5, 4, 4 rows, then an empty block
            whole = torch.arange(m * 5, dtype=torch.float32).view(m, 5) * 1.5 - 7
            lo, hi = shard.row_block(m, world, rank)
            got.append(bool(torch.equal(shard.gather_rows(whole[lo:hi].clone(), m), whole)))
        q.put((rank, got))
    finally:
        dist.destroy_process_group()


def test_row_blocks_gather_into_the_whole_matrix_on_every_rank():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 28500 + os.getpid() % 1000
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.terminate()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert results == {r: [True, True, True] for r in range(3)}
