"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU (no collective anywhere in its runtime); the sharded forms follow the partition its
operations allow:
  row_block / sharded_gemm   the multiply split into contiguous row blocks of A and C, B replicated: every rank
                             computes its block with no exchange (rows are independent in mma_unordered's contract).
  range_of / sharded_saxpy   contiguous index ranges of a `parallel` region: no exchange.
  sharded_sum_f32            each rank reduces its range to a part (the double-double total and the special-value
                             flags, cairn_b200_sum_f32_partial); one all-gather of 24 bytes per rank; every rank
                             combines the parts in rank order and rounds once (on the device, or exactly on the host
                             with cairn_b200_sum_f32_combine), so the total is the host's exact sum of all terms.
  sharded_sum_u64            each rank's (wrapped total, overflow flag) is all-gathered and folded in rank order
                             with cr::Sum's rule (runtime/cairn_runtime.hpp:158-166): the flag is set exactly when
                             the whole sum does not fit.
"""

from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from ._lib import ERR_OVERFLOW, CairnError, check, lib
from .ops import gemm, reduce_sum, saxpy


def range_of(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rank `rank`'s contiguous share [lo, hi) of n indices: shares differ in length by at most one."""
    return n * rank // world, n * (rank + 1) // world


def row_block(m: int, world: int, rank: int) -> tuple[int, int]:
    """The rows of A and C rank `rank` owns in the row-block partition."""
    return range_of(m, world, rank)


def sharded_gemm(a_block: torch.Tensor, b: torch.Tensor, **kw) -> torch.Tensor:
    """This rank's row block of op(A) * op(B): no communication."""
    return gemm(a_block, b, **kw)


def sharded_saxpy(a: float, x_local: torch.Tensor, y_local: torch.Tensor, out_local: torch.Tensor | None = None):
    return saxpy(a, x_local, y_local, out_local)


def combine_f32_parts(parts: torch.Tensor) -> float:
    """The correctly rounded total of every rank's part (a (world, 3) f64 tensor), added exactly on the host."""
    host = parts.detach().to("cpu", torch.float64).contiguous()
    result = C.c_float(0.0)
    check(lib().cairn_b200_sum_f32_combine(host.data_ptr(), host.shape[0], C.byref(result)), "combine_f32_parts")
    return result.value


def fold_u64(cells: list[int], flags: list[int]) -> tuple[int, bool]:
    """cr::Sum<u64> folded in rank order: the wrapped total and a flag set when any part overflowed or the fold
    wrapped."""
    total, over = 0, False
    for v, f in zip(cells, flags):
        s = (total + v) & (2**64 - 1)
        over = over or bool(f) or s < total
        total = s
    return total, over


def sharded_sum_f32(x_local: torch.Tensor, group=None) -> float:
    """`reduce + parallel` over the concatenation of every rank's x_local (rank order), the host's exact sum."""
    world = dist.get_world_size(group)
    part = torch.empty(3, dtype=torch.float64, device=x_local.device)
    reduce_sum(x_local, out=part)
    flat = torch.empty(world * 3, dtype=torch.float64, device=x_local.device)
    dist.all_gather_into_tensor(flat, part, group=group)
    parts = flat.view(world, 3)
    if parts.is_cuda:
        total = torch.empty(1, dtype=torch.float32, device=parts.device)
        check(lib().cairn_b200_sum_f32_combine_device(torch.cuda.current_stream(parts.device).cuda_stream,
                                                      parts.data_ptr(), world, total.data_ptr()), "sharded_sum_f32")
        return float(total.item())
    return combine_f32_parts(parts)


def sharded_sum_u64(x_local: torch.Tensor, group=None) -> int:
    """The checked u64 `reduce +` over every rank's x_local; raises CairnError where the reference traps."""
    world = dist.get_world_size(group)
    cell = torch.zeros(1, dtype=torch.int64, device=x_local.device)
    flag = torch.zeros(1, dtype=torch.int32, device=x_local.device)
    reduce_sum(x_local, out=cell.view(torch.uint64), overflow=flag)
    cells = torch.zeros(world, dtype=torch.int64, device=x_local.device)
    flags = torch.zeros(world, dtype=torch.int32, device=x_local.device)
    dist.all_gather_into_tensor(cells, cell, group=group)
    dist.all_gather_into_tensor(flags, flag, group=group)
    total, over = fold_u64([int(v) & (2**64 - 1) for v in cells.cpu().tolist()], flags.cpu().tolist())
    if over:
        raise CairnError(ERR_OVERFLOW, "sharded_sum_u64")
    return total
