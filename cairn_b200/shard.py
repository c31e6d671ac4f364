"""Multi-GPU forms of the hot path: one process per GPU, torch.distributed for the plumbing.

The reference is single-GPU (no collective anywhere in its runtime); the sharded forms follow the partition its
operations allow:
  row_block / sharded_gemm   the multiply split into contiguous row blocks of A and C, B replicated: every rank
                             computes its block with no exchange (rows are independent in mma_unordered's contract);
                             with gather=True, one NCCL all-gather then gives every rank the whole C (gather_rows),
                             the one collective the product's partition ever needs.
  range_of / sharded_saxpy   contiguous index ranges of a `parallel` region: no exchange.
  sharded_sum_f32            each rank reduces its range to a part (the double-double total and the special-value
                             flags, cairn_b200_sum_f32_partial); one all-gather of 24 bytes per rank; every rank
                             combines the parts in rank order and rounds once (on the device, or exactly on the host
                             with cairn_b200_sum_f32_combine), so the total is the host's exact sum of all terms.
  sharded_sum_u64            each rank's (wrapped total, overflow flag) is all-gathered and folded in rank order
                             with cr::Sum's rule (runtime/cairn_runtime.hpp:158-166): the flag is set exactly when
                             the whole sum does not fit.

Failure detection (the reference has none across devices; its device guards trap): a rank that leaves between steps
is found on the host. `Liveness` marks each rank's arrival at a step in the process group's store, and `require`
raises CairnError(ERR_TIMEOUT) naming the ranks that did not arrive within a deadline, before any collective or
kernel of the step is queued. A collective that a peer never joins ends with the process group's own timeout; the
sums' exchanges turn that error into the same CairnError, so no rank waits on a lost peer for ever.
"""

from __future__ import annotations

import ctypes as C
from datetime import timedelta

import torch
import torch.distributed as dist

from ._lib import ERR_OVERFLOW, ERR_SHAPE, ERR_TIMEOUT, CairnError, check, lib
from .ops import gemm, reduce_sum, saxpy


def range_of(n: int, world: int, rank: int) -> tuple[int, int]:
    """Rank `rank`'s contiguous share [lo, hi) of n indices: shares differ in length by at most one."""
    return n * rank // world, n * (rank + 1) // world


def row_block(m: int, world: int, rank: int) -> tuple[int, int]:
    """The rows of A and C rank `rank` owns in the row-block partition."""
    return range_of(m, world, rank)


def gather_rows(block: torch.Tensor, m: int, group=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Every rank's row block (row_block's partition of m rows, rank order) gathered into the whole m-row matrix on
    every rank, by one NCCL all-gather. When the blocks are equal (m divisible by the world size) they land straight
    in `out`; otherwise each block is padded to the largest, gathered, and the padding dropped. A peer that never
    joins ends the call with CairnError(ERR_TIMEOUT) after the process group's timeout."""
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    lo, hi = row_block(m, world, rank)
    if block.shape[0] != hi - lo:
        raise CairnError(ERR_SHAPE, f"gather_rows: rank {rank} holds {block.shape[0]} rows, its block is {hi - lo}")
    rest = tuple(block.shape[1:])
    if out is None:
        out = torch.empty((m, *rest), dtype=block.dtype, device=block.device)
    elif tuple(out.shape) != (m, *rest) or out.dtype != block.dtype or not out.is_contiguous():
        raise CairnError(ERR_SHAPE, "gather_rows: out is the whole contiguous matrix of the blocks' type")
    block = block.contiguous()
    if m % world == 0:
        _all_gather(out.view(-1), block.view(-1), group, "gather_rows")
        return out
    tall = -(-m // world)
    padded = torch.zeros((tall, *rest), dtype=block.dtype, device=block.device)
    padded[: hi - lo].copy_(block)
    flat = torch.empty((world * tall, *rest), dtype=block.dtype, device=block.device)
    _all_gather(flat.view(-1), padded.view(-1), group, "gather_rows")
    for r in range(world):
        r0, r1 = row_block(m, world, r)
        out[r0:r1].copy_(flat[r * tall: r * tall + (r1 - r0)])
    return out


def sharded_gemm(a_block: torch.Tensor, b: torch.Tensor, *, gather: bool = False, m: int | None = None, group=None,
                 **kw) -> torch.Tensor:
    """This rank's row block of op(A) * op(B), with no communication; with gather=True, the whole product on every
    rank (gather_rows over the m rows of A, m defaulting to the sum of the ranks' blocks at equal sizes)."""
    block = gemm(a_block, b, **kw)
    if not gather:
        return block
    if m is None:
        m = block.shape[0] * dist.get_world_size(group)
    return gather_rows(block, m, group)


def sharded_saxpy(a: float, x_local: torch.Tensor, y_local: torch.Tensor, out_local: torch.Tensor | None = None):
    return saxpy(a, x_local, y_local, out_local)


class Liveness:
    """Which ranks reached a step, kept in a torch.distributed store shared by the ranks (the process group's own,
    a TCPStore or a FileStore). Each rank marks a step as it begins it; `missing` lists the other ranks that have not
    marked it within a deadline, and `require` raises CairnError(ERR_TIMEOUT) naming them."""

    def __init__(self, store, rank: int, world: int, prefix: str = "cairn_b200/alive"):
        self.store, self.rank, self.world, self.prefix = store, rank, world, prefix

    def _key(self, step: int, rank: int) -> str:
        return f"{self.prefix}/{step}/{rank}"

    def mark(self, step: int) -> None:
        self.store.set(self._key(step, self.rank), "1")

    def missing(self, step: int, timeout_s: float) -> list[int]:
        others = [r for r in range(self.world) if r != self.rank]
        try:
            self.store.wait([self._key(step, r) for r in others], timedelta(seconds=timeout_s))
            return []
        except Exception:  # the store's timeout: find which ranks it was waiting for
            return [r for r in others if not self.store.check([self._key(step, r)])]

    def require(self, step: int, timeout_s: float) -> None:
        gone = self.missing(step, timeout_s)
        if gone:
            raise CairnError(ERR_TIMEOUT, f"step {step}: ranks {gone} did not arrive within {timeout_s} s")


def _all_gather(out: torch.Tensor, part: torch.Tensor, group, what: str) -> None:
    """dist.all_gather_into_tensor, with a lost peer (the process group's timeout, or a closed connection) reported
    as CairnError(ERR_TIMEOUT)."""
    try:
        dist.all_gather_into_tensor(out, part, group=group)
    except (RuntimeError, dist.DistError) as e:
        raise CairnError(ERR_TIMEOUT, f"{what}: a rank did not join the exchange ({type(e).__name__})") from e


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
    _all_gather(flat, part, group, "sharded_sum_f32")
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
    _all_gather(cells, cell, group, "sharded_sum_u64")
    _all_gather(flags, flag, group, "sharded_sum_u64")
    total, over = fold_u64([int(v) & (2**64 - 1) for v in cells.cpu().tolist()], flags.cpu().tolist())
    if over:
        raise CairnError(ERR_OVERFLOW, "sharded_sum_u64")
    return total
