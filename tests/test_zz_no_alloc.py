"""cairn_b200_sum_f32_noalloc, the f32 sum for callers that cannot allocate device memory (a process whose device
memory is reserved up front by its own allocator, or a loop that cannot afford a cudaMalloc's implicit
synchronization), against the ordinary allocating entry, cairn_b200_sum_f32, through the C ABI.

Both entries run the same kernel, so the tolerance is the one the other sum tests use: the same bits. Two calls in
a row on different inputs show that the shared static scratch is reset between calls (its ticket) and fully
rewritten (its partials). This file sorts last so that a run stopping at its first failure has run every other
test first; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cairn_b200

pytestmark = pytest.mark.gpu


def _bits(t: torch.Tensor) -> int:
    return int(t.cpu().numpy().view(np.uint32)[0])


def test_the_allocation_free_sum_matches_the_allocating_entry_twice_in_a_row(cuda):
    lib = cairn_b200.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    rng = np.random.default_rng(2024)
    for call, n in enumerate((3_000_001, 777_777)):
        x_np = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-40, 40, n)).astype(np.float32)
        x = torch.from_numpy(x_np).to(cuda)
        want = torch.empty(1, dtype=torch.float32, device=cuda)
        got = torch.empty(1, dtype=torch.float32, device=cuda)
        assert lib.cairn_b200_sum_f32(stream, n, x.data_ptr(), want.data_ptr()) == 0
        assert lib.cairn_b200_sum_f32_noalloc(stream, n, x.data_ptr(), got.data_ptr()) == 0
        assert lib.cairn_b200_stream_status(stream) == 0
        assert _bits(got) == _bits(want), (call, got.item(), want.item())


def test_the_allocation_free_sum_refuses_bad_views_before_touching_the_device(cuda):
    lib = cairn_b200.lib()
    x = torch.zeros(16, dtype=torch.float32, device=cuda)
    assert lib.cairn_b200_sum_f32_noalloc(None, 16, x.data_ptr(), None) == cairn_b200._lib.ERR_VIEW
    assert lib.cairn_b200_sum_f32_noalloc(None, 16, x.data_ptr(), x.data_ptr() + 8) == cairn_b200._lib.ERR_OVERLAP
