"""cairn_b200_sum_f32_noalloc, the f32 sum for callers that cannot allocate device memory (a process whose device
memory is reserved up front by its own allocator, or a loop that cannot afford a cudaMalloc's implicit
synchronization), against the ordinary allocating entry, cairn_b200_sum_f32, through the C ABI.

Both entries run the same kernel, so the tolerance is the one the other sum tests use: the same bits. Two calls in
a row on different inputs show that the shared static scratch is reset between calls (its ticket) and fully
rewritten (its partials). A child process calls the entry before anything else of the library has run, and checks
that a call leaves the device's free memory as it found it, that n = 0 gives +0.0, and that the totals are the
oracle's exact sums rounded once. This file sorts last so that a run stopping at its first failure has run every
other test first; it passes alone in a fresh process as well.
"""

from __future__ import annotations

import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

import cairn_b200

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


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
    # an output inside the input: the same status from either entry, so one can stand in for the other
    for name in ("cairn_b200_sum_f32_noalloc", "cairn_b200_sum_f32"):
        assert getattr(lib, name)(None, 16, x.data_ptr(), x.data_ptr() + 8) == cairn_b200._lib.ERR_OVERLAP, name


_FIRST_CALL = textwrap.dedent(
    """
    import sys
    sys.path[:0] = [{root!r}, {tests!r}]
    import numpy as np
    import torch
    import cairn_b200
    from oracle import restated

    torch.cuda.set_device(0)
    lib = cairn_b200.lib()
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(7)
    xs = [(rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-30, 30, n)).astype(np.float32) for n in (1_000_003, 65_537)]
    dev = [torch.from_numpy(x).cuda() for x in xs]
    out = torch.full((1,), 5.0, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()

    # the library's first call in this process: n = 0 gives +0.0 without touching the scratch
    assert lib.cairn_b200_sum_f32_noalloc(stream, 0, None, out.data_ptr()) == 0
    assert lib.cairn_b200_stream_status(stream) == 0
    assert int(out.cpu().numpy().view(np.uint32)[0]) == 0, out.item()

    for call, (x, d) in enumerate(zip(xs, dev)):
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        assert lib.cairn_b200_sum_f32_noalloc(stream, x.size, d.data_ptr(), out.data_ptr()) == 0
        assert lib.cairn_b200_stream_status(stream) == 0
        free_after = torch.cuda.mem_get_info()[0]
        if call:  # the first launch may still load the library's module; from then on nothing is allocated
            assert free_after == free_before, (free_before, free_after)
        got = int(out.cpu().numpy().view(np.uint32)[0])
        want = int(restated.sum_f32(x).view(np.uint32))
        assert got == want, (call, got, want)
    print("noalloc first-call ok")
    """
)


def test_the_allocation_free_sum_as_the_first_call_of_a_fresh_process(cuda):
    code = _FIRST_CALL.format(root=str(ROOT), tests=str(ROOT / "tests"))
    done = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300)
    assert done.returncode == 0, done.stdout[-2000:] + done.stderr[-4000:]
    assert "noalloc first-call ok" in done.stdout
