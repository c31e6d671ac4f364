"""The device watchdog on the B200: every wait in this library's kernels is bounded, records a fault word and returns,
so a wait whose partner never comes ends with an error status and a usable context (the reference's device guards
trap instead, runtime/cairn_kernels.hpp:33-59). The self-test makes such a wait run out on purpose, on a
shared-memory barrier that nothing completes; no fault, trap or hang is involved. Afterwards the same stream still
computes a multiply and a sum that agree with the oracle."""

from __future__ import annotations

import time

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu


def test_watchdog_wait_gives_up_reports_and_leaves_the_context_usable(cuda):
    cairn_b200.stream_status()
    t0 = time.perf_counter()
    cairn_b200.watchdog_selftest()
    waited = time.perf_counter() - t0
    assert 1.9 <= waited < 30, waited  # the bound is 2 s of the device's global timer
    cairn_b200.stream_status()  # the fault was read and cleared

    m, n, k = 256, 512, 128
    c, a, b = inputs.mma_case("bf16", m, n, k, seed=3)
    ct = torch.from_numpy(c.copy()).to(cuda)
    at = torch.from_numpy(a.view(np.int16).copy()).to(cuda).view(torch.bfloat16)
    bt = torch.from_numpy(b.view(np.int16).copy()).to(cuda).view(torch.bfloat16)
    cairn_b200.mma_unordered(m, n, k, ct, at, bt)
    cairn_b200.stream_status()
    av = np.abs(inputs.decode("bf16", a).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", b).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(c.reshape(m, n)) + av @ bv)
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - restated.mma("bf16", c, a, b, m, n, k).reshape(m, n)) <= tol).all()
    x = np.random.default_rng(9).uniform(-1, 1, 100_003).astype(np.float32)
    got = np.float32(cairn_b200.reduce_sum(torch.from_numpy(x).to(cuda)))
    assert got.view(np.uint32) == restated.sum_f32(x).view(np.uint32)
