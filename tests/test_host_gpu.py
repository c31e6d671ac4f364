"""cairn_b200.HostGemm: the multiply from pinned host memory to pinned host memory, copies and products overlapped
in row chunks over three streams and two sets of device buffers. Each result is held to the multiply's contract
against the CPU oracle (tests/soundness/test_tensor.py:182-226: within twice (k + 1) * 2^-22 * sum |a * b|, and one
bf16 rounding for a bf16 output), including calls queued back to back before any result is read."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu


def _case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    return a, b, bias


def _host(bits: np.ndarray, shape) -> torch.Tensor:
    return torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).view(shape).pin_memory()


def _bound(a, b, m, n, k):
    av = np.abs(inputs.decode("bf16", a).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", b).reshape(k, n))
    return 2 * (k + 1) * 2.0**-22 * (av @ bv)


def test_calls_in_flight_each_match_the_oracle(cuda):
    m, n, k = 1000, 768, 520  # row chunks of 125, ragged against the pair kernel's 256-row tiles
    hg = cairn_b200.HostGemm(m, n, k, out_dtype=torch.float32, device=cuda, chunks=8, depth=2)  # many ragged chunks
    cases = [_case(m, n, k, seed) for seed in range(3)]
    outs = [torch.empty((m, n), dtype=torch.float32).pin_memory() for _ in cases]
    b_h = _host(cases[0][1], (k, n))
    events = [hg.submit(_host(a, (m, k)), b_h, out) for (a, _, _), out in zip(cases, outs)]
    for e in events:
        e.synchronize()
    cairn_b200.stream_status()
    for (a, _, _), out in zip(cases, outs):
        want = restated.mma("bf16", np.zeros(m * n, np.float32), a, cases[0][1], m, n, k).reshape(m, n)
        assert (np.abs(out.numpy() - want) <= _bound(a, cases[0][1], m, n, k)).all()


def test_resident_weights_give_the_same_bits_as_weights_from_host(cuda):
    """B and the bias as device tensors kept from call to call (a layer's weights): only A crosses in, and each
    result equals, bit for bit, the same call with B and the bias copied in from host memory."""
    m, n, k = 768, 512, 384
    hg = cairn_b200.HostGemm(m, n, k, bias=True, device=cuda, chunks=2, depth=2)
    cases = [_case(m, n, k, seed) for seed in (11, 12)]
    b_bits, bias = cases[0][1], cases[0][2]
    b_dev = _host(b_bits, (k, n)).to(cuda)
    bias_dev = torch.from_numpy(bias).to(cuda)
    for a, _, _ in cases:
        resident = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
        copied = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
        hg.submit(_host(a, (m, k)), b_dev, resident, bias_dev, relu=True).synchronize()
        hg.submit(_host(a, (m, k)), _host(b_bits, (k, n)), copied, torch.from_numpy(bias).pin_memory(),
                  relu=True).synchronize()
        assert torch.equal(resident.view(torch.int16), copied.view(torch.int16))
    cairn_b200.stream_status()
    with pytest.raises(cairn_b200.CairnError):  # a B of the wrong shape, resident or not
        hg.submit(_host(cases[0][0], (m, k)), b_dev[:-1], resident, bias_dev)


def test_bias_relu_bf16_from_host(cuda):
    m, n, k = 512, 1024, 256
    a, b, bias = _case(m, n, k, 7)
    hg = cairn_b200.HostGemm(m, n, k, bias=True, device=cuda)
    out = torch.empty((m, n), dtype=torch.bfloat16).pin_memory()
    hg.submit(_host(a, (m, k)), _host(b, (k, n)), out, torch.from_numpy(bias).pin_memory(), relu=True).synchronize()
    cairn_b200.stream_status()
    acc = restated.mma("bf16", np.zeros(m * n, np.float32), a, b, m, n, k)
    want = inputs.decode("bf16", restated.bias_act(acc, bias, True, m, n)).reshape(m, n)
    got = out.float().numpy()
    # one bf16 ulp (2^-7 of the larger) where the f32 accumulators round differently, plus the contract bound
    assert (np.abs(got - want) <= 2.0**-7 * np.maximum(np.abs(got), np.abs(want)) + 2 * _bound(a, b, m, n, k)).all()
    assert (got >= 0).all()


def test_transposed_a_from_host(cuda):
    m, n, k = 384, 520, 264
    a, b, _ = _case(m, n, k, 9)
    at = np.ascontiguousarray(a.reshape(m, k).T)
    hg = cairn_b200.HostGemm(m, n, k, trans_a=True, out_dtype=torch.float32, device=cuda)
    out = torch.empty((m, n), dtype=torch.float32).pin_memory()
    hg.submit(_host(at, (k, m)), _host(b, (k, n)), out).synchronize()
    cairn_b200.stream_status()
    want = inputs.decode("bf16", a).reshape(m, k) @ inputs.decode("bf16", b).reshape(k, n)
    assert (np.abs(out.numpy() - want) <= _bound(a, b, m, n, k)).all()


def test_wrong_host_tensors_are_refused(cuda):
    hg = cairn_b200.HostGemm(64, 64, 64, device=cuda)
    good = torch.empty((64, 64), dtype=torch.bfloat16)
    with pytest.raises(cairn_b200.CairnError):
        hg.submit(good, good, torch.empty((64, 63), dtype=torch.bfloat16))
    with pytest.raises(cairn_b200.CairnError):
        hg.submit(good, good, good, torch.zeros(64))  # no bias was declared


def test_host_saxpy_bit_for_bit_with_calls_in_flight(cuda):
    n = 1_000_003
    hs = cairn_b200.HostSaxpy(n, device=cuda, chunks=4, depth=2)
    cases = [inputs.saxpy_case(n, seed=s) for s in range(3)]
    outs = [torch.empty(n, dtype=torch.float32).pin_memory() for _ in cases]
    events = [hs.submit(float(a), torch.from_numpy(x).pin_memory(), torch.from_numpy(y).pin_memory(), o)
              for (x, y, a), o in zip(cases, outs)]
    for e in events:
        e.synchronize()
    cairn_b200.stream_status()
    for (x, y, a), o in zip(cases, outs):
        assert np.array_equal(o.numpy().view(np.uint32), restated.saxpy(float(a), x, y).view(np.uint32))
