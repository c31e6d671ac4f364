"""BASELINE configs 5 and 3 at their full sizes on one B200, checked where a check at that size is affordable.

Config 5 (bf16 GEMM M = 65536, N = K = 8192, f32 out; one GPU computing the whole product, the M-sharded form's
single-rank case): sampled rows against the oracle's host multiply (the order of cr::tensor::reference,
runtime/cairn_tensor.hpp:28-41), every element within twice the contract bound (k + 1) 2^-22 sum |a b|
(docs/numerics.md, "The tensor-core multiply") and the north star's 2e-2 relative Frobenius tolerance.

Config 3 (the MLP step: batch 8192, 4096 -> 16384 -> 4096, bf16 weights ~ N(0, 0.02)): each of the six products on
sampled rows (or, for the weight gradients, sampled columns) against f64 sums of the very bf16 operands the device
read, within twice the contract bound (f32 outputs) or one bf16 rounding more (bf16 outputs); the loss gradient dY
bit for bit from the device's Y; the ReLU gradient exactly zero wherever H is not positive. The sampled sums run on
the GPU in f64 (a reference for floating-point products, as the north star's tolerances are stated against).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from cairn_b200 import mlp
from oracle import restated

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16).ravel()


def _contract(k: int, mag: torch.Tensor) -> torch.Tensor:
    return 2 * (k + 1) * 2.0**-22 * mag


def test_baseline_config_5_whole_product_on_sampled_rows(cuda):
    m, n, k = 65536, 8192, 8192
    g = torch.Generator(device=cuda).manual_seed(0)
    a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
    b = (torch.randn(k, n, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    out = cairn_b200.gemm(a, b)
    cairn_b200.stream_status()
    b_bits = _bits(b)
    b_abs = np.abs(inputs.decode("bf16", b_bits).astype(np.float32)).reshape(k, n)
    for r in (0, 255, 256, 32767, 65535):
        a_row = _bits(a[r])
        want = restated.mma_bf16_rows(a_row, b_bits, 1, n, k, 0, 1).astype(np.float64)
        got = out[r].cpu().numpy().astype(np.float64)
        mag = np.abs(inputs.decode("bf16", a_row).astype(np.float32)) @ b_abs
        tol = 2 * (k + 1) * 2.0**-22 * mag.astype(np.float64)
        bad = np.flatnonzero(np.abs(got - want) > tol)
        assert bad.size == 0, (r, bad[:4], got[bad[:4]], want[bad[:4]])
        assert np.linalg.norm(got - want) <= 2e-2 * np.linalg.norm(want), r


def test_baseline_config_3_full_step_on_sampled_rows_and_columns(cuda):
    B, D, Hd, O = 8192, 4096, 16384, 4096
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(B, D, device=cuda, generator=g).to(torch.bfloat16)
    w1 = (torch.randn(D, Hd, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    w2 = (torch.randn(Hd, O, device=cuda, generator=g) * 0.02).to(torch.bfloat16)
    t = torch.randn(B, O, device=cuda, generator=g)
    ws = mlp.mlp_step(x, w1, w2, t)
    cairn_b200.stream_status()
    rows, cols = [0, 1, 4095, 8191], [0, 777, 4095]
    f64 = lambda v: v.double()  # noqa: E731

    def check_f32(got: torch.Tensor, a: torch.Tensor, b: torch.Tensor, k: int, what: str):
        want = f64(a) @ f64(b)
        tol = _contract(k, f64(a).abs() @ f64(b).abs())
        err = (f64(got) - want).abs()
        assert bool((err <= tol).all()), (what, float((err - tol).max()))

    def check_bf16(got: torch.Tensor, a: torch.Tensor, b: torch.Tensor, k: int, what: str, relu: bool = False):
        want = f64(a) @ f64(b)
        if relu:
            want = want.clamp_min(0.0)
        tol = _contract(k, f64(a).abs() @ f64(b).abs()) + 2.0**-7 * f64(got).abs()
        err = (f64(got) - want).abs()
        assert bool((err <= tol).all()), (what, float((err - tol).max()))

    # forward: H = bf16(relu(X W1)), Y = H W2 (the device's own bf16 H as the second product's operand)
    check_bf16(ws.h[rows], x[rows], w1, D, "H", relu=True)
    check_f32(ws.y[rows], ws.h[rows], w2, Hd, "Y")
    # the loss gradient, bit for bit from the device's Y: dY = bf16(f32(Y - T) * f32(2 / n))
    n = B * O
    d = (ws.y.cpu().numpy() - t.cpu().numpy()).ravel()
    want_dy = inputs.encode("bf16", (d * (np.float32(2.0) / np.float32(n))).astype(np.float32))
    assert np.array_equal(_bits(ws.dy), want_dy)
    loss = np.float32(np.sum(d.astype(np.float64) ** 2) / n)
    assert abs(int(np.float32(ws.loss.item()).view(np.int32)) - int(loss.view(np.int32))) <= 1
    del d
    # backward: dW2 = H^T dY (columns), dH = bf16(dY W2^T) where H > 0 (rows), dW1 = X^T dH, dX = dH W1^T
    check_f32(ws.dw2[:, cols], ws.h.t(), ws.dy[:, cols], B, "dW2")
    dh_rows = ws.dh[rows]
    positive = f64(ws.h[rows]) > 0
    assert bool((f64(dh_rows)[~positive] == 0).all()), "dH outside the ReLU's support"
    want = f64(ws.dy[rows]) @ f64(w2).t()
    tol = _contract(O, f64(ws.dy[rows]).abs() @ f64(w2).abs().t()) + 2.0**-7 * f64(dh_rows).abs()
    err = (f64(dh_rows) - want).abs()[positive]
    assert bool((err <= tol[positive]).all()), ("dH", float((err - tol[positive]).max()))
    check_f32(ws.dw1[:, cols], x.t(), ws.dh[:, cols], B, "dW1")
    check_f32(ws.dx[rows], ws.dh[rows], w1.t(), Hd, "dX")
