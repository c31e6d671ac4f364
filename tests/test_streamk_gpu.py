"""The pair multiply's stream-K split on the B200, through the C ABI.

When a product has few 256 x 256 G tiles (at most half the resident pairs) and a long k loop, the pair kernel
spreads the k-blocks of all tiles evenly over more pairs, at least 32 k-blocks each. A pair holding part of a tile's
k-blocks leaves its raw f32 sum in a workspace slot; after a grid barrier every epilogue warp of the grid takes 32 x
32 blocks of the split tiles, adds their parts in pair order and runs the epilogue. These shapes are in that regime
(about 74 resident pairs on a B200; up to 32 pairs share one tile) and hold the split tiles to the multiply's
contract (tests/soundness/test_tensor.py:182-226): every output within twice (k + 1) * 2^-22 * (|c| + sum |a * b|) of
the exact sum, here computed in f64 from the decoded operands. The parts are added in one fixed order, so two runs
give the same bits.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import cairn_b200
import inputs

pytestmark = pytest.mark.gpu
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f8e4m3": torch.float8_e4m3fn, "f8e5m2": torch.float8_e5m2}

# (m, n, k): G = 2 tiles (n >= 512) and G = 1 tiles (256 <= n < 512), ragged in every direction; the last is one
# tile over 32 pairs.
SPLIT_SHAPES = [(512, 1024, 8192), (300, 700, 9000), (1000, 300, 6000), (256, 256, 65536)]


def operands(fmt: str, m: int, n: int, k: int, seed: int):
    rng = np.random.default_rng(seed)
    if fmt == "f32":
        a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
        b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
        return a, b, a.astype(np.float64), b.astype(np.float64)
    a = inputs.encode(fmt, rng.standard_normal(m * k))
    b = inputs.encode(fmt, rng.standard_normal(k * n))
    return a, b, inputs.decode(fmt, a).reshape(m, k), inputs.decode(fmt, b).reshape(k, n)


def to_dev(fmt: str, bits: np.ndarray, shape, dev) -> torch.Tensor:
    if fmt == "f32":
        return torch.from_numpy(np.ascontiguousarray(bits)).to(dev).view(shape)
    view = np.int16 if inputs.WIDTH[fmt] == 16 else np.uint8
    return torch.from_numpy(np.ascontiguousarray(bits).view(view).copy()).to(dev).view(TORCH[fmt]).view(shape)


def contract(av: np.ndarray, bv: np.ndarray, k: int, c: np.ndarray | float = 0.0) -> np.ndarray:
    return 2 * (k + 1) * 2.0**-22 * (np.abs(c) + np.abs(av) @ np.abs(bv))


@pytest.mark.parametrize("fmt", inputs.FORMATS + ["f32"])
@pytest.mark.parametrize("shape", SPLIT_SHAPES)
def test_split_tiles_within_the_contract(cuda, fmt, shape):
    m, n, k = shape
    a, b, av, bv = operands(fmt, m, n, k, seed=m + n + k)
    got = cairn_b200.gemm(to_dev(fmt, a, (m, k), cuda), to_dev(fmt, b, (k, n), cuda)).cpu().numpy()
    cairn_b200.stream_status()
    tol = contract(av, bv, k)
    if fmt == "f32":  # each operand read as tf32 (10 fraction bits)
        tol = tol + 2.0**-9 * (np.abs(av) @ np.abs(bv))
    err = np.abs(got - av @ bv)
    assert (err <= tol).all(), (fmt, shape, np.argwhere(err > tol)[:4].tolist())


@pytest.mark.parametrize("trans_a,trans_b", [(False, True), (True, False), (True, True)])
def test_split_tiles_of_transposed_operands(cuda, trans_a, trans_b):
    m, n, k = 520, 1032, 8200
    a, b, av, bv = operands("bf16", m, n, k, seed=7)
    a_st = np.ascontiguousarray(a.reshape(m, k).T) if trans_a else a.reshape(m, k)
    b_st = np.ascontiguousarray(b.reshape(k, n).T) if trans_b else b.reshape(k, n)
    got = cairn_b200.gemm(to_dev("bf16", a_st, a_st.shape, cuda), to_dev("bf16", b_st, b_st.shape, cuda),
                          trans_a=trans_a, trans_b=trans_b).cpu().numpy()
    cairn_b200.stream_status()
    assert (np.abs(got - av @ bv) <= contract(av, bv, k)).all()


def test_split_tiles_accumulate_into_the_old_values(cuda):
    m, n, k = 300, 700, 9000
    a, b, av, bv = operands("bf16", m, n, k, seed=9)
    c = np.random.default_rng(10).uniform(-4, 4, (m, n)).astype(np.float32)
    out = torch.from_numpy(c.copy()).to(cuda)
    cairn_b200.gemm(to_dev("bf16", a, (m, k), cuda), to_dev("bf16", b, (k, n), cuda), out=out, accumulate=True)
    cairn_b200.stream_status()
    want = c.astype(np.float64) + av @ bv
    assert (np.abs(out.cpu().numpy() - want) <= contract(av, bv, k, c)).all()


@pytest.mark.parametrize("relu", [True, False])
def test_split_tiles_through_the_bias_relu_bf16_epilogue(cuda, relu):
    m, n, k = 512, 1024, 8192
    a, b, av, bv = operands("bf16", m, n, k, seed=11)
    bias = (np.random.default_rng(12).standard_normal(n) * 0.1).astype(np.float32)
    got = cairn_b200.gemm(to_dev("bf16", a, (m, k), cuda), to_dev("bf16", b, (k, n), cuda),
                          bias=torch.from_numpy(bias).to(cuda), relu=relu, out_dtype=torch.bfloat16)
    cairn_b200.stream_status()
    g = got.float().cpu().numpy().astype(np.float64)
    w = av @ bv + bias
    if relu:
        w = np.maximum(w, 0.0)
    assert (np.abs(g - w) <= 2.0**-7 * np.maximum(np.abs(g), np.abs(w)) + 2 * contract(av, bv, k)).all()
    if relu:
        assert (g >= 0).all()


def test_split_tiles_give_the_same_bits_twice_and_after_other_shapes(cuda):
    """The workspace is lent again with a new epoch on every launch, grown for a larger split and reused for a
    smaller one: none of that changes a result."""
    m, n, k = 512, 1024, 8192
    a, b, _, _ = operands("bf16", m, n, k, seed=13)
    at, bt = to_dev("bf16", a, (m, k), cuda), to_dev("bf16", b, (k, n), cuda)
    first = cairn_b200.gemm(at, bt).clone()
    for shape in ((256, 256, 65536), (4096, 4096, 128), (300, 700, 9000)):
        x, y, _, _ = operands("bf16", *shape, seed=1)
        cairn_b200.gemm(to_dev("bf16", x, shape[::2], cuda), to_dev("bf16", y, shape[:0:-1], cuda))
    again = cairn_b200.gemm(at, bt)
    cairn_b200.stream_status()
    assert torch.equal(first.view(torch.int32), again.view(torch.int32))
