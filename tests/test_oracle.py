"""Pins the CPU oracle (oracle/cairn_oracle.c) before any GPU result is judged against it.

1. Against the golden fixtures (tests/golden/*.npz), which hold the CAIRN reference's own host path's outputs
   (cr::tensor::multiply, cr::par::sum, cr::par::reduce over cr::Sum, cr::par::run, and config 3's step from the
   reference compiler's `derive grad` output): bit for bit. Runs anywhere.
2. Against the reference's host path live (oracle/_ref, built from the reference's headers where its source tree
   exists): bit for bit on fresh seeded inputs.
3. The exact sum against an independent rational model (Fraction arithmetic) on the rounding-boundary cases.
"""

from __future__ import annotations

import struct
from pathlib import Path

import numpy as np
import pytest

import inputs
from oracle import exact_sum_f32_bits, reference, restated

GOLDEN = Path(__file__).resolve().parent / "golden"
needs_ref = pytest.mark.skipif(not reference.available(), reason="the reference's host path is not built here")


def _groups(npz, depth: int):
    keys = sorted({"/".join(k.split("/")[:depth]) for k in npz.files})
    return keys


def test_restated_multiply_equals_the_reference_fixtures_bit_for_bit():
    d = np.load(GOLDEN / "mma.npz")
    cases = _groups(d, 3)
    assert len(cases) == 4 * (len(inputs.MMA_SHAPES) + len(inputs.TILE_SHAPES))
    for key in cases:
        fmt, _, shape = key.split("/")
        m, n, k = map(int, shape.split("x"))
        got = restated.mma(fmt, d[key + "/c"], d[key + "/a"], d[key + "/b"], m, n, k)
        want = d[key + "/want"]
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), key


def test_restated_sum_equals_the_reference_fixtures_bit_for_bit():
    d = np.load(GOLDEN / "sum.npz")
    for key in _groups(d, 1):
        got = np.asarray([restated.sum_f32(d[key + "/x"])], np.float32).view(np.uint32)[0]
        assert got == d[key + "/want"][0], (str(d[key + "/name"]), hex(got), hex(d[key + "/want"][0]))


def test_restated_u64_sum_equals_the_reference_fixtures():
    d = np.load(GOLDEN / "u64.npz")
    for name, x in inputs.u64_cases().items():
        v, over = restated.sum_u64(x)
        assert [v, int(over)] == [int(t) for t in d[name + "/want"]], name
    assert restated.sum_u64(np.arange(1_000_000, dtype=np.uint64)) == (499_999_500_000, False)


def test_restated_saxpy_equals_the_reference_fixture():
    d = np.load(GOLDEN / "saxpy.npz")
    got = restated.saxpy(float(d["a"][0]), d["x"], d["y"])
    assert np.array_equal(got.view(np.uint32), d["want"].view(np.uint32))


def test_restated_scans_equal_the_reference_fixture():
    d = np.load(GOLDEN / "scan.npz")
    sizes = sorted({int(k.split("/")[1]) for k in d.files})
    assert sizes, "scan.npz holds no cases"
    for n in sizes:
        got, total = restated.scan_u32(d[f"u32/{n}/x"])
        assert np.array_equal(got, d[f"u32/{n}/want"]) and total == int(d[f"u32/{n}/total"][0]), n
        got, total = restated.runmax_i32(d[f"max/{n}/x"])
        assert np.array_equal(got, d[f"max/{n}/want"]) and total == int(d[f"max/{n}/total"][0]), n


def test_restated_f32_region_gemm_equals_the_reference_fixture():
    d = np.load(GOLDEN / "f32gemm.npz")
    m, n, k = map(int, d["shape"])
    got = restated.mma("f32", np.zeros(m * n, np.float32), d["a"], d["b"], m, n, k)
    assert np.array_equal(got.view(np.uint32), d["want"].view(np.uint32))


def test_restated_f32_region_gemm_at_config_1_size():
    """M = N = K = 512, A and B ~ U[-1, 1] from seed 0, against the reference's region."""
    d = np.load(GOLDEN / "f32gemm.npz")
    a, b = inputs.config1_gemm()
    assert np.array_equal(np.concatenate([a[:4], b[:4]]).view(np.uint32), d["512/first"].view(np.uint32))
    got = restated.mma("f32", np.zeros(512 * 512, np.float32), a, b, 512, 512, 512)
    assert np.array_equal(got.view(np.uint32), d["512/want"].view(np.uint32))


MLP_KEYS = ("H", "Y", "dY", "dW2", "dH", "dW1", "dX")


def _mlp_loss_bound(want_loss: float, m: int) -> float:
    """The reference sums the m squares in f32 in index order (mse, a host `reduce +` over `for`); the step and the
    restatement sum them exactly in f64 and round once. Both lie within (m + 1) 2^-24 of the exact mean."""
    return 2 * (m + 1) * 2.0**-24 * abs(want_loss)


def test_restated_mlp_step_equals_the_reference_derive_grad_fixture():
    """Config 3's step at a reduced shape against the reference's own code: the dense layers and the adjoints its
    `derive grad` writes (oracle/grad/mlp_grad.cairn through the reference's compiler), relu_grad, mse_grad and
    cr::fp::narrow (tests/golden/mlp_grad.npz). Every tensor bit for bit; the loss within the f32 sum's bound."""
    d = np.load(GOLDEN / "mlp_grad.npz")
    B, D, H, O = map(int, d["shape"])
    got = restated.mlp_step(d["x"], d["w1"], d["w2"], d["t"], B, D, H, O)
    for key in MLP_KEYS:
        a, w = np.asarray(got[key]), np.asarray(d[f"want/{key}"])
        assert a.dtype == w.dtype and np.array_equal(a.view(np.uint8), w.view(np.uint8)), key
    want_loss = float(d["want/loss"][0])
    assert abs(float(got["loss"][0]) - want_loss) <= _mlp_loss_bound(want_loss, B * O)


@pytest.mark.skipif(not reference.grad_available(), reason="oracle/_ref/libmlp_grad.so is not built here")
def test_the_reference_derive_grad_chain_live():
    """The reference's derive-grad chain run now gives the fixture again, and agrees with the restatement on a
    second shape and seed."""
    d = np.load(GOLDEN / "mlp_grad.npz")
    B, D, H, O = map(int, d["shape"])
    live = reference.mlp_step(d["x"], d["w1"], d["w2"], d["t"], B, D, H, O)
    for key in (*MLP_KEYS, "loss"):
        assert np.array_equal(np.asarray(live[key]).view(np.uint8), np.asarray(d[f"want/{key}"]).view(np.uint8)), key
    B, D, H, O = 12, 40, 72, 24
    x, w1, w2, t = inputs.mlp_case(B, D, H, O, seed=5)
    ref, rest = reference.mlp_step(x, w1, w2, t, B, D, H, O), restated.mlp_step(x, w1, w2, t, B, D, H, O)
    for key in MLP_KEYS:
        assert np.array_equal(np.asarray(ref[key]).view(np.uint8), np.asarray(rest[key]).view(np.uint8)), key


def test_the_exact_sum_matches_an_independent_rational_model():
    for name, terms in inputs.sum_boundary_cases():
        x = np.asarray([inputs.f32(t) for t in terms], np.float32)
        got = int(np.asarray([restated.sum_f32(x)], np.float32).view(np.uint32)[0])
        want = exact_sum_f32_bits([float(t) for t in x])
        assert got == want, (name, hex(got), hex(want))
    rng = np.random.default_rng(11)
    for _ in range(20):
        x = (rng.uniform(-1, 1, 300) * 2.0 ** rng.integers(-140, 120, 300)).astype(np.float32)
        got = int(np.asarray([restated.sum_f32(x)], np.float32).view(np.uint32)[0])
        assert got == exact_sum_f32_bits([float(t) for t in x])


def test_storage_float_widening_is_exact_for_every_pattern():
    for fmt in inputs.FORMATS:
        bits = np.arange(1 << inputs.WIDTH[fmt], dtype=np.uint16 if inputs.WIDTH[fmt] == 16 else np.uint8)
        if inputs.WIDTH[fmt] == 16:
            bits = bits[::7]  # a spread of the 65536 patterns; the 8-bit formats are checked exhaustively
        got = restated.widen(fmt, bits).astype(np.float64)
        want = inputs.decode(fmt, bits)
        same = (got == want) | (np.isnan(got) & np.isnan(want))
        assert same.all(), (fmt, bits[~same][:5])


def test_bias_relu_epilogue_rounds_to_nearest_even():
    acc = np.asarray([1.0, -2.0, 1.00390625, 1.01171875, np.nan, -0.0, 3e38, -1e-40], np.float32)
    bias = np.zeros(8, np.float32)
    got = restated.bias_act(acc, bias, True, 1, 8)
    # 1 + 2^-8 is the tie between bf16 1.0 and 1.0078125: to even (1.0); 1 + 3 * 2^-8 ties up to 1.015625
    assert list(got[:4]) == [0x3F80, 0x0000, 0x3F80, 0x3F82]
    assert got[4] & 0x7FC0 == 0x7FC0 and got[5] in (0x0000, 0x8000) and got[6] == 0x7F62 and got[7] == 0


@needs_ref
@pytest.mark.parametrize("fmt", inputs.FORMATS)
def test_restated_multiply_equals_the_reference_live(fmt):
    for i, (m, n, k) in enumerate([(33, 47, 29), (1, 70, 130), (64, 8, 256), (5, 300, 3)]):
        c, a, b = inputs.mma_case(fmt, m, n, k, seed=77 + i)
        got = restated.mma(fmt, c, a, b, m, n, k)
        want = reference.mma(fmt, c, a, b, m, n, k)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (fmt, m, n, k)


@needs_ref
def test_restated_sums_equal_the_reference_live():
    rng = np.random.default_rng(5)
    for n in (1, 7, 8191, 16384, 100_001, 1 << 20):
        x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-30, 30, n)).astype(np.float32)
        assert restated.sum_f32(x).view(np.uint32) == reference.sum_f32(x).view(np.uint32), n
        u = rng.integers(0, 2**44, n, dtype=np.uint64)
        assert restated.sum_u64(u) == reference.sum_u64(u), n


@needs_ref
def test_restated_scans_equal_the_reference_live():
    if not reference.available():
        pytest.skip("oracle/_ref is not built (it needs the CAIRN reference tree)")
    rng = np.random.default_rng(21)
    for n in (1, 4097, 250_003):
        x = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
        a, b = restated.scan_u32(x), reference.scan_u32(x)
        assert np.array_equal(a[0], b[0]) and a[1] == b[1]
        v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
        a, b = restated.runmax_i32(v), reference.runmax_i32(v)
        assert np.array_equal(a[0], b[0]) and a[1] == b[1]


def test_restated_widening_and_saxpy_equal_the_reference_live():
    for fmt in inputs.FORMATS:
        bits = np.arange(256, dtype=np.uint8 if inputs.WIDTH[fmt] == 8 else np.uint16)
        r, o = reference.widen(fmt, bits), restated.widen(fmt, bits)
        assert np.array_equal(r.view(np.uint32), o.view(np.uint32)) or np.allclose(r, o, equal_nan=True), fmt
    x, y, a = inputs.saxpy_case(50_000, seed=9)
    assert np.array_equal(restated.saxpy(float(a), x, y).view(np.uint32),
                          reference.saxpy(float(a), x, y).view(np.uint32))


@needs_ref
def test_bf16_rounding_equals_the_reference_narrow():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(2000), rng.uniform(-1e30, 1e30, 200)]).astype(np.float32)
    got = restated.f32_to_bf16(x)
    want = np.asarray([reference.narrow_bf16(float(v)) for v in x], np.uint16)
    assert np.array_equal(got, want)


def test_f32_helper_rounds_like_struct():
    assert struct.pack("<f", inputs.f32(1.0 + 2**-30)) == struct.pack("<f", 1.0)
