"""The tensor-core multiply on the B200 against the CPU oracle, through the C ABI.

The bar is the reference's own device test (tests/soundness/test_tensor.py:182-226): every output within 2x the
contract bound (k + 1) * 2^-22 * (|c| + sum |a * b|) of the host reference, on its shapes (tails in every direction,
empty extents). Beyond it: the golden fixtures of the reference's own host multiply, the transposed operands of the
dense layer's backward, the fused bias/ReLU/bf16 epilogue, tf32, and the BASELINE 4096^3 product on sampled rows
within the north star's 2e-2 Frobenius tolerance. Two runs on one device give the same bits (docs/numerics.md: "Two
runs on one device give the same bits").
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"
TORCH = {"bf16": torch.bfloat16, "f16": torch.float16, "f8e4m3": torch.float8_e4m3fn, "f8e5m2": torch.float8_e5m2}
BITS = {"bf16": torch.int16, "f16": torch.int16, "f8e4m3": torch.uint8, "f8e5m2": torch.uint8}


def to_dev(fmt: str, bits: np.ndarray, dev) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(bits).view(np.int16 if inputs.WIDTH[fmt] == 16 else np.uint8).copy())
    return t.to(dev).view(TORCH[fmt])


def bound(fmt: str, c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
    av = np.abs(inputs.decode(fmt, a).reshape(m, k)) if fmt != "f32" else np.abs(a.reshape(m, k).astype(np.float64))
    bv = np.abs(inputs.decode(fmt, b).reshape(k, n)) if fmt != "f32" else np.abs(b.reshape(k, n).astype(np.float64))
    return (k + 1) * 2.0**-22 * (np.abs(c.reshape(m, n).astype(np.float64)) + av @ bv)


def device_mma(fmt: str, c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, dev) -> np.ndarray:
    ct = torch.from_numpy(c.copy()).to(dev)
    cairn_b200.mma_unordered(m, n, k, ct, to_dev(fmt, a, dev), to_dev(fmt, b, dev))
    cairn_b200.stream_status()
    return ct.cpu().numpy()


def within(got: np.ndarray, want: np.ndarray, tol: np.ndarray) -> np.ndarray:
    return np.abs(got.astype(np.float64) - want.astype(np.float64)) <= tol.ravel()


def test_the_reference_fixtures_within_twice_the_contract(cuda):
    d = np.load(GOLDEN / "mma.npz")
    keys = sorted({"/".join(k.split("/")[:3]) for k in d.files})
    for key in keys:
        fmt, _, shape = key.split("/")
        m, n, k = map(int, shape.split("x"))
        c, a, b, want = d[key + "/c"], d[key + "/a"], d[key + "/b"], d[key + "/want"]
        got = device_mma(fmt, c, a, b, m, n, k, cuda)
        if m * n == 0:
            continue
        ok = within(got, want, 2 * bound(fmt, c, a, b, m, n, k))
        assert ok.all(), (key, np.argwhere(~ok)[:4].ravel(), got[~ok][:4], want[~ok][:4])


@pytest.mark.parametrize("fmt", inputs.FORMATS)
@pytest.mark.parametrize("shape", [(128, 256, 64), (129, 264, 72), (256, 512, 1024), (1, 8, 8), (257, 136, 520),
                                   (300, 128, 8), (64, 1000, 200), (513, 392, 96)])
def test_tensor_path_shapes_against_the_oracle(cuda, fmt, shape):
    m, n, k = shape
    c, a, b = inputs.mma_case(fmt, m, n, k, seed=hash(shape) % 1000)
    want = restated.mma(fmt, c, a, b, m, n, k)
    got = device_mma(fmt, c, a, b, m, n, k, cuda)
    ok = within(got, want, 2 * bound(fmt, c, a, b, m, n, k))
    assert ok.all(), (fmt, shape, np.argwhere(~ok)[:4].ravel())


@pytest.mark.parametrize("shape", [(65, 63, 33), (3, 129, 31), (130, 70, 100), (7, 5, 3)])
def test_shapes_off_the_tensor_map_rules_take_the_simt_tiles(cuda, shape):
    """k or n not a multiple of 8 leaves rows off 16 bytes: the SIMT tile kernel computes the same contract."""
    m, n, k = shape
    for fmt in inputs.FORMATS:
        c, a, b = inputs.tile_case(fmt, m, n, k)
        want = restated.mma(fmt, c, a, b, m, n, k)
        got = device_mma(fmt, c, a, b, m, n, k, cuda)
        assert within(got, want, 2 * bound(fmt, c, a, b, m, n, k)).all(), (fmt, shape)


def test_a_multiply_with_no_products_keeps_every_old_value(cuda):
    c = np.asarray([-0.0, 1.5, -2.0, 3.0], np.float32)
    got = device_mma("bf16", c, np.zeros(0, np.uint16), np.zeros(0, np.uint16), 2, 2, 0, cuda)
    assert np.array_equal(got.view(np.uint32), c.view(np.uint32))


def test_two_runs_give_the_same_bits(cuda):
    m, n, k = 640, 768, 1024
    c, a, b = inputs.mma_case("bf16", m, n, k, seed=5)
    first = device_mma("bf16", c, a, b, m, n, k, cuda)
    second = device_mma("bf16", c, a, b, m, n, k, cuda)
    assert np.array_equal(first.view(np.uint32), second.view(np.uint32))


@pytest.mark.parametrize("trans_a,trans_b", [(False, False), (False, True), (True, False), (True, True)])
@pytest.mark.parametrize("fmt", ["bf16", "f16"])
def test_transposed_operands_of_the_backward(cuda, fmt, trans_a, trans_b):
    """dX = dY * W^T (trans_b) and dW = X^T * dY (trans_a), as derive grad's loops form them."""
    m, n, k = 200, 328, 136
    rng = np.random.default_rng(17)
    a = inputs.encode(fmt, rng.standard_normal(m * k))
    b = inputs.encode(fmt, rng.standard_normal(k * n))
    c = np.zeros(m * n, np.float32)
    want = restated.gemm_t16(c, a, b, m, n, k, trans_a, trans_b, fmt)
    at, bt = to_dev(fmt, a, cuda), to_dev(fmt, b, cuda)
    at = at.view(k, m) if trans_a else at.view(m, k)
    bt = bt.view(n, k) if trans_b else bt.view(k, n)
    got = cairn_b200.gemm(at, bt, trans_a=trans_a, trans_b=trans_b).cpu().numpy().ravel()
    cairn_b200.stream_status()
    av = np.abs(inputs.decode(fmt, a)).reshape(k, m).T if trans_a else np.abs(inputs.decode(fmt, a)).reshape(m, k)
    bv = np.abs(inputs.decode(fmt, b)).reshape(n, k).T if trans_b else np.abs(inputs.decode(fmt, b)).reshape(k, n)
    tol = 2 * (k + 1) * 2.0**-22 * (av @ bv)
    assert within(got, want, tol).all()


def test_accumulate_and_store_epilogues(cuda):
    m, n, k = 256, 256, 128
    rng = np.random.default_rng(4)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    c = rng.uniform(-4, 4, m * n).astype(np.float32)
    at, bt = to_dev("bf16", a, cuda).view(m, k), to_dev("bf16", b, cuda).view(k, n)
    out = torch.from_numpy(c.copy()).to(cuda).view(m, n)
    cairn_b200.gemm(at, bt, out=out, accumulate=True)
    stored = cairn_b200.gemm(at, bt)
    cairn_b200.stream_status()
    tol = 2 * bound("bf16", c, a, b, m, n, k)
    assert within(out.cpu().numpy().ravel(), restated.mma("bf16", c, a, b, m, n, k), tol).all()
    zero = np.zeros(m * n, np.float32)
    assert within(stored.cpu().numpy().ravel(), restated.mma("bf16", zero, a, b, m, n, k), tol).all()


def _bf16_close(got_bits: np.ndarray, want_bits: np.ndarray, acc_tol: np.ndarray) -> np.ndarray:
    g, w = inputs.decode("bf16", got_bits), inputs.decode("bf16", want_bits)
    return (np.abs(g - w) <= 2.0**-7 * np.maximum(np.abs(g), np.abs(w)) + acc_tol.ravel()) | (got_bits == want_bits)


@pytest.mark.parametrize("relu", [True, False])
@pytest.mark.parametrize("shape", [(384, 520, 256), (300, 264, 136), (520, 776, 72)])
def test_fused_bias_relu_bf16_epilogue(cuda, relu, shape):
    """bf16(act(acc + bias)): within one bf16 rounding of the oracle's epilogue on its own accumulator. The shapes
    leave partial tiles in both directions, on the 256 x 512 and the 256 x 256 pair tiles, whose chunks the TMA
    stores clip at the output's edges."""
    m, n, k = shape
    rng = np.random.default_rng(8)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    acc = restated.mma("bf16", np.zeros(m * n, np.float32), a, b, m, n, k)
    want = restated.bias_act(acc, bias, relu, m, n)
    at, bt = to_dev("bf16", a, cuda).view(m, k), to_dev("bf16", b, cuda).view(k, n)
    got = cairn_b200.gemm(at, bt, bias=torch.from_numpy(bias).to(cuda), relu=relu, out_dtype=torch.bfloat16)
    cairn_b200.stream_status()
    got_bits = got.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    ok = _bf16_close(got_bits, want, 2 * bound("bf16", np.zeros(m * n, np.float32), a, b, m, n, k))
    assert ok.all()
    if relu:
        assert (inputs.decode("bf16", got_bits) >= 0).all()


# ---- mixed-width tiles: shapes whose uniform 256 x 512 cover leaves pairs idle get tiles of 512 and 384 columns ----
PLANNED = [(2900, 3900, 72), (3072, 4096, 64), (2816, 3200, 136)]


@pytest.mark.parametrize("shape", PLANNED)
def test_planned_tiles_bias_relu_bf16_against_the_oracle(cuda, shape):
    """Shapes the host's tile planner covers with 512- and 384-column tiles (ragged bands and a ragged last unit in
    the first): bf16(relu(acc + bias)) within one bf16 rounding of the oracle's epilogue, every element."""
    m, n, k = shape
    rng = np.random.default_rng(m)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    acc = restated.mma("bf16", np.zeros(m * n, np.float32), a, b, m, n, k)
    want = restated.bias_act(acc, bias, True, m, n)
    at, bt = to_dev("bf16", a, cuda).view(m, k), to_dev("bf16", b, cuda).view(k, n)
    got = cairn_b200.gemm(at, bt, bias=torch.from_numpy(bias).to(cuda), relu=True, out_dtype=torch.bfloat16)
    cairn_b200.stream_status()
    got_bits = got.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    assert _bf16_close(got_bits, want, 2 * bound("bf16", np.zeros(m * n, np.float32), a, b, m, n, k)).all()


@pytest.mark.parametrize("fmt", ["bf16", "f16"])
@pytest.mark.parametrize("form", ["accumulate", "store", "transposed_a", "transposed_b"])
def test_planned_tiles_f32_outputs_against_the_oracle(cuda, fmt, form):
    """The planned cover with the f32 epilogues: mma_unordered's C += A B (TMA reduce-adds), C = A B stored, A read
    transposed (A's layout does not enter the tiles), and B stored n x k (its K-major boxes of 64 rows, one per
    128-column unit's half, take tiles of 3 units as well as 4)."""
    m, n, k = 2900, 3900, 72
    c, a, b = inputs.mma_case(fmt, m, n, k, seed=k)
    if form == "accumulate":
        want = restated.mma(fmt, c, a, b, m, n, k)
        ct = torch.from_numpy(c.copy()).to(cuda)
        cairn_b200.mma_unordered(m, n, k, ct, to_dev(fmt, a, cuda), to_dev(fmt, b, cuda))
        tol = 2 * bound(fmt, c, a, b, m, n, k)
    else:
        want = restated.mma(fmt, np.zeros(m * n, np.float32), a, b, m, n, k)
        a_dev, b_dev = to_dev(fmt, a, cuda).view(m, k), to_dev(fmt, b, cuda).view(k, n)
        if form == "transposed_a":
            a_dev = a_dev.t().contiguous()
        if form == "transposed_b":
            b_dev = b_dev.t().contiguous()
        ct = cairn_b200.gemm(a_dev, b_dev, trans_a=form == "transposed_a", trans_b=form == "transposed_b",
                             out_dtype=torch.float32)
        tol = 2 * bound(fmt, np.zeros(m * n, np.float32), a, b, m, n, k)
    cairn_b200.stream_status()
    assert within(ct.cpu().numpy().ravel(), want.ravel(), tol).all()


_UNIFORM_COVER = r"""
import sys
sys.path[:0] = [sys.argv[1], sys.argv[1] + "/tests"]
import numpy as np, torch
import cairn_b200
d = dict(np.load(sys.argv[2]))
dev = torch.device("cuda", 0)
m, n, k = (int(v) for v in d["mnk"])
a = torch.from_numpy(d["a"].view(np.int16)).to(dev).view(torch.bfloat16).view(m, k)
b = torch.from_numpy(d["b"].view(np.int16)).to(dev).view(torch.bfloat16).view(k, n)
out = cairn_b200.gemm(a, b, bias=torch.from_numpy(d["bias"]).to(dev), relu=True, out_dtype=torch.bfloat16)
f32 = cairn_b200.gemm(a, b, out_dtype=torch.float32)
tb = cairn_b200.gemm(a, b.t().contiguous(), trans_b=True, out_dtype=torch.float32)
cairn_b200.stream_status()
np.savez(sys.argv[3], bf16=out.view(torch.int16).cpu().numpy(), f32=f32.cpu().numpy(), tb=tb.cpu().numpy())
"""


@pytest.mark.parametrize("shape", [(4096, 4096, 256), (2900, 3900, 72)])
def test_planned_and_uniform_covers_give_the_same_bits(cuda, tmp_path, shape):
    """Each output's k order is the same whatever the width of the tile that holds it, so the planned cover and the
    uniform one (CAIRN_B200_PLAN=0, in a child process) give the same bits: no tile is missed or run twice."""
    import os
    import subprocess
    import sys
    from pathlib import Path

    m, n, k = shape
    rng = np.random.default_rng(k)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    src, dst = tmp_path / "in.npz", tmp_path / "out.npz"
    np.savez(src, a=a, b=b, bias=bias, mnk=np.asarray(shape))
    root = str(Path(__file__).resolve().parents[1])
    done = subprocess.run([sys.executable, "-c", _UNIFORM_COVER, root, str(src), str(dst)], capture_output=True,
                          text=True, timeout=600, env=dict(os.environ, CAIRN_B200_PLAN="0"))
    assert done.returncode == 0, done.stderr[-3000:]
    uniform = np.load(dst)
    at, bt = to_dev("bf16", a, cuda).view(m, k), to_dev("bf16", b, cuda).view(k, n)
    planned = cairn_b200.gemm(at, bt, bias=torch.from_numpy(bias).to(cuda), relu=True, out_dtype=torch.bfloat16)
    planned_f32 = cairn_b200.gemm(at, bt, out_dtype=torch.float32)
    planned_tb = cairn_b200.gemm(at, bt.t().contiguous(), trans_b=True, out_dtype=torch.float32)
    cairn_b200.stream_status()
    assert np.array_equal(planned.view(torch.int16).cpu().numpy(), uniform["bf16"])
    assert np.array_equal(planned_f32.cpu().numpy().view(np.uint32), uniform["f32"].view(np.uint32))
    assert np.array_equal(planned_tb.cpu().numpy().view(np.uint32), uniform["tb"].view(np.uint32))


def test_tf32_multiply_of_f32_operands(cuda):
    m, n, k = 300, 264, 392
    rng = np.random.default_rng(12)
    a = rng.uniform(-1, 1, m * k).astype(np.float32)
    b = rng.uniform(-1, 1, k * n).astype(np.float32)
    c = rng.uniform(-4, 4, m * n).astype(np.float32)
    want = restated.mma("f32", c, a, b, m, n, k)
    ct = torch.from_numpy(c.copy()).to(cuda)
    cairn_b200.mma_unordered(m, n, k, ct, torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda))
    cairn_b200.stream_status()
    mag = np.abs(c).reshape(m, n).astype(np.float64) + np.abs(a.reshape(m, k)).astype(np.float64) @ np.abs(
        b.reshape(k, n)).astype(np.float64)
    tol = (2.0**-9 + (k + 1) * 2.0**-22) * mag  # each operand rounded to tf32 (10 fraction bits), then f32 sums
    assert within(ct.cpu().numpy(), want, tol).all()


@pytest.mark.slow
def test_baseline_4096_cubed_bias_relu_on_sampled_rows(cuda):
    """4096^3 bf16, A, B ~ N(0,1) cast to bf16, bias ~ N(0, 0.1), ReLU, bf16 out. Sampled rows
    against the oracle: Frobenius relative error within 2e-2 (the north star) and every element within one bf16
    rounding plus twice the contract bound."""
    m = n = k = 4096
    g = torch.Generator(device=cuda).manual_seed(0)
    a = torch.randn(m, k, device=cuda, generator=g).to(torch.bfloat16)
    b = torch.randn(k, n, device=cuda, generator=g).to(torch.bfloat16)
    bias = torch.randn(n, device=cuda, generator=g) * 0.1
    out = cairn_b200.gemm(a, b, bias=bias, relu=True, out_dtype=torch.bfloat16)
    cairn_b200.stream_status()
    rows = [0, 1, 127, 128, 2047, 4095]
    a_np = a.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    b_np = b.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    bias_np = bias.cpu().numpy()
    for r in rows:
        acc = restated.mma_bf16_rows(a_np, b_np, m, n, k, r, r + 1)
        want = restated.bias_act(acc, bias_np, True, 1, n)
        got = out[r].view(torch.int16).cpu().numpy().view(np.uint16)
        gv, wv = inputs.decode("bf16", got), inputs.decode("bf16", want)
        assert np.linalg.norm(gv - wv) <= 2e-2 * np.linalg.norm(wv), r
        av = np.abs(inputs.decode("bf16", a_np[r * k:(r + 1) * k]))
        tol = 2 * (k + 1) * 2.0**-22 * (av @ np.abs(inputs.decode("bf16", b_np).reshape(k, n)))
        assert _bf16_close(got, want, tol).all(), r


@pytest.mark.parametrize("trans_a,trans_b", [(False, False), (False, True), (True, False), (True, True)])
def test_tf32_every_operand_layout(cuda, trans_a, trans_b):
    """An M/N-major 32-bit operand needs the 32-byte-atom swizzle (SW128_32B); both layouts are held to f64 within
    the tf32 bound."""
    m, n, k = 264, 392, 200
    rng = np.random.default_rng(31)
    a = rng.uniform(-1, 1, (m, k)).astype(np.float32)
    b = rng.uniform(-1, 1, (k, n)).astype(np.float32)
    at = torch.from_numpy(np.ascontiguousarray(a.T) if trans_a else a).to(cuda)
    bt = torch.from_numpy(np.ascontiguousarray(b.T) if trans_b else b).to(cuda)
    got = cairn_b200.gemm(at, bt, trans_a=trans_a, trans_b=trans_b).cpu().numpy()
    cairn_b200.stream_status()
    want = a.astype(np.float64) @ b.astype(np.float64)
    tol = (2.0**-9 + (k + 1) * 2.0**-22) * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64))
    assert (np.abs(got - want) <= tol).all()


@pytest.mark.parametrize("fmt", inputs.FORMATS)
@pytest.mark.parametrize("shape", [(256, 256, 64), (384, 520, 200), (257, 264, 72), (1024, 768, 1000)])
def test_the_two_sm_pair_tile_against_the_oracle(cuda, fmt, shape):
    """m and n of 256 or more run the cta_group::2 kernel (256 x 256 tiles over CTA pairs)."""
    m, n, k = shape
    c, a, b = inputs.mma_case(fmt, m, n, k, seed=sum(shape))
    want = restated.mma(fmt, c, a, b, m, n, k)
    got = device_mma(fmt, c, a, b, m, n, k, cuda)
    ok = within(got, want, 2 * bound(fmt, c, a, b, m, n, k))
    assert ok.all(), (fmt, shape, np.argwhere(~ok)[:4].ravel())


@pytest.mark.parametrize("trans_a,trans_b", [(False, True), (True, False), (True, True)])
@pytest.mark.parametrize("fmt", ["bf16", "f16", "f8e4m3"])
def test_the_pair_tile_with_transposed_operands(cuda, fmt, trans_a, trans_b):
    m, n, k = 320, 392, 264
    rng = np.random.default_rng(3)
    a = inputs.encode(fmt, rng.standard_normal(m * k))
    b = inputs.encode(fmt, rng.standard_normal(k * n))
    av = inputs.decode(fmt, a).reshape(m, k)
    bv = inputs.decode(fmt, b).reshape(k, n)
    a_st = np.ascontiguousarray(a.reshape(m, k).T) if trans_a else a.reshape(m, k)
    b_st = np.ascontiguousarray(b.reshape(k, n).T) if trans_b else b.reshape(k, n)
    got = cairn_b200.gemm(to_dev(fmt, a_st, cuda).view(a_st.shape), to_dev(fmt, b_st, cuda).view(b_st.shape),
                          trans_a=trans_a, trans_b=trans_b).cpu().numpy()
    cairn_b200.stream_status()
    want = av @ bv
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(av) @ np.abs(bv))
    assert (np.abs(got - want) <= tol).all()


def test_baseline_config_1_f32_gemm_512_cubed(cuda):
    """BASELINE config 1's f32 GEMM (512^3, A, B ~ U[-1, 1] from seed 0), which the reference runs as a `parallel`
    region on its host pool: the device form reads the f32 operands as tf32, within the tf32 bound of the oracle's
    in-order f32 sums."""
    m = n = k = 512
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, m * k).astype(np.float32)
    b = rng.uniform(-1, 1, k * n).astype(np.float32)
    c = np.zeros(m * n, np.float32)
    want = restated.mma("f32", c, a, b, m, n, k)
    ct = torch.from_numpy(c.copy()).to(cuda)
    cairn_b200.mma_unordered(m, n, k, ct, torch.from_numpy(a).to(cuda), torch.from_numpy(b).to(cuda))
    cairn_b200.stream_status()
    mag = np.abs(a.reshape(m, k)).astype(np.float64) @ np.abs(b.reshape(k, n)).astype(np.float64)
    tol = (2.0**-9 + (k + 1) * 2.0**-22) * mag
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want.reshape(m, n)) <= tol).all()


# bf16 bit patterns of every kind a ReLU's forward output can hold: +-0, +-subnormal, +-normal, +-max, +-inf, NaNs
MASK_SPECIALS = np.asarray([0x0000, 0x8000, 0x0001, 0x8001, 0x007F, 0x0080, 0x3F80, 0xBF80, 0x7F7F, 0xFF7F, 0x7F80,
                            0xFF80, 0x7FC0, 0xFFC0, 0x7F81], np.uint16)


@pytest.mark.parametrize("m,n,k,trans_b", [(512, 768, 128, True), (256, 1024, 256, False), (300, 260, 64, True),
                                           (64, 200, 32, True)])
def test_relu_grad_is_the_product_kept_where_the_forward_was_positive(cuda, m, n, k, trans_b):
    """cairn_b200_gemm_relu_grad against the plain bf16 product of the same operands with the mask applied on the
    host: the product's bits wherever the mask is > 0 (as a float), +0 elsewhere. The shapes reach the pair tile
    with 16-byte rows (the mask read where the outputs are written back), rows off 16 bytes (n = 260, the mask read
    per element) and the one-SM tile (m = 64)."""
    rng = np.random.default_rng(m + n + k)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    mask = np.where(rng.random(m * n) < 0.5, inputs.encode("bf16", rng.standard_normal(m * n)),
                    rng.choice(MASK_SPECIALS, m * n)).astype(np.uint16)
    at = to_dev("bf16", a, cuda).view(m, k)
    bt = to_dev("bf16", b, cuda).view(n, k) if trans_b else to_dev("bf16", b, cuda).view(k, n)
    mt = to_dev("bf16", mask, cuda)
    plain = cairn_b200.gemm(at, bt, trans_b=trans_b, out_dtype=torch.bfloat16)
    got = torch.empty(m, n, dtype=torch.bfloat16, device=cuda)
    lib = cairn_b200.lib()
    status = lib.cairn_b200_gemm_relu_grad(torch.cuda.current_stream(cuda).cuda_stream, cairn_b200._lib.BF16, m, n, k,
                                           at.data_ptr(), 0, bt.data_ptr(), int(trans_b), got.data_ptr(),
                                           mt.data_ptr())
    assert status == 0
    cairn_b200.stream_status()
    positive = inputs.decode("bf16", mask) > 0
    plain_bits = plain.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    got_bits = got.view(torch.int16).cpu().numpy().view(np.uint16).ravel()
    want = np.where(positive, plain_bits, np.uint16(0))
    bad = np.flatnonzero(got_bits != want)
    assert bad.size == 0, (bad[:4], got_bits[bad[:4]], want[bad[:4]], mask[bad[:4]])


@pytest.mark.parametrize("shape", [(300, 776, 136), (520, 264, 72), (257, 512, 64)])
def test_stored_f32_products_with_partial_tiles(cuda, shape):
    """C = A B stored as f32 (no old value read) on shapes whose last row band and column tile are partial: the
    chunks leave through TMA stores in 16-column halves, clipped at the output's edges; every element within twice
    the contract bound of the oracle."""
    m, n, k = shape
    rng = np.random.default_rng(m + n)
    a = inputs.encode("bf16", rng.standard_normal(m * k))
    b = inputs.encode("bf16", rng.standard_normal(k * n))
    at, bt = to_dev("bf16", a, cuda).view(m, k), to_dev("bf16", b, cuda).view(k, n)
    out = torch.full((m, n), float("nan"), device=cuda)
    cairn_b200.gemm(at, bt, out=out)
    cairn_b200.stream_status()
    zero = np.zeros(m * n, np.float32)
    want = restated.mma("bf16", zero, a, b, m, n, k)
    assert within(out.cpu().numpy().ravel(), want, 2 * bound("bf16", zero, a, b, m, n, k)).all()


def test_a_chain_of_products_on_one_stream_reads_each_output_after_it_is_written(cuda):
    """Products queued back to back on one stream, each reading what the one before wrote (and the third overwriting
    what the second reads), give the same bits as the same chain with the host waiting after every product: a pair
    launch that starts while the product before it runs touches no operand or output before that product is done."""
    rng = torch.Generator(device=cuda).manual_seed(21)
    m = n = 1024
    a = torch.randn(m, 512, device=cuda, generator=rng).bfloat16()
    b1 = torch.randn(512, n, device=cuda, generator=rng).bfloat16()
    b3 = torch.randn(512, n, device=cuda, generator=rng).bfloat16()
    w = (torch.randn(n, n, device=cuda, generator=rng) * 0.05).bfloat16()
    bias = (torch.randn(n, device=cuda, generator=rng) * 0.1).float()
    c1 = torch.empty(m, n, device=cuda, dtype=torch.bfloat16)
    c2 = torch.empty_like(c1)
    c3 = torch.empty(n, n, device=cuda)

    def chain(wait: bool):
        for t in (c1, c2, c3):
            t.fill_(float("nan"))
        steps = [
            lambda: cairn_b200.gemm(a, b1, out=c1, bias=bias, relu=True, out_dtype=torch.bfloat16),
            lambda: cairn_b200.gemm(c1, w, out=c2, out_dtype=torch.bfloat16),
            lambda: cairn_b200.gemm(a, b3, out=c1, out_dtype=torch.bfloat16),
            lambda: cairn_b200.gemm(c2, c1, trans_a=True, out=c3),
        ]
        for s in steps:
            s()
            if wait:
                torch.cuda.synchronize(cuda)
        cairn_b200.stream_status()
        return c2.view(torch.int16).clone(), c3.view(torch.int32).clone()

    want2, want3 = chain(wait=True)
    assert not torch.isnan(want3.view(torch.float32)).any()
    ref2 = (torch.relu(a.float() @ b1.float() + bias).bfloat16().float() @ w.float())
    assert ((want2.view(torch.bfloat16).float() - ref2).norm() / ref2.norm()).item() < 2e-2
    for _ in range(5):
        got2, got3 = chain(wait=False)
        assert torch.equal(got2, want2) and torch.equal(got3, want3)
