"""The `parallel` saxpy region and the `reduce +` collectors on the B200 against the CPU oracle, through the C ABI.

saxpy and the u64 checked sum are held bit for bit (north star: bit-exact for integer work; saxpy's two roundings
are exact IEEE operations). The f32 sum is held bit for bit to the host's exact sum rounded once (cr::par::sum) on
the reference's boundary and random cases, and within the north star's 1e-5 relative at BASELINE size.
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


def f32_bits(x) -> int:
    return int(np.asarray([x], np.float32).view(np.uint32)[0])


def test_saxpy_equals_the_reference_fixture_bit_for_bit(cuda):
    d = np.load(GOLDEN / "saxpy.npz")
    x, y = torch.from_numpy(d["x"]).to(cuda), torch.from_numpy(d["y"]).to(cuda)
    out = cairn_b200.saxpy(float(d["a"][0]), x, y)
    cairn_b200.stream_status()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), d["want"].view(np.uint32))


@pytest.mark.parametrize("n", [0, 1, 3, 4, 5, 31, 4097, (1 << 20) + 3])
@pytest.mark.parametrize("offset", [0, 1])
def test_saxpy_sizes_and_alignments(cuda, n, offset):
    x_np, y_np, a = inputs.saxpy_case(n + offset, seed=n)
    want = restated.saxpy(float(a), x_np[offset:], y_np[offset:])
    x, y = torch.from_numpy(x_np).to(cuda)[offset:], torch.from_numpy(y_np).to(cuda)[offset:]
    out = cairn_b200.saxpy(float(a), x, y)
    cairn_b200.stream_status()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_saxpy_in_place(cuda):
    x_np, y_np, a = inputs.saxpy_case(100_001, seed=1)
    want = restated.saxpy(float(a), x_np, y_np)
    x, y = torch.from_numpy(x_np).to(cuda), torch.from_numpy(y_np).to(cuda)
    cairn_b200.saxpy(float(a), x, y, out=y)
    cairn_b200.stream_status()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_sum_f32_equals_the_reference_exact_sum_bit_for_bit(cuda):
    d = np.load(GOLDEN / "sum.npz")
    keys = sorted({k.split("/")[0] for k in d.files})
    wrong = []
    for key in keys:
        x = torch.from_numpy(d[key + "/x"]).to(cuda)
        got = f32_bits(cairn_b200.reduce_sum(x))
        if got != int(d[key + "/want"][0]):
            wrong.append((str(d[key + "/name"]), hex(got), hex(int(d[key + "/want"][0]))))
    assert not wrong, wrong


def test_sum_f32_device_cell_and_unaligned_views(cuda):
    x_np = np.random.default_rng(3).uniform(-1, 1, 1_000_003).astype(np.float32)
    want = f32_bits(restated.sum_f32(x_np))
    x = torch.from_numpy(x_np).to(cuda)
    out = torch.empty(1, dtype=torch.float32, device=cuda)
    cairn_b200.reduce_sum(x, out=out)
    cairn_b200.stream_status()
    assert f32_bits(out.item()) == want
    for off in (1, 2, 3):
        assert f32_bits(cairn_b200.reduce_sum(x[off:])) == f32_bits(restated.sum_f32(x_np[off:]))


def test_sharded_parts_combine_to_the_whole_sum(cuda):
    """Four contiguous ranges reduced to parts and combined on the host equal the exact sum of the whole."""
    rng = np.random.default_rng(21)
    x_np = (rng.uniform(-1, 1, 400_000) * 2.0 ** rng.integers(-40, 40, 400_000)).astype(np.float32)
    x = torch.from_numpy(x_np).to(cuda)
    bounds = [0, 100_000, 200_001, 300_000, 400_000]
    parts = torch.empty(4, 3, dtype=torch.float64, device=cuda)
    for r in range(4):
        cairn_b200.reduce_sum(x[bounds[r]:bounds[r + 1]], out=parts[r])
    cairn_b200.stream_status()
    host = parts.cpu().numpy().ravel().copy()
    import ctypes as C
    result = C.c_float(0)
    assert cairn_b200.lib().cairn_b200_sum_f32_combine(host.ctypes.data, 4, C.byref(result)) == 0
    assert f32_bits(result.value) == f32_bits(restated.sum_f32(x_np))


def test_sum_u64_equals_the_reference_fixtures(cuda):
    d = np.load(GOLDEN / "u64.npz")
    for name, x_np in inputs.u64_cases().items():
        want_v, want_over = (int(t) for t in d[name + "/want"])
        x = torch.from_numpy(x_np.view(np.int64).copy()).to(cuda).view(torch.uint64)
        out = torch.zeros(1, dtype=torch.int64, device=cuda).view(torch.uint64)
        over = torch.zeros(1, dtype=torch.int32, device=cuda)
        cairn_b200.reduce_sum(x, out=out, overflow=over)
        cairn_b200.stream_status()
        assert int(out.view(torch.int64).item()) & (2**64 - 1) == want_v, name
        assert bool(over.item()) == bool(want_over), name
        if want_over:
            with pytest.raises(cairn_b200.CairnError):
                cairn_b200.reduce_sum(x)
        else:
            assert cairn_b200.reduce_sum(x) == want_v


@pytest.mark.slow
def test_baseline_2_30_saxpy_and_sums(cuda):
    """BASELINE config 4 on one GPU: n = 2^30, x, y ~ U[-1, 1] (seed 0), a = 2.5; u64 data[i] = i. saxpy is checked
    bit for bit on sampled blocks, the f32 sum against the oracle's exact sum within 1e-5 relative (and, as it is
    designed to be, bit for bit), and the u64 sum against n (n - 1) / 2."""
    n = 1 << 30
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.rand(n, device=cuda, generator=g) * 2 - 1
    y = torch.rand(n, device=cuda, generator=g) * 2 - 1
    out = cairn_b200.saxpy(2.5, x, y)
    cairn_b200.stream_status()
    for start in (0, 12345678, n - 4096):
        xs, ys = x[start:start + 4096].cpu().numpy(), y[start:start + 4096].cpu().numpy()
        want = restated.saxpy(2.5, xs, ys)
        assert np.array_equal(out[start:start + 4096].cpu().numpy().view(np.uint32), want.view(np.uint32))
    del out, y
    total = cairn_b200.reduce_sum(x)
    exact = restated.sum_f32(x.cpu().numpy())
    assert abs(total - float(exact)) <= 1e-5 * abs(float(exact))
    assert f32_bits(total) == f32_bits(exact)
    del x
    u = torch.arange(n, device=cuda, dtype=torch.int64).view(torch.uint64)
    assert cairn_b200.reduce_sum(u) == n * (n - 1) // 2


@pytest.mark.parametrize("n", [0, 3, 4, 1_000_003, (1 << 22) + 5])
@pytest.mark.parametrize("offset", [0, 1])
def test_mse_gradient_bit_for_bit_and_its_loss(cuda, n, offset):
    """cairn_b200_mse_grad (the MLP step's head): dy[i] = bf16((y[i] - t[i]) * (2 / n)), each operation rounded once
    as the oracle's step does it, bit for bit; loss = f32(sum (y - t)^2 / n) with the sum in f64, within one f32
    ulp of numpy's (the two add the exact squares in different orders). Offset 1 leaves the views off 16 bytes (the
    per-element path); n = 1,000,003 and 2^22 + 5 reach the vector path's tail."""
    rng = np.random.default_rng(n + offset)
    y_np = rng.standard_normal(n + offset).astype(np.float32)
    t_np = rng.standard_normal(n + offset).astype(np.float32)
    y = torch.from_numpy(y_np).to(cuda)[offset:]
    t = torch.from_numpy(t_np).to(cuda)[offset:]
    dy = torch.empty(n + offset, dtype=torch.int16, device=cuda)[offset:]
    loss = torch.full((1,), float("nan"), dtype=torch.float32, device=cuda)
    lib = cairn_b200.lib()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    assert lib.cairn_b200_mse_grad(stream, n, y.data_ptr(), t.data_ptr(), dy.data_ptr(), loss.data_ptr()) == 0
    cairn_b200.stream_status()
    d = y_np[offset:] - t_np[offset:]  # f32 subtraction, rounded once
    scale = np.float32(2.0) / np.float32(n) if n else np.float32(0.0)
    want_dy = inputs.encode("bf16", (d * scale).astype(np.float32))
    assert np.array_equal(dy.cpu().numpy().view(np.uint16), want_dy)
    want_loss = np.float32(np.sum(d.astype(np.float64) ** 2) / n) if n else np.float32(0.0)
    got = np.float32(loss.item())
    assert abs(int(got.view(np.int32)) - int(want_loss.view(np.int32))) <= 1, (got, want_loss)


def test_clock_marks_give_each_sms_clock_over_an_interval(cuda):
    """cairn_b200_clock_marks before and after 50 ms of work on the stream: every SM wrote both marks (one block lands
    on each SM at least), the timer advanced by the interval, and each SM's cycles over nanoseconds is a B200's clock
    (between 0.3 and 2.1 GHz). A misaligned or null slot array is refused."""
    from cairn_b200._lib import ERR_VIEW

    lib = cairn_b200.lib()
    stream = torch.cuda.current_stream(cuda)
    sms = lib.cairn_b200_sm_count()
    a = torch.zeros(512, dtype=torch.int64, device=cuda)
    b = torch.zeros(512, dtype=torch.int64, device=cuda)
    assert lib.cairn_b200_clock_marks(stream.cuda_stream, a.data_ptr(), 256) == 0
    torch.cuda._sleep(100_000_000)  # about 50 ms of spinning on the stream
    assert lib.cairn_b200_clock_marks(stream.cuda_stream, b.data_ptr(), 256) == 0
    cairn_b200.stream_status()
    a, b = a.view(-1, 2).cpu().numpy(), b.view(-1, 2).cpu().numpy()
    seen = (a[:, 1] > 0) & (b[:, 1] > a[:, 1])
    assert seen.sum() >= 0.9 * sms  # (%smid numbers the SMs; a block on each is all but certain)
    ghz = (b[seen, 0] - a[seen, 0]) / (b[seen, 1] - a[seen, 1])
    assert (ghz > 0.3).all() and (ghz < 2.1).all(), ghz
    assert ((b[seen, 1] - a[seen, 1]) > 1_000_000).all()  # more than 1 ms between the marks
    assert lib.cairn_b200_clock_marks(stream.cuda_stream, None, 256) == ERR_VIEW
    c = torch.zeros(8, dtype=torch.int64, device=cuda)
    assert lib.cairn_b200_clock_marks(stream.cuda_stream, c.data_ptr() + 4, 2) == ERR_VIEW
