"""Compiler-emitted CAIRN programs on the drop-in runtime headers (include/cairn_b200/runtime).

tests/dropin/programs/hotpath.cairn is compiled by the reference's own compiler (`cairn build --kind library --header
--device-target sm_100a`), and the C++ it emits is built, unchanged, by the reference toolchain's own device command
(-Werror all-warnings included) with the drop-in headers first on the include path (tests/dropin/build_emitted.py).
The reference's cairn_exec.hpp and cairn_reuse.hpp then run the B200 machine, whose regions, collectors and multiply
are this project's. Each cf_/cq_ entry is held to the oracle: regions, integer collectors and the compaction bit for
bit; the f32 `reduce +` (the device path's f32 fold in an unspecified order, docs/numerics.md) within
n * 2^-24 * sum |x|; the multiply within twice its contract bound. The same emitted library built over the
reference's headers alone (baseline/_ref/libhotpath_ref.so) runs the reference's own machine for the last test.

The libraries are built by __graft_entry__.build() where the CAIRN reference tree is present; without them these
tests are skipped, naming why."""

from __future__ import annotations

import ctypes as C
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]
LIB = ROOT / "tests" / "dropin" / "_build" / "libhotpath.so"
PROBE = ROOT / "tests" / "dropin" / "_build" / "libscanprobe.so"
REF_LIB = ROOT / "baseline" / "_ref" / "libhotpath_ref.so"

z, p, f32, u32, u64, i32 = C.c_size_t, C.c_void_p, C.c_float, C.c_uint32, C.c_uint64, C.c_int32
# The entries of tests/dropin/_build/hotpath.h (the header the reference compiler wrote), with their C types.
ENTRIES = {
    "cf_saxpy": (None, [z, p, p, p, f32]), "cq_saxpy": (None, [p, z, p, p, p, f32]),
    "cf_saxpy4": (None, [z, p, p, p, f32]), "cq_saxpy4": (None, [p, z, p, p, p, f32]),
    "cf_scaled": (None, [z, p, f32]), "cq_scaled": (None, [p, z, p, f32]),
    "cf_blend": (None, [z, p, p, f32, f32]),
    "cf_blur": (None, [z, p, p]), "cq_blur": (None, [p, z, p, p]), "cf_mix": (None, [z, p, p, p]),
    "cf_dsum": (f32, [z, p]), "cf_usum": (u64, [z, p]), "cf_vmax": (i32, [z, p]), "cf_usum_into": (None, [z, p, p]),
    "cf_prefix": (u64, [z, p, p]), "cf_wprefix": (u32, [z, p, p]), "cf_runmax": (i32, [z, p, p]),
    "cf_wscan": (None, [z, p, p]), "cf_positives": (z, [z, p, p]),
    "cf_gemm": (None, [z, z, z, z, p, z, p, z, p]), "cq_gemm": (None, [p, z, z, z, z, p, z, p, z, p]),
    "cf_gemm_f16": (None, [z, z, z, z, p, z, p, z, p]), "cf_gemm_e4m3": (None, [z, z, z, z, p, z, p, z, p]),
    "cairn_hotpath_device_stream": (None, [p]),
}


def _typed(h: C.CDLL, entries: dict) -> C.CDLL:
    for name, (res, args) in entries.items():
        fn = getattr(h, name)
        fn.restype, fn.argtypes = res, args
    return h


@pytest.fixture(scope="module")
def emitted(cuda):
    if not LIB.exists():
        pytest.skip("tests/dropin/_build/libhotpath.so is not built (it needs the CAIRN reference's compiler)")
    cairn_b200.lib()  # the program links libcairn_b200.so: load it from the tree first
    return _typed(C.CDLL(str(LIB)), ENTRIES)


@pytest.fixture(scope="module")
def probe(cuda):
    if not PROBE.exists():
        pytest.skip("tests/dropin/_build/libscanprobe.so is not built (it needs the CAIRN reference's headers)")
    return _typed(C.CDLL(str(PROBE)), {"cf_prefix_escape": (None, [z, p, p]), "b200_scan_u32_scratch": (z, [z]),
                                       "b200_scan_u32": (None, [p, z, p, p, p])})


def _dev(a: np.ndarray, cuda) -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.cpu().numpy().view(np.uint32)


# ---- regions -----------------------------------------------------------------------------------------------------
SIZES = [1, 31, 1023, 1024, 1025, 4097, (1 << 22) + 3]


@pytest.mark.parametrize("entry", ["cf_saxpy", "cf_saxpy4"])
@pytest.mark.parametrize("n", SIZES)
def test_emitted_saxpy_regions(emitted, cuda, entry, n):
    x_np, y_np, a = inputs.saxpy_case(n, seed=n)
    x, y = _dev(x_np, cuda), _dev(y_np, cuda)
    out = torch.empty_like(x)
    getattr(emitted, entry)(n, out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    assert np.array_equal(_bits(out), restated.saxpy(float(a), x_np, y_np).view(np.uint32))


@pytest.mark.parametrize("n", [5, 4099, 1_000_001])
def test_emitted_vector_region_off_its_chunk_width_runs_the_scalar_lanes(emitted, cuda, n):
    """`plan saxpy4 { vector 4; }` with views one element past a 16-byte boundary: the chunk check at launch sends
    the region to its scalar lanes, with the same bits."""
    x_np, y_np, a = inputs.saxpy_case(n + 1, seed=n)
    x, y = _dev(x_np, cuda)[1:], _dev(y_np, cuda)[1:]
    out = torch.empty(n + 1, dtype=torch.float32, device=cuda)[1:]
    emitted.cf_saxpy4(n, out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    assert np.array_equal(_bits(out), restated.saxpy(float(a), x_np[1:], y_np[1:]).view(np.uint32))


@pytest.mark.parametrize("entry", ["cq_saxpy", "cq_saxpy4"])
def test_emitted_enqueued_regions_on_the_callers_stream(emitted, cuda, entry):
    x_np, y_np, a = inputs.saxpy_case(3_000_001, seed=2)
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):  # inputs made on the caller's stream: the region must run after them
        x, y = _dev(x_np, cuda), _dev(y_np, cuda)
        out = torch.empty_like(x)
        getattr(emitted, entry)(s.cuda_stream, x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    s.synchronize()
    assert np.array_equal(_bits(out), restated.saxpy(float(a), x_np, y_np).view(np.uint32))


@pytest.mark.parametrize("n", [1, 127, 128 * 4 + 1, 2_000_003])
def test_emitted_planned_region_block_per_lane_unroll(emitted, cuda, n):
    """`plan scaled { block 128; per_lane 4; unroll 4; }`: x = a * x in place, every index once (a second pass would
    scale twice), whole tiles and the partial one."""
    x_np = np.random.default_rng(n).uniform(-4, 4, n).astype(np.float32)
    x = _dev(x_np, cuda)
    emitted.cf_scaled(n, x.data_ptr(), 1.75)
    assert np.array_equal(_bits(x), (np.float32(1.75) * x_np).view(np.uint32))
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        emitted.cq_scaled(s.cuda_stream, n, x.data_ptr(), -0.5)
    s.synchronize()
    assert np.array_equal(_bits(x), (np.float32(-0.5) * (np.float32(1.75) * x_np)).view(np.uint32))


@pytest.mark.parametrize("n", [1, 4097, 3_000_017])
def test_emitted_fused_chain(emitted, cuda, n):
    """`plan blend { fuse 2; }`: two regions run as one, the scaled value held in each lane; out = (a * x) + b with
    both roundings, bit for bit."""
    x_np = np.random.default_rng(n + 9).uniform(-1, 1, n).astype(np.float32)
    x, out = _dev(x_np, cuda), torch.empty(n, dtype=torch.float32, device=cuda)
    emitted.cf_blend(n, out.data_ptr(), x.data_ptr(), 2.5, -0.75)
    want = (np.float32(2.5) * x_np) + np.float32(-0.75)
    assert np.array_equal(_bits(out), want.view(np.uint32))


def _blur(x: np.ndarray) -> np.ndarray:
    want = x.copy()
    if x.size >= 5:
        two, three = np.float32(2.0), np.float32(3.0)
        mid = x[:-4] + x[1:-3] * two
        mid = mid + x[2:-2] * three
        mid = mid + x[3:-1]
        want[2:-2] = mid + x[4:]
    return want


@pytest.mark.parametrize("n", [1, 4, 5, 127, 128, 129, 131, 100_003, 5_000_011])
def test_emitted_staged_region(emitted, cuda, n):
    """`plan blur { stage 2; block 128; }`: every tile a block loads holds what its lanes read, at the array's edges,
    between blocks and across the two tiles a block alternates between; the body's f32 arithmetic in source order
    (--fmad=false), bit for bit."""
    x_np = np.random.default_rng(n + 4).uniform(-1, 1, n).astype(np.float32)
    x, out = _dev(x_np, cuda), torch.empty(n, dtype=torch.float32, device=cuda)
    emitted.cf_blur(n, out.data_ptr(), x.data_ptr())
    assert np.array_equal(_bits(out), _blur(x_np).view(np.uint32))
    out.zero_()
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        emitted.cq_blur(s.cuda_stream, n, out.data_ptr(), x.data_ptr())
    s.synchronize()
    assert np.array_equal(_bits(out), _blur(x_np).view(np.uint32))


@pytest.mark.parametrize("n", [1, 2, 3, 255, 256, 257, 2047, 2048, 2049, 2051, 100_003, 4_194_305])
def test_emitted_staged_region_of_two_arrays_at_the_default_block(emitted, cuda, n):
    """`plan mix { stage 1; }`: an f32 and an f64 array staged in one tile (the f64 one placed after the f32 one's
    bytes, both sized by the tile's width), at the plan's default block of 256 threads, whose tiles hold 2048
    indices: out = (f64(x[i-1]) + y[i+1]) - y[i-1] * 0.5 inside, y[i] at the ends, bit for bit."""
    rng = np.random.default_rng(n + 11)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n)
    xd, yd, out = _dev(x, cuda), _dev(y, cuda), torch.empty(n, dtype=torch.float64, device=cuda)
    emitted.cf_mix(n, out.data_ptr(), xd.data_ptr(), yd.data_ptr())
    want = y.copy()
    if n >= 3:
        want[1:-1] = (x[:-2].astype(np.float64) + y[2:]) - y[:-2] * 0.5
    assert np.array_equal(out.cpu().numpy().view(np.uint64), want.view(np.uint64))


def test_a_bound_stream_orders_the_synchronous_entries(emitted, cuda):
    """cairn_hotpath_device_stream(stream): the thread's synchronous device work runs on the caller's stream, after
    what the caller queued there (cairn_exec.hpp use_stream); NULL gives the thread its own stream back."""
    n = 8_000_003
    x_np, y_np, a = inputs.saxpy_case(n, seed=11)
    s = torch.cuda.Stream(cuda)
    x, y = _dev(x_np, cuda), _dev(y_np, cuda)
    out = torch.empty_like(x)
    torch.cuda.synchronize()
    emitted.cairn_hotpath_device_stream(s.cuda_stream)
    try:
        with torch.cuda.stream(s):
            x.mul_(1.0)  # queued on s ahead of the region, which reads x
            y.add_(0.0)
        emitted.cf_saxpy(n, out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    finally:
        emitted.cairn_hotpath_device_stream(None)
    assert np.array_equal(_bits(out), restated.saxpy(float(a), x_np, y_np).view(np.uint32))


# ---- collectors --------------------------------------------------------------------------------------------------
def test_emitted_reductions(emitted, cuda):
    rng = np.random.default_rng(4)
    for n in (1, 300, 2047, 2048, 2049, 1_000_003, 20_000_001):
        x_np = rng.uniform(-1, 1, n).astype(np.float32)
        got = emitted.cf_dsum(n, _dev(x_np, cuda).data_ptr())
        exact = float(restated.sum_f32(x_np))
        assert abs(got - exact) <= n * 2.0**-24 * float(np.abs(x_np.astype(np.float64)).sum()) + 1e-30, n
        u = np.arange(n, dtype=np.uint64)
        assert emitted.cf_usum(n, _dev(u.view(np.int64), cuda).data_ptr()) == n * (n - 1) // 2
        v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
        assert emitted.cf_vmax(n, _dev(v, cuda).data_ptr()) == int(v.max())


def test_emitted_reduction_into_device_memory(emitted, cuda):
    """`reduce + total[0] parallel ...` over device views: the total stays on the device (reduce_into)."""
    want = np.load(ROOT / "tests" / "golden" / "u64.npz")["iota_1e6/want"]  # the reference's total, and no overflow
    x = inputs.u64_cases()["iota_1e6"]
    total = torch.zeros(1, dtype=torch.int64, device=cuda)
    emitted.cf_usum_into(x.size, _dev(x.view(np.int64), cuda).data_ptr(), total.data_ptr())
    assert int(total.cpu().numpy().view(np.uint64)[0]) == int(want[0]) and int(want[1]) == 0


_OVERFLOW = r"""
import ctypes as C, sys
import numpy as np, torch
h = C.CDLL(sys.argv[1])
h.cf_usum.restype, h.cf_usum.argtypes = C.c_uint64, [C.c_size_t, C.c_void_p]
x = torch.from_numpy(np.array([1 << 63, 1 << 63, 5], np.uint64).view(np.int64)).cuda()
torch.cuda.synchronize()
print(h.cf_usum(3, x.data_ptr()), flush=True)
"""


def test_emitted_checked_sum_traps_on_the_host_when_it_overflows(emitted, cuda):
    """A checked unsigned `reduce +` whose total does not fit ends the process with the reference's trap (std::abort
    on the host, after the device work has finished: cr::Sum::checked, cairn_runtime.hpp:158-166). Run in a child."""
    done = subprocess.run([sys.executable, "-c", _OVERFLOW, str(LIB)], capture_output=True, text=True, timeout=300)
    assert done.returncode == -6, (done.returncode, done.stdout, done.stderr[-2000:])
    assert done.stdout.strip() == ""


SCAN_SIZES = [1, 31, 2048, 2049, 4096, 4097, 65 * 4096 + 7, 1_000_003]


@pytest.mark.parametrize("n", SCAN_SIZES)
def test_emitted_integer_scans(emitted, cuda, n):
    rng = np.random.default_rng(n)
    x = rng.integers(0, 1 << 40, n, dtype=np.uint64)
    out = torch.empty(n, dtype=torch.int64, device=cuda)
    total = emitted.cf_prefix(n, out.data_ptr(), _dev(x.view(np.int64), cuda).data_ptr())
    want = np.cumsum(x, dtype=np.uint64)
    assert np.array_equal(out.cpu().numpy().view(np.uint64), want) and total == int(want[-1])

    w = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    wout = torch.empty(n, dtype=torch.int32, device=cuda)
    wtotal = emitted.cf_wprefix(n, wout.data_ptr(), _dev(w.view(np.int32), cuda).data_ptr())
    wwant, wwant_total = restated.scan_u32(w)  # add_wrap: modulo 2^32
    assert np.array_equal(wout.cpu().numpy().view(np.uint32), wwant) and wtotal == wwant_total
    wout.zero_()
    emitted.cf_wscan(n, wout.data_ptr(), _dev(w.view(np.int32), cuda).data_ptr())  # no total: scan_into
    assert np.array_equal(wout.cpu().numpy().view(np.uint32), wwant)

    v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    vout = torch.empty(n, dtype=torch.int32, device=cuda)
    vtotal = emitted.cf_runmax(n, vout.data_ptr(), _dev(v, cuda).data_ptr())
    vwant, vwant_total = restated.runmax_i32(v)
    assert np.array_equal(vout.cpu().numpy(), vwant) and vtotal == vwant_total


def test_emitted_scans_against_the_reference_fixture(emitted, cuda):
    d = np.load(ROOT / "tests" / "golden" / "scan.npz")
    for n in sorted({int(k.split("/")[1]) for k in d.files}):
        x = d[f"u32/{n}/x"]
        out = torch.empty(n, dtype=torch.int32, device=cuda)
        total = emitted.cf_wprefix(n, out.data_ptr(), _dev(x.view(np.int32), cuda).data_ptr())
        assert np.array_equal(out.cpu().numpy().view(np.uint32), d[f"u32/{n}/want"])
        assert total == int(d[f"u32/{n}/total"][0])
        v = d[f"max/{n}/x"]
        vout = torch.empty(n, dtype=torch.int32, device=cuda)
        vtotal = emitted.cf_runmax(n, vout.data_ptr(), _dev(v, cuda).data_ptr())
        assert np.array_equal(vout.cpu().numpy(), d[f"max/{n}/want"]) and vtotal == int(d[f"max/{n}/total"][0])


@pytest.mark.parametrize("n", [1, 2, 4097, 1_000_003])
def test_emitted_compaction_keeps_order(emitted, cuda, n):
    x = np.random.default_rng(n + 2).standard_normal(n).astype(np.float32)
    out = torch.full((n,), -7.0, dtype=torch.float32, device=cuda)
    used = emitted.cf_positives(n, out.data_ptr(), _dev(x, cuda).data_ptr())
    keep = x[x > 0]
    got = out.cpu().numpy()
    assert used == keep.size
    assert np.array_equal(got[:used].view(np.uint32), keep.view(np.uint32))
    assert (got[used:] == -7.0).all()  # the tail of out is left alone


def test_machine_scan_many_look_back_windows_against_the_oracle(emitted, cuda):
    """2^27 u32 values: 8,192 tiles, so look-backs cross many 32-tile windows while others are still in flight."""
    n = 1 << 27
    x = np.random.default_rng(27).integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    want, total = restated.scan_u32(x)
    out = torch.empty(n, dtype=torch.int32, device=cuda)
    assert emitted.cf_wprefix(n, out.data_ptr(), _dev(x.view(np.int32), cuda).data_ptr()) == total
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want)


@pytest.mark.parametrize("n", [5000, 200_003])
def test_scan_look_back_escape_gives_the_same_prefixes(probe, cuda, n):
    """With no time to wait, every block that finds a predecessor unpublished folds the inputs before its tile
    itself: the answer is the same."""
    x = np.random.default_rng(n + 3).integers(0, 1 << 40, n, dtype=np.uint64)
    out = torch.empty(n, dtype=torch.int64, device=cuda)
    probe.cf_prefix_escape(n, out.data_ptr(), _dev(x.view(np.int64), cuda).data_ptr())
    assert np.array_equal(out.cpu().numpy().view(np.uint64), np.cumsum(x, dtype=np.uint64))


def test_the_machine_scan_kernel_alone(probe, cuda):
    n = 3 * 4096 * 37 + 11
    x = np.random.default_rng(5).integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    want, _ = restated.scan_u32(x)
    temp = torch.empty(probe.b200_scan_u32_scratch(n), dtype=torch.uint8, device=cuda)
    raw = torch.empty(n, dtype=torch.int32, device=cuda)
    probe.b200_scan_u32(torch.cuda.current_stream(cuda).cuda_stream, n, raw.data_ptr(),
                        _dev(x.view(np.int32), cuda).data_ptr(), temp.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(raw.cpu().numpy().view(np.uint32), want)


@pytest.mark.slow
def test_machine_scan_at_the_bench_size_by_differences(emitted, probe, cuda):
    """n = 2^30 (the bench's size): out[0] = x[0] and out[i] - out[i - 1] = x[i] modulo 2^32 at every i, checked on
    the device, through the emitted entry and the machine's kernel alone."""
    n = 1 << 30
    g = torch.Generator(device=cuda).manual_seed(30)
    x = torch.randint(-2**31, 2**31 - 1, (n,), device=cuda, dtype=torch.int32, generator=g)
    out = torch.empty_like(x)

    def holds() -> bool:
        ok = bool(out[0] == x[0])
        for lo in range(1, n, 1 << 28):  # int32 differences wrap like add_wrap's u32 sums
            hi = min(n, lo + (1 << 28))
            ok = ok and bool(((out[lo:hi] - out[lo - 1:hi - 1]) == x[lo:hi]).all())
        return ok

    emitted.cf_wscan(n, out.data_ptr(), x.data_ptr())
    assert holds()
    out.zero_()
    temp = torch.empty(probe.b200_scan_u32_scratch(n), dtype=torch.uint8, device=cuda)
    probe.b200_scan_u32(torch.cuda.current_stream(cuda).cuda_stream, n, out.data_ptr(), x.data_ptr(), temp.data_ptr())
    torch.cuda.synchronize()
    assert holds()


# ---- the multiply ------------------------------------------------------------------------------------------------
@pytest.mark.parametrize("fmt,entry", [("bf16", "cf_gemm"), ("f16", "cf_gemm_f16"), ("f8e4m3", "cf_gemm_e4m3")])
@pytest.mark.parametrize("shape", [(65, 63, 33), (256, 512, 1024), (300, 264, 136)])
def test_emitted_multiply_runs_the_tensor_cores(emitted, cuda, fmt, entry, shape):
    m, n, k = shape
    c, a, b = inputs.mma_case(fmt, m, n, k, seed=m)
    want = restated.mma(fmt, c, a, b, m, n, k)
    view = np.int16 if a.dtype.itemsize == 2 else np.int8
    ct, at, bt = _dev(c.copy(), cuda), _dev(a.view(view), cuda), _dev(b.view(view), cuda)
    getattr(emitted, entry)(m, n, k, m * n, ct.data_ptr(), m * k, at.data_ptr(), k * n, bt.data_ptr())
    av = np.abs(inputs.decode(fmt, a).reshape(m, k))
    bv = np.abs(inputs.decode(fmt, b).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(c.reshape(m, n)) + av @ bv)
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want.reshape(m, n)) <= tol).all()


def test_emitted_enqueued_multiply(emitted, cuda):
    m, n, k = 512, 768, 256
    c, a, b = inputs.mma_case("bf16", m, n, k, seed=3)
    want = restated.mma("bf16", c, a, b, m, n, k)
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        ct, at, bt = _dev(c.copy(), cuda), _dev(a.view(np.int16), cuda), _dev(b.view(np.int16), cuda)
        emitted.cq_gemm(s.cuda_stream, m, n, k, m * n, ct.data_ptr(), m * k, at.data_ptr(), k * n, bt.data_ptr())
    s.synchronize()
    av = np.abs(inputs.decode("bf16", a).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", b).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(c.reshape(m, n)) + av @ bv)
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want.reshape(m, n)) <= tol).all()


# ---- the same emitted program on the reference's own machine -------------------------------------------------------
# Runs in a process of its own (two builds of one program in one process would share their template symbols):
# argv = library, inputs .npz, outputs .npz. Every entry is the reference machine's (cairn_gpu.hpp, cairn_kernels.hpp,
# cairn_cub.hpp, cairn_tensor.hpp of the reference tree), reached through the program's cf_ entries.
_ON_REFERENCE_MACHINE = r"""
import ctypes as C, sys
import numpy as np, torch
h = C.CDLL(sys.argv[1])
z, p = C.c_size_t, C.c_void_p
for name, res, args in (("cf_saxpy", None, [z, p, p, p, C.c_float]), ("cf_saxpy4", None, [z, p, p, p, C.c_float]),
                        ("cf_blur", None, [z, p, p]), ("cf_usum", C.c_uint64, [z, p]),
                        ("cf_dsum", C.c_float, [z, p]), ("cf_wprefix", C.c_uint32, [z, p, p]),
                        ("cf_gemm", None, [z, z, z, z, p, z, p, z, p])):
    f = getattr(h, name)
    f.restype, f.argtypes = res, args
d = dict(np.load(sys.argv[2]))
dev = torch.device("cuda", 0)
g = lambda a: torch.from_numpy(a).to(dev)
x, y = g(d["x"]), g(d["y"])
out, out4, blur = torch.empty_like(x), torch.empty_like(x), torch.empty_like(x)
h.cf_saxpy(x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(d["a"][0]))
h.cf_saxpy4(x.numel(), out4.data_ptr(), x.data_ptr(), y.data_ptr(), float(d["a"][0]))
h.cf_blur(x.numel(), blur.data_ptr(), x.data_ptr())
u = g(d["u"].view(np.int64))
usum = h.cf_usum(u.numel(), u.data_ptr())
dsum = h.cf_dsum(x.numel(), x.data_ptr())
w = g(d["w"].view(np.int32))
wout = torch.empty_like(w)
wtotal = h.cf_wprefix(w.numel(), wout.data_ptr(), w.data_ptr())
m, n, k = (int(v) for v in d["mnk"])
a, b, c = g(d["ga"].view(np.int16)), g(d["gb"].view(np.int16)), g(d["gc"])
h.cf_gemm(m, n, k, m * n, c.data_ptr(), m * k, a.data_ptr(), k * n, b.data_ptr())
torch.cuda.synchronize()
np.savez(sys.argv[3], saxpy=out.cpu().numpy(), saxpy4=out4.cpu().numpy(), blur=blur.cpu().numpy(),
         usum=np.asarray([usum], np.uint64), dsum=np.asarray([dsum], np.float32),
         wprefix=wout.cpu().numpy().view(np.uint32), wtotal=np.asarray([wtotal], np.uint32), gemm=c.cpu().numpy())
"""


def test_the_program_on_the_reference_machine_agrees_with_the_b200_machine(emitted, cuda, tmp_path):
    """The emitted library built over the reference's headers alone (its lane kernels, CUB collectors and WMMA
    multiply, compiled for sm_100a) and over the drop-in headers: saxpy in both plans, the staged blur, the checked
    u64 sum and the add_wrap scan give the same bits on both machines and the oracle; the f32 `reduce +` lies within
    n * 2^-24 * sum |x| of the exact sum on both; the multiply within twice its contract bound on both."""
    if not REF_LIB.exists():
        pytest.skip("baseline/_ref/libhotpath_ref.so is not built (it needs the CAIRN reference's compiler)")
    rng = np.random.default_rng(77)
    x_np, y_np, a = inputs.saxpy_case((1 << 22) + 3, seed=5)
    u_np = np.arange(1_000_003, dtype=np.uint64)
    w_np = rng.integers(0, 2**32, 3_000_017, dtype=np.uint64).astype(np.uint32)
    m, n, k = 256, 512, 1024
    ga = inputs.encode("bf16", rng.standard_normal(m * k))
    gb = inputs.encode("bf16", rng.standard_normal(k * n))
    gc = rng.uniform(-2, 2, m * n).astype(np.float32)
    src = tmp_path / "in.npz"
    np.savez(src, x=x_np, y=y_np, a=np.asarray([a], np.float32), u=u_np, w=w_np, mnk=np.asarray([m, n, k]), ga=ga,
             gb=gb, gc=gc)
    dst = tmp_path / "out.npz"
    done = subprocess.run([sys.executable, "-c", _ON_REFERENCE_MACHINE, str(REF_LIB), str(src), str(dst)],
                          capture_output=True, text=True, timeout=600)
    assert done.returncode == 0, done.stderr[-3000:]
    ref = np.load(dst)

    x, y = _dev(x_np, cuda), _dev(y_np, cuda)
    want = restated.saxpy(float(a), x_np, y_np).view(np.uint32)
    for entry in ("cf_saxpy", "cf_saxpy4"):
        out = torch.empty_like(x)
        getattr(emitted, entry)(x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
        assert np.array_equal(ref[entry[3:]].view(np.uint32), want)
        assert np.array_equal(_bits(out), want)
    blur = torch.empty_like(x)
    emitted.cf_blur(x.numel(), blur.data_ptr(), x.data_ptr())
    assert np.array_equal(ref["blur"].view(np.uint32), _blur(x_np).view(np.uint32))
    assert np.array_equal(_bits(blur), _blur(x_np).view(np.uint32))

    u = _dev(u_np.view(np.int64), cuda)
    assert int(ref["usum"][0]) == emitted.cf_usum(u.numel(), u.data_ptr()) == u_np.size * (u_np.size - 1) // 2

    exact = float(restated.sum_f32(x_np))
    bound = x_np.size * 2.0**-24 * float(np.abs(x_np.astype(np.float64)).sum())
    assert abs(float(ref["dsum"][0]) - exact) <= bound
    assert abs(emitted.cf_dsum(x.numel(), x.data_ptr()) - exact) <= bound

    w = _dev(w_np.view(np.int32), cuda)
    wout = torch.empty_like(w)
    total = emitted.cf_wprefix(w.numel(), wout.data_ptr(), w.data_ptr())
    want_scan, want_total = restated.scan_u32(w_np)
    assert np.array_equal(ref["wprefix"], want_scan) and int(ref["wtotal"][0]) == want_total
    assert np.array_equal(wout.cpu().numpy().view(np.uint32), want_scan) and total == want_total

    ct, at, bt = _dev(gc.copy(), cuda), _dev(ga.view(np.int16), cuda), _dev(gb.view(np.int16), cuda)
    emitted.cf_gemm(m, n, k, m * n, ct.data_ptr(), m * k, at.data_ptr(), k * n, bt.data_ptr())
    want_c = restated.mma("bf16", gc, ga, gb, m, n, k).reshape(m, n)
    av = np.abs(inputs.decode("bf16", ga).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", gb).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(gc.reshape(m, n)) + av @ bv)
    assert (np.abs(ref["gemm"].reshape(m, n) - want_c) <= tol).all()
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want_c) <= tol).all()


def test_emitted_entries_from_several_host_threads_at_once(emitted, cuda):
    """Four host threads call the emitted entries at once, twenty rounds each (ctypes lets go of the interpreter lock
    for the call): every thread has the reference's thread-local context over this machine, with its own stream
    and arena, while the machine's per-device state (the memory pool, the SM count, the resident-grid memos) is
    shared. Every result is still the oracle's."""
    import threading

    n = 1_000_003
    cases = []
    for t in range(4):
        x_np, y_np, a = inputs.saxpy_case(n, seed=100 + t)
        w = np.random.default_rng(200 + t).integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
        u = np.random.default_rng(300 + t).integers(0, 1 << 40, n, dtype=np.uint64)
        cases.append(dict(x=_dev(x_np, cuda), y=_dev(y_np, cuda), a=float(a), w=_dev(w.view(np.int32), cuda),
                          u=_dev(u.view(np.int64), cuda), out=torch.empty(n, dtype=torch.float32, device=cuda),
                          wout=torch.empty(n, dtype=torch.int32, device=cuda),
                          saxpy=restated.saxpy(float(a), x_np, y_np).view(np.uint32),
                          scan=restated.scan_u32(w), usum=int(u.sum(dtype=np.uint64))))
    torch.cuda.synchronize()
    failures: list[str] = []

    def work(t: int):
        c = cases[t]
        try:
            for r in range(20):
                emitted.cf_saxpy4(n, c["out"].data_ptr(), c["x"].data_ptr(), c["y"].data_ptr(), c["a"])
                total = emitted.cf_wprefix(n, c["wout"].data_ptr(), c["w"].data_ptr())
                usum = emitted.cf_usum(n, c["u"].data_ptr())
                if total != c["scan"][1] or usum != c["usum"]:
                    failures.append(f"thread {t} round {r}: totals {total} {usum}")
        except Exception as e:  # noqa: BLE001 - reported below
            failures.append(f"thread {t}: {e!r}")

    threads = [threading.Thread(target=work, args=(t,)) for t in range(4)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=300)
    assert not any(th.is_alive() for th in threads)
    assert not failures, failures[:4]
    torch.cuda.synchronize()
    for c in cases:
        assert np.array_equal(_bits(c["out"]), c["saxpy"])
        assert np.array_equal(c["wout"].cpu().numpy().view(np.uint32), c["scan"][0])


# ---- the enqueued entries inside a CUDA graph ----------------------------------------------------------------------
# argv = repository root, library, inputs .npz, outputs .npz. A process of its own: a capture that failed would end in
# the reference's trap (std::abort on the host), not in an exception.
_IN_A_GRAPH = r"""
import ctypes as C, sys
import numpy as np, torch
sys.path[:0] = [sys.argv[1]]
import cairn_b200
cairn_b200.lib()
h = C.CDLL(sys.argv[2])
z, p, f = C.c_size_t, C.c_void_p, C.c_float
h.cq_saxpy4.restype, h.cq_saxpy4.argtypes = None, [p, z, p, p, p, f]
h.cq_blur.restype, h.cq_blur.argtypes = None, [p, z, p, p]
h.cq_gemm.restype, h.cq_gemm.argtypes = None, [p, z, z, z, z, p, z, p, z, p]
d = dict(np.load(sys.argv[3]))
dev = torch.device("cuda", 0)
g = lambda v: torch.from_numpy(v).to(dev)
x, y, a = g(d["x"]), g(d["y"]), float(d["a"][0])
n = x.numel()
m, nn, k = (int(v) for v in d["mnk"])
ga, gb = g(d["ga"].view(np.int16)), g(d["gb"].view(np.int16))
out4, blur = torch.empty_like(x), torch.empty_like(x)
once, twice = torch.zeros(m * nn, device=dev), torch.zeros(m * nn, device=dev)
s = torch.cuda.Stream(dev)
torch.cuda.synchronize()
def enqueue(c):
    h.cq_saxpy4(s.cuda_stream, n, out4.data_ptr(), x.data_ptr(), y.data_ptr(), a)
    h.cq_blur(s.cuda_stream, n, blur.data_ptr(), x.data_ptr())
    h.cq_gemm(s.cuda_stream, m, nn, k, m * nn, c.data_ptr(), m * k, ga.data_ptr(), k * nn, gb.data_ptr())
with torch.cuda.stream(s):
    enqueue(once)  # outside a capture first: the machine sizes its grids and the multiply configures its kernel
s.synchronize()
graph = torch.cuda.CUDAGraph()
with torch.cuda.graph(graph, stream=s):
    enqueue(twice)
out4.zero_(); blur.zero_(); twice.zero_()
torch.cuda.synchronize()
graph.replay()
graph.replay()  # C += A B twice: every element is twice the single product, exactly
torch.cuda.synchronize()
np.savez(sys.argv[4], saxpy4=out4.cpu().numpy(), blur=blur.cpu().numpy(), once=once.cpu().numpy(),
         twice=twice.cpu().numpy())
"""


def test_the_enqueued_entries_run_inside_a_cuda_graph(emitted, cuda, tmp_path):
    """cq_saxpy4 (a vector region), cq_blur (a staged region) and cq_gemm (`mma_unordered` over the B200 multiply)
    captured in one CUDA graph on the caller's stream after one call outside it, as the header says an enqueued
    entry may be (it makes no stream, event or allocation): the graph replays to the oracle's saxpy and blur bits,
    and two replays of C += A B give exactly twice one call's product."""
    n = 1_000_003
    x, y, a = inputs.saxpy_case(n, seed=77)
    m, nn, k = 512, 768, 256
    _, ga, gb = inputs.mma_case("bf16", m, nn, k, seed=8)
    src, dst = tmp_path / "in.npz", tmp_path / "out.npz"
    np.savez(src, x=x, y=y, a=np.asarray([a], np.float32), ga=ga, gb=gb, mnk=np.asarray([m, nn, k]))
    done = subprocess.run([sys.executable, "-c", _IN_A_GRAPH, str(ROOT), str(LIB), str(src), str(dst)],
                          capture_output=True, text=True, timeout=600)
    assert done.returncode == 0, (done.returncode, done.stderr[-3000:])
    got = np.load(dst)
    assert np.array_equal(got["saxpy4"].view(np.uint32), restated.saxpy(float(a), x, y).view(np.uint32))
    assert np.array_equal(got["blur"].view(np.uint32), _blur(x).view(np.uint32))
    assert np.array_equal(got["twice"], got["once"] * np.float32(2))
    want = restated.mma("bf16", np.zeros(m * nn, np.float32), ga, gb, m, nn, k)
    av = np.abs(inputs.decode("bf16", ga).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", gb).reshape(k, nn))
    tol = 2 * (k + 1) * 2.0**-22 * (av @ bv)
    assert (np.abs(got["once"].reshape(m, nn) - want.reshape(m, nn)) <= tol).all()
