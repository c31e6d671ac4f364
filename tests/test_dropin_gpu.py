"""The drop-in runtime headers (include/cairn_b200/runtime) under a program written the way cairnc emits one
(tests/dropin/emitted_program.cu): the reference's own cairn_exec.hpp and cairn_reuse.hpp, unchanged, run the B200
machine, whose regions, collectors and multiply are this project's. Each cf_/cq_ entry is held to the oracle: saxpy
and the u64 sum bit for bit, the f32 `reduce +` (the device path's f32 fold in an unspecified order,
docs/numerics.md) within n * 2^-24 * sum |x|, the multiply within twice its contract bound. The scans and the
compaction (cairn_reuse.hpp:430-524 over the machine's own single-pass scan, not CUB's): integer scans and the
compaction bit for bit, the f32 scan within i * 2^-24 * sum |x[0..i]| at each i; sizes around the scan's tiles
(4096 four-byte or 2048 eight-byte elements) and its 32-tile look-back window.

The program is built by __graft_entry__.build() where the CAIRN reference tree is present; without the built
library these tests are skipped, naming why."""

from __future__ import annotations

import ctypes as C
from pathlib import Path

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu
LIB = Path(__file__).resolve().parent / "dropin" / "_build" / "libemitted.so"


@pytest.fixture(scope="module")
def emitted(cuda):
    if not LIB.exists():
        pytest.skip("tests/dropin/_build/libemitted.so is not built (it needs the CAIRN reference's headers)")
    cairn_b200.lib()  # the program links libcairn_b200.so: load it from the tree first
    h = C.CDLL(str(LIB))
    z, p = C.c_size_t, C.c_void_p
    for name, res, args in (("cf_saxpy", None, [z, p, p, p, C.c_float]), ("cf_saxpy4", None, [z, p, p, p, C.c_float]),
                            ("cq_saxpy", None, [p, z, p, p, p, C.c_float]), ("cf_dsum", C.c_float, [z, p]),
                            ("cf_usum", C.c_uint64, [z, p]), ("cf_vmax", C.c_int32, [z, p]),
                            ("cf_gemm", None, [z, z, z, z, p, z, p, z, p]), ("cf_prefix", C.c_uint64, [z, p, p]),
                            ("cf_wprefix", C.c_uint32, [z, p, p]), ("cf_runmax", C.c_int32, [z, p, p]),
                            ("cf_fprefix", C.c_float, [z, p, p]), ("cf_positives", C.c_size_t, [z, p, p]),
                            ("cf_prefix_escape", None, [z, p, p]), ("cf_blur", None, [z, p, p]),
                            ("cq_wscan", None, [p, z, p, p]), ("b200_scan_u32_scratch", z, [z]),
                            ("b200_scan_u32", None, [p, z, p, p, p])):
        f = getattr(h, name)
        f.restype, f.argtypes = res, args
    return h


@pytest.mark.parametrize("entry", ["cf_saxpy", "cf_saxpy4"])
@pytest.mark.parametrize("n", [1, 1023, (1 << 22) + 3])
def test_emitted_saxpy_regions(emitted, cuda, entry, n):
    x_np, y_np, a = inputs.saxpy_case(n, seed=n)
    x, y = torch.from_numpy(x_np).to(cuda), torch.from_numpy(y_np).to(cuda)
    out = torch.empty_like(x)
    getattr(emitted, entry)(n, out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    assert np.array_equal(out.cpu().numpy().view(np.uint32), restated.saxpy(float(a), x_np, y_np).view(np.uint32))


def test_emitted_enqueued_saxpy_on_the_callers_stream(emitted, cuda):
    x_np, y_np, a = inputs.saxpy_case(100_000, seed=2)
    x, y = torch.from_numpy(x_np).to(cuda), torch.from_numpy(y_np).to(cuda)
    out = torch.empty_like(x)
    s = torch.cuda.Stream(cuda)
    with torch.cuda.stream(s):
        emitted.cq_saxpy(s.cuda_stream, x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    s.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), restated.saxpy(float(a), x_np, y_np).view(np.uint32))


def test_emitted_reductions(emitted, cuda):
    rng = np.random.default_rng(4)
    for n in (1, 300, 1_000_003):
        x_np = rng.uniform(-1, 1, n).astype(np.float32)
        got = emitted.cf_dsum(n, torch.from_numpy(x_np).to(cuda).data_ptr())
        exact = float(restated.sum_f32(x_np))
        assert abs(got - exact) <= n * 2.0**-24 * float(np.abs(x_np).sum()) + 1e-30
        u = np.arange(n, dtype=np.uint64)
        assert emitted.cf_usum(n, torch.from_numpy(u.view(np.int64)).to(cuda).data_ptr()) == n * (n - 1) // 2
        v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
        assert emitted.cf_vmax(n, torch.from_numpy(v).to(cuda).data_ptr()) == int(v.max())


@pytest.mark.parametrize("shape", [(65, 63, 33), (256, 512, 1024), (300, 264, 136)])
def test_emitted_multiply_runs_the_tensor_cores(emitted, cuda, shape):
    m, n, k = shape
    c, a, b = inputs.mma_case("bf16", m, n, k, seed=m)
    want = restated.mma("bf16", c, a, b, m, n, k)
    ct = torch.from_numpy(c.copy()).to(cuda)
    at = torch.from_numpy(a.view(np.int16).copy()).to(cuda)
    bt = torch.from_numpy(b.view(np.int16).copy()).to(cuda)
    emitted.cf_gemm(m, n, k, m * n, ct.data_ptr(), m * k, at.data_ptr(), k * n, bt.data_ptr())
    av = np.abs(inputs.decode("bf16", a).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", b).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(c.reshape(m, n)) + av @ bv)
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want.reshape(m, n)) <= tol).all()


SCAN_SIZES = [1, 31, 2048, 2049, 4096, 4097, 65 * 4096 + 7, 1_000_003]


def _dev(a: np.ndarray, cuda) -> torch.Tensor:
    return torch.from_numpy(a).to(cuda)


@pytest.mark.parametrize("n", SCAN_SIZES)
def test_emitted_integer_scans(emitted, cuda, n):
    rng = np.random.default_rng(n)
    x = rng.integers(0, 1 << 40, n, dtype=np.uint64)
    xt, out = _dev(x.view(np.int64), cuda), torch.empty(n, dtype=torch.int64, device=cuda)
    total = emitted.cf_prefix(n, out.data_ptr(), xt.data_ptr())
    want = np.cumsum(x, dtype=np.uint64)
    assert np.array_equal(out.cpu().numpy().view(np.uint64), want) and total == int(want[-1])

    w = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    wt, wout = _dev(w.view(np.int32), cuda), torch.empty(n, dtype=torch.int32, device=cuda)
    wtotal = emitted.cf_wprefix(n, wout.data_ptr(), wt.data_ptr())
    wwant, wwant_total = restated.scan_u32(w)  # add_wrap: modulo 2^32
    assert np.array_equal(wout.cpu().numpy().view(np.uint32), wwant) and wtotal == wwant_total

    v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
    vt, vout = _dev(v, cuda), torch.empty(n, dtype=torch.int32, device=cuda)
    vtotal = emitted.cf_runmax(n, vout.data_ptr(), vt.data_ptr())
    vwant, vwant_total = restated.runmax_i32(v)
    assert np.array_equal(vout.cpu().numpy(), vwant) and vtotal == vwant_total


def test_emitted_scans_against_the_reference_fixture(emitted, cuda):
    d = np.load(Path(__file__).resolve().parent / "golden" / "scan.npz")
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


def test_enqueued_scan_and_the_machine_kernel_alone(emitted, cuda):
    """cq_wscan (scan_into on the caller's stream) and the machine's scan kernel called directly give the oracle's
    prefixes."""
    n = 3 * 4096 * 37 + 11
    x = np.random.default_rng(5).integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    want, _ = restated.scan_u32(x)
    xt = _dev(x.view(np.int32), cuda)
    s = torch.cuda.Stream(cuda)
    out = torch.empty(n, dtype=torch.int32, device=cuda)
    with torch.cuda.stream(s):
        emitted.cq_wscan(s.cuda_stream, n, out.data_ptr(), xt.data_ptr())
    s.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want)
    temp = torch.empty(emitted.b200_scan_u32_scratch(n), dtype=torch.uint8, device=cuda)
    raw = torch.empty(n, dtype=torch.int32, device=cuda)
    emitted.b200_scan_u32(torch.cuda.current_stream(cuda).cuda_stream, n, raw.data_ptr(), xt.data_ptr(),
                          temp.data_ptr())
    torch.cuda.synchronize()
    assert np.array_equal(raw.cpu().numpy().view(np.uint32), want)


@pytest.mark.parametrize("n", [1, 4097, 1_000_003])
def test_emitted_f32_scan(emitted, cuda, n):
    x = np.random.default_rng(n + 1).uniform(-1, 1, n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    total = emitted.cf_fprefix(n, out.data_ptr(), _dev(x, cuda).data_ptr())
    got = out.cpu().numpy().astype(np.float64)
    exact = np.cumsum(x.astype(np.float64))
    idx = np.arange(1, n + 1)
    tol = idx * 2.0**-24 * np.cumsum(np.abs(x).astype(np.float64)) + 1e-30
    assert (np.abs(got - exact) <= tol).all()
    assert total == np.float32(got[-1])


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


@pytest.mark.parametrize("n", [5000, 200_003])
def test_scan_look_back_escape_gives_the_same_prefixes(emitted, cuda, n):
    """With no time to wait, every block that finds a predecessor unpublished folds the inputs before its tile
    itself: the answer is the same."""
    x = np.random.default_rng(n + 3).integers(0, 1 << 40, n, dtype=np.uint64)
    out = torch.empty(n, dtype=torch.int64, device=cuda)
    emitted.cf_prefix_escape(n, out.data_ptr(), _dev(x.view(np.int64), cuda).data_ptr())
    assert np.array_equal(out.cpu().numpy().view(np.uint64), np.cumsum(x, dtype=np.uint64))


@pytest.mark.parametrize("n", [1, 4, 5, 127, 128, 129, 131, 100_003])
def test_emitted_staged_region(emitted, cuda, n):
    """`plan blur { stage 2; block 128; }`: every tile a block loads holds what its lanes read, at the array's edges
    and between blocks; the body's f32 arithmetic in source order (--fmad=false), bit for bit."""
    x = np.random.default_rng(n + 4).uniform(-1, 1, n).astype(np.float32)
    out = torch.empty(n, dtype=torch.float32, device=cuda)
    emitted.cf_blur(n, out.data_ptr(), _dev(x, cuda).data_ptr())
    want = x.copy()
    if n >= 5:
        two, three = np.float32(2.0), np.float32(3.0)
        mid = x[:-4] + x[1:-3] * two
        mid = mid + x[2:-2] * three
        mid = mid + x[3:-1]
        want[2:-2] = mid + x[4:]
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_machine_scan_many_look_back_windows_against_the_oracle(emitted, cuda):
    """2^27 u32 values: 8,192 tiles, so look-backs cross many 128-tile windows while others are still in flight."""
    n = 1 << 27
    x = np.random.default_rng(27).integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
    want, total = restated.scan_u32(x)
    out = torch.empty(n, dtype=torch.int32, device=cuda)
    got_total = emitted.cf_wprefix(n, out.data_ptr(), _dev(x.view(np.int32), cuda).data_ptr())
    assert got_total == total
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want)


@pytest.mark.slow
def test_machine_scan_at_the_bench_size_by_differences(emitted, cuda):
    """n = 2^30 (the bench's size): out[0] = x[0] and out[i] - out[i - 1] = x[i] modulo 2^32 at every i, checked on
    the device, through both the enqueued entry and the machine's kernel alone."""
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

    emitted.cq_wscan(torch.cuda.current_stream(cuda).cuda_stream, n, out.data_ptr(), x.data_ptr())
    torch.cuda.synchronize()
    assert holds()
    out.zero_()
    temp = torch.empty(emitted.b200_scan_u32_scratch(n), dtype=torch.uint8, device=cuda)
    emitted.b200_scan_u32(torch.cuda.current_stream(cuda).cuda_stream, n, out.data_ptr(), x.data_ptr(), temp.data_ptr())
    torch.cuda.synchronize()
    assert holds()


# ---- the same program on the reference's own machine ----------------------------------------------------------------
REF_DEVICE = Path(__file__).resolve().parents[1] / "baseline" / "_ref" / "libemitted_ref.so"

# Runs in a process of its own (two builds of one program in one process would share their template symbols):
# argv = library, inputs .npz, outputs .npz. Every entry is the reference machine's (cairn_gpu.hpp, cairn_kernels.hpp,
# cairn_cub.hpp, cairn_tensor.hpp of the reference tree), reached through the program's cf_ entries.
_ON_REFERENCE_MACHINE = r"""
import ctypes as C, sys
import numpy as np, torch
h = C.CDLL(sys.argv[1])
z, p = C.c_size_t, C.c_void_p
for name, res, args in (("cf_saxpy", None, [z, p, p, p, C.c_float]), ("cf_usum", C.c_uint64, [z, p]),
                        ("cf_dsum", C.c_float, [z, p]), ("cf_wprefix", C.c_uint32, [z, p, p]),
                        ("cf_gemm", None, [z, z, z, z, p, z, p, z, p])):
    f = getattr(h, name)
    f.restype, f.argtypes = res, args
d = dict(np.load(sys.argv[2]))
dev = torch.device("cuda", 0)
g = lambda a: torch.from_numpy(a).to(dev)
x, y = g(d["x"]), g(d["y"])
out = torch.empty_like(x)
h.cf_saxpy(x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(d["a"][0]))
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
np.savez(sys.argv[3], saxpy=out.cpu().numpy(), usum=np.asarray([usum], np.uint64),
         dsum=np.asarray([dsum], np.float32), wprefix=wout.cpu().numpy().view(np.uint32),
         wtotal=np.asarray([wtotal], np.uint32), gemm=c.cpu().numpy())
"""


def test_the_program_on_the_reference_machine_agrees_with_the_b200_machine(emitted, cuda, tmp_path):
    """The emitted program built over the reference's headers alone (the reference's lane kernels, CUB collectors
    and WMMA multiply, compiled for sm_100a) and over the drop-in headers: saxpy, the checked u64 sum and the
    add_wrap scan give the same bits on both machines and the oracle; the f32 `reduce +` lies within
    n * 2^-24 * sum |x| of the exact sum on both (the device fold's order is unspecified, docs/numerics.md); the
    multiply within twice its contract bound on both."""
    import subprocess
    import sys

    if not REF_DEVICE.exists():
        pytest.skip("baseline/_ref/libemitted_ref.so is not built (it needs the CAIRN reference's headers)")
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
    done = subprocess.run([sys.executable, "-c", _ON_REFERENCE_MACHINE, str(REF_DEVICE), str(src), str(dst)],
                          capture_output=True, text=True, timeout=600)
    assert done.returncode == 0, done.stderr[-3000:]
    ref = np.load(dst)

    # this project's machine, the same entries
    x, y = torch.from_numpy(x_np).to(cuda), torch.from_numpy(y_np).to(cuda)
    out = torch.empty_like(x)
    emitted.cf_saxpy(x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a))
    want = restated.saxpy(float(a), x_np, y_np).view(np.uint32)
    assert np.array_equal(ref["saxpy"].view(np.uint32), want)
    assert np.array_equal(out.cpu().numpy().view(np.uint32), want)

    u = torch.from_numpy(u_np.view(np.int64)).to(cuda)
    assert int(ref["usum"][0]) == emitted.cf_usum(u.numel(), u.data_ptr()) == u_np.size * (u_np.size - 1) // 2

    exact = float(restated.sum_f32(x_np))
    bound = x_np.size * 2.0**-24 * float(np.abs(x_np.astype(np.float64)).sum())
    assert abs(float(ref["dsum"][0]) - exact) <= bound
    assert abs(emitted.cf_dsum(x.numel(), x.data_ptr()) - exact) <= bound

    w = torch.from_numpy(w_np.view(np.int32)).to(cuda)
    wout = torch.empty_like(w)
    total = emitted.cf_wprefix(w.numel(), wout.data_ptr(), w.data_ptr())
    want_scan, want_total = restated.scan_u32(w_np)
    assert np.array_equal(ref["wprefix"], want_scan) and int(ref["wtotal"][0]) == want_total
    assert np.array_equal(wout.cpu().numpy().view(np.uint32), want_scan) and total == want_total

    ct = torch.from_numpy(gc.copy()).to(cuda)
    at = torch.from_numpy(ga.view(np.int16).copy()).to(cuda)
    bt = torch.from_numpy(gb.view(np.int16).copy()).to(cuda)
    emitted.cf_gemm(m, n, k, m * n, ct.data_ptr(), m * k, at.data_ptr(), k * n, bt.data_ptr())
    want_c = restated.mma("bf16", gc, ga, gb, m, n, k).reshape(m, n)
    av = np.abs(inputs.decode("bf16", ga).reshape(m, k))
    bv = np.abs(inputs.decode("bf16", gb).reshape(k, n))
    tol = 2 * (k + 1) * 2.0**-22 * (np.abs(gc.reshape(m, n)) + av @ bv)
    assert (np.abs(ref["gemm"].reshape(m, n) - want_c) <= tol).all()
    assert (np.abs(ct.cpu().numpy().reshape(m, n) - want_c) <= tol).all()
