"""Writes tests/golden/*.npz: inputs and the outputs of the CAIRN reference's own host path on them.

Run where the reference's host path is built (oracle/_ref/libcairn_ref.so, compiled from the reference's runtime
headers by oracle/Makefile):  python tests/golden/make_golden.py

The fixtures pin oracle/cairn_oracle.c (tests/test_oracle.py) on machines that have no reference tree, such as the
GPU box, and give the GPU parity tests the reference's own answers for the cases of its tests:
  mma.npz    cr::tensor::multiply<A> (runtime/cairn_tensor.hpp:37-41) on the shapes of tests/soundness/test_tensor.py
             and tests/runtime/tensor_runtime.cpp, every storage format, random finite patterns and the tile test's
             1/16 grid
  sum.npz    cr::par::sum<float> (runtime/cairn_sum.hpp:311-331) on rounding-boundary, special-value and random cases
  u64.npz    cr::par::reduce over cr::Sum<u64> on tests/inputs.py's u64_cases: data[i] = i for n = 1e6 (BASELINE
             config 1) and overflow cases
  saxpy.npz  cr::par::run of out = a * x + y
  f32gemm.npz  the `parallel e in m*n` f32 GEMM region of BASELINE config 1, at a reduced size
  scan.npz   cr::par::scan: inclusive add_wrap over u32 and exclusive max over i32, on sizes around the device
             scan's tiles (4096 four-byte elements) and with wrapping totals
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import inputs  # noqa: E402
from oracle import reference  # noqa: E402

HERE = Path(__file__).resolve().parent


def mma() -> dict:
    out = {}
    for fmt in inputs.FORMATS:
        for idx, (m, n, k) in enumerate(inputs.MMA_SHAPES):
            c, a, b = inputs.mma_case(fmt, m, n, k, seed=1000 + idx)
            key = f"{fmt}/rand/{m}x{n}x{k}"
            out[key + "/c"], out[key + "/a"], out[key + "/b"] = c, a, b
            out[key + "/want"] = reference.mma(fmt, c, a, b, m, n, k)
        for m, n, k in inputs.TILE_SHAPES:
            c, a, b = inputs.tile_case(fmt, m, n, k)
            key = f"{fmt}/tile/{m}x{n}x{k}"
            out[key + "/c"], out[key + "/a"], out[key + "/b"] = c, a, b
            out[key + "/want"] = reference.mma(fmt, c, a, b, m, n, k)
    return out


def sums() -> dict:
    out = {}
    for i, (name, terms) in enumerate([*inputs.sum_boundary_cases(), *inputs.sum_random_cases()]):
        x = np.asarray([inputs.f32(t) for t in terms] if isinstance(terms, list) else terms, np.float32)
        out[f"{i:03d}/x"] = x
        out[f"{i:03d}/want"] = np.asarray([reference.sum_f32(x)], np.float32).view(np.uint32)
        out[f"{i:03d}/name"] = np.asarray(name)
    return out


def u64() -> dict:
    out = {}
    for name, x in inputs.u64_cases().items():
        v, over = reference.sum_u64(x)
        out[f"{name}/want"] = np.asarray([v, int(over)], np.uint64)
    return out


def saxpy() -> dict:
    x, y, a = inputs.saxpy_case(20_003, seed=3)
    return {"x": x, "y": y, "a": np.asarray([a], np.float32), "want": reference.saxpy(float(a), x, y)}


def f32gemm() -> dict:
    rng = np.random.default_rng(0)
    m = n = k = 96
    a = rng.uniform(-1, 1, m * k).astype(np.float32)
    b = rng.uniform(-1, 1, k * n).astype(np.float32)
    c = np.zeros(m * n, np.float32)
    return {"a": a, "b": b, "shape": np.asarray([m, n, k]), "want": reference.gemm_f32_region(c, a, b, m, n, k)}


SCAN_SIZES = (1, 2, 4095, 4096, 4097, 8193)


def scan() -> dict:
    out = {}
    for n in SCAN_SIZES:
        rng = np.random.default_rng(n)
        x = rng.integers(0, 1 << 32, n, dtype=np.uint64).astype(np.uint32)
        got, total = reference.scan_u32(x)
        out[f"u32/{n}/x"], out[f"u32/{n}/want"], out[f"u32/{n}/total"] = x, got, np.asarray([total], np.uint32)
        v = rng.integers(-2**31, 2**31 - 1, n, dtype=np.int64).astype(np.int32)
        got, total = reference.runmax_i32(v)
        out[f"max/{n}/x"], out[f"max/{n}/want"], out[f"max/{n}/total"] = v, got, np.asarray([total], np.int32)
    return out


def main() -> None:
    if not reference.available():
        raise SystemExit("oracle/_ref/libcairn_ref.so is not built: make -C oracle REF=<cairn>/src/cairn/runtime")
    for name, fn in (("mma", mma), ("sum", sums), ("u64", u64), ("saxpy", saxpy), ("f32gemm", f32gemm),
                     ("scan", scan)):
        np.savez_compressed(HERE / f"{name}.npz", **fn())
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
