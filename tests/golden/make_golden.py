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


def main() -> None:
    if not reference.available():
        raise SystemExit("oracle/_ref/libcairn_ref.so is not built: make -C oracle REF=<cairn>/src/cairn/runtime")
    for name, fn in (("mma", mma), ("sum", sums), ("u64", u64), ("saxpy", saxpy), ("f32gemm", f32gemm)):
        np.savez_compressed(HERE / f"{name}.npz", **fn())
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
