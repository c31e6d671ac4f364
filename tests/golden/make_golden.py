"""Writes tests/golden/*.npz: inputs and the outputs of the CAIRN reference's own host path on them.

Run where the reference's host path is built (oracle/_ref, by oracle.build with the CAIRN reference checkout):
    python tests/golden/make_golden.py [NAME ...]        (every fixture, or the named ones)

The fixtures pin oracle/cairn_oracle.c (tests/test_oracle.py) on machines that have no reference tree, such as the
GPU box, and give the GPU parity tests the reference's own answers for the cases of its tests:
  mma.npz    cr::tensor::multiply<A> (runtime/cairn_tensor.hpp:37-41) on the shapes of tests/soundness/test_tensor.py
             and tests/runtime/tensor_runtime.cpp, every storage format, random finite patterns and the tile test's
             1/16 grid
  sum.npz    cr::par::sum<float> (runtime/cairn_sum.hpp:311-331) on rounding-boundary, special-value and random cases
  u64.npz    cr::par::reduce over cr::Sum<u64> on tests/inputs.py's u64_cases: data[i] = i for n = 1e6 (BASELINE
             config 1) and overflow cases
  saxpy.npz  cr::par::run of out = a * x + y
  f32gemm.npz  the `parallel e in m*n` f32 GEMM region of BASELINE config 1 at its size, M = N = K = 512, with
             A then B drawn U[-1, 1] from numpy's default_rng(0) (the test draws them again; the first values are
             kept to show the stream has not changed); a 96^3 case with its inputs stored
  scan.npz   cr::par::scan: inclusive add_wrap over u32 and exclusive max over i32, on sizes around the device
             scan's tiles (4096 four-byte elements) and with wrapping totals
  mlp_grad.npz  BASELINE config 3's step at a reduced shape (batch 32, 128 -> 512 -> 128) from the reference's own
             code: oracle/grad/mlp_grad.cairn built by the reference's compiler (its dense layer and the adjoints
             `derive grad` writes for it, relu and mse with theirs; oracle/_ref/libmlp_grad.so), chained as a CAIRN
             program would chain them, with cr::fp::narrow to bf16 where the step stores bf16 (H, dY, dH)
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
    out = {"a": a, "b": b, "shape": np.asarray([m, n, k]), "want": reference.gemm_f32_region(c, a, b, m, n, k)}
    a512, b512 = inputs.config1_gemm()
    out["512/want"] = reference.gemm_f32_region(np.zeros(512 * 512, np.float32), a512, b512, 512, 512, 512)
    out["512/first"] = np.concatenate([a512[:4], b512[:4]])
    return out


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


def mlp_grad() -> dict:
    B, D, H, O = inputs.MLP_GOLDEN_SHAPE
    x, w1, w2, t = inputs.mlp_case(B, D, H, O, seed=33)
    out = {"x": x, "w1": w1, "w2": w2, "t": t, "shape": np.asarray([B, D, H, O])}
    for key, v in reference.mlp_step(x, w1, w2, t, B, D, H, O).items():
        out[f"want/{key}"] = v
    return out


def main() -> None:
    if not reference.available() or not reference.grad_available():
        raise SystemExit("oracle/_ref is not built: CAIRN_REFERENCE=<cairn checkout> python -c "
                         "'import __graft_entry__ as g; g.build()'")
    only = set(sys.argv[1:])
    for name, fn in (("mma", mma), ("sum", sums), ("u64", u64), ("saxpy", saxpy), ("f32gemm", f32gemm),
                     ("scan", scan), ("mlp_grad", mlp_grad)):
        if only and name not in only:
            continue
        np.savez_compressed(HERE / f"{name}.npz", **fn())
        print(f"wrote {name}.npz")


if __name__ == "__main__":
    main()
