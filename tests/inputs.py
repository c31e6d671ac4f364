"""Seeded synthetic inputs shared by the golden-fixture generator, the parity tests and the bench.

Shapes and value ranges follow the reference's own tests of this path:
  MMA_SHAPES      tests/soundness/test_tensor.py:65 (host multiply vs replay) and :214-222 (device vs host)
  TILE_SHAPES     tests/runtime/tensor_runtime.cpp:99-110 (tails in every direction, empties, chunked shapes)
  finite_patterns tests/soundness/test_tensor.py:48-56: random bit patterns of the format, finite, |v| <= limit
  sum cases       the categories of tests/soundness/test_exact_sum.py:boundaries/randoms (rounding boundaries,
                  special values, subnormals, overflow, cancellation, sizes around the pool's chunk and cutoff),
                  generated here by this file's own code.
"""

from __future__ import annotations

import math
import struct

import numpy as np

MMA_SHAPES = [(1, 1, 1), (3, 5, 7), (8, 8, 8), (17, 3, 33), (2, 40, 5), (4, 4, 0), (0, 3, 3), (12, 13, 64)]
TILE_SHAPES = [(1, 1, 1), (64, 64, 32), (65, 63, 33), (130, 70, 100), (17, 200, 64), (0, 5, 5), (5, 5, 0),
               (3, 129, 31), (72, 80, 96), (1, 8, 8), (100, 64, 40), (129, 136, 8)]
FORMATS = ["bf16", "f16", "f8e4m3", "f8e5m2"]
WIDTH = {"bf16": 16, "f16": 16, "f8e4m3": 8, "f8e5m2": 8}


def decode(fmt: str, bits: np.ndarray) -> np.ndarray:
    """Exact f64 values of storage-float patterns (the format definitions of runtime/cairn_float.hpp:160-167)."""
    bits = np.asarray(bits).astype(np.int64)
    if fmt == "bf16":
        with np.errstate(invalid="ignore"):
            return (bits.astype(np.uint32) << 16).view(np.float32).astype(np.float64)
    E, M, inf = {"f16": (5, 10, True), "f8e4m3": (4, 3, False), "f8e5m2": (5, 2, True)}[fmt]
    sign = np.where((bits >> (E + M)) & 1, -1.0, 1.0)
    e = (bits >> M) & ((1 << E) - 1)
    f = (bits & ((1 << M) - 1)).astype(np.float64)
    bias = (1 << (E - 1)) - 1
    top = (1 << E) - 1
    normal = np.ldexp(1.0 + f / (1 << M), (e - bias).astype(np.int64))
    sub = np.ldexp(f, 1 - bias - M)
    v = np.where(e == 0, sub, normal)
    special = (e == top) & (inf | (f == (1 << M) - 1))
    v = np.where(special, np.where(inf & (f == 0), np.inf, np.nan), v)
    return sign * v


def finite_patterns(fmt: str, rng: np.random.Generator, count: int, limit: float) -> np.ndarray:
    dtype = np.uint16 if WIDTH[fmt] == 16 else np.uint8
    out = np.empty(0, dtype)
    while out.size < count:
        cand = rng.integers(0, 1 << WIDTH[fmt], size=max(2 * (count - out.size), 16), dtype=np.int64).astype(dtype)
        v = decode(fmt, cand)
        keep = cand[np.isfinite(v) & (np.abs(v) <= limit)]
        out = np.concatenate([out, keep])
    return out[:count]


def mma_case(fmt: str, m: int, n: int, k: int, seed: int):
    """(c, a, b) for one multiply: finite patterns of the format and c ~ U(-4, 4) as f32."""
    rng = np.random.default_rng(seed)
    limit = 1e6 if fmt == "bf16" else 448.0
    a = finite_patterns(fmt, rng, m * k, limit)
    b = finite_patterns(fmt, rng, k * n, limit)
    c = rng.uniform(-4, 4, size=m * n).astype(np.float32)
    return c, a, b


def tile_case(fmt: str, m: int, n: int, k: int):
    """Multiples of 1/16 in [-30/16, 30/16] from a hash of the index, as tensor_runtime.cpp's matrix() draws them
    (every such value is exact in every format), and c in quarters in [-1, 1]."""
    def mix(x: np.ndarray) -> np.ndarray:
        x = x.astype(np.uint64)
        x ^= x >> np.uint64(31)
        x *= np.uint64(0x7FB5D329728EA185)
        x ^= x >> np.uint64(27)
        return x

    def values(count: int, seed: int) -> np.ndarray:
        h = mix(np.arange(count, dtype=np.uint64) + np.uint64(seed))
        return ((h % np.uint64(61)).astype(np.int64) - 30) / 16.0

    av, bv = values(m * k, 1 + m), values(k * n, 7 + n)
    c = ((mix(np.arange(m * n, dtype=np.uint64) + np.uint64(99)) % np.uint64(9)).astype(np.int64) - 4) / 4.0
    return c.astype(np.float32), encode(fmt, av), encode(fmt, bv)


def encode(fmt: str, v: np.ndarray) -> np.ndarray:
    """Patterns of f32-exact values rounded once to the format, nearest-even (cr::fp::narrow, cairn_float.hpp:324-334,
    for values inside the format's range)."""
    v = np.asarray(v, np.float64).astype(np.float32)
    if fmt == "bf16":
        u = v.view(np.uint32).astype(np.uint64)
        u = u + np.uint64(0x7FFF) + ((u >> np.uint64(16)) & np.uint64(1))
        return (u >> np.uint64(16)).astype(np.uint16)
    if fmt == "f16":
        return v.astype(np.float16).view(np.uint16)
    import torch

    dtype = torch.float8_e4m3fn if fmt == "f8e4m3" else torch.float8_e5m2
    return torch.from_numpy(v.copy()).to(dtype).view(torch.uint8).numpy()


# ---- sums ----------------------------------------------------------------------------------------------------------
def f32(x: float) -> float:
    try:
        return struct.unpack("<f", struct.pack("<f", x))[0]
    except OverflowError:
        return math.copysign(math.inf, x)


def sum_boundary_cases():
    """f32 terms whose exact sums sit on or beside rounding boundaries, and the special values."""
    big = struct.unpack("<f", struct.pack("<I", 0x7F7FFFFF))[0]
    tiny = struct.unpack("<f", struct.pack("<I", 1))[0]
    half = 2.0**-24
    top = 2.0 ** (127 - 24)
    least_normal = 2.0**-126
    yield "empty", []
    for v in (1.0, 3.0, -0.0, 0.0, tiny, -tiny, least_normal, big, -big, math.inf, -math.inf, math.nan):
        yield f"one {v!r}", [v]
    yield "all -0.0", [-0.0] * 9
    yield "-0.0 and +0.0", [-0.0, 0.0, -0.0]
    yield "x and -x", [1.5, -1.5]
    yield "cancellation", [big / 2, 1.0, -big / 2]
    yield "tie to even, down", [1.0, half]
    yield "tie to even, up", [1.0 + 2 * half, half]
    yield "above a tie", [1.0, half, tiny]
    yield "below a tie", [1.0, half, -tiny]
    yield "tie below a power of two", [1.0, 1.0, -half]
    yield "one ulp below two", [2.0, -2 * half]
    yield "largest and half its ulp", [big, top]
    yield "just below overflow", [big, top, -tiny]
    yield "overflow", [big, big]
    yield "negative overflow", [-big, -big, 1.0]
    yield "over the top and back", [big, big, -big]
    yield "subnormals", [tiny] * 7
    yield "least normal less least subnormal", [least_normal, -tiny]
    yield "NaN among finite", [1.0, math.nan, 2.0]
    yield "both infinities", [math.inf, 1.0, -math.inf]
    yield "no double rounding, up", [1.0, 2.0**-24, 2.0**-100]
    yield "no double rounding, down", [1.0, 2.0**-24, -(2.0**-100)]


def sum_random_cases(seed: int = 2):
    rng = np.random.default_rng(seed)
    for n in (255, 256, 257, 16_383, 16_385, 65_537):
        yield f"uniform {n}", rng.random(n).astype(np.float32)
        yield f"signed {n}", rng.uniform(-1, 1, n).astype(np.float32)
        yield f"medium {n}", (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-60, 60, n)).astype(np.float32)
        pairs = (rng.uniform(-1, 1, n // 2) * 2.0 ** rng.integers(-30, 30, n // 2)).astype(np.float32)
        yield f"pairs that cancel {n}", np.concatenate([pairs, -pairs[::-1], np.float32([2.0**-40])])
        yield f"subnormal {n}", (rng.choice([-1, 1], n) * rng.integers(1, 2**20, n) * 2.0**-149).astype(np.float32)


def u64_cases() -> dict[str, np.ndarray]:
    """Checked u64 sums: data[i] = i over 1e6 (499999500000), a total that fits beside one that
    does not while every block total fits (tests/soundness/test_pooled_reduce.py:118-140's shape, in u64), a wrap
    in the last terms, and the largest term."""
    return {
        "iota_1e6": np.arange(1_000_000, dtype=np.uint64),
        "fits": np.full(100_000, 150_000 * 2**30, np.uint64),
        "over": np.full(100_000, 200_000 * 2**30, np.uint64),
        "wrap_at_end": np.asarray([2**63, 2**62, 2**62 - 1, 1, 5], np.uint64),
        "top": np.asarray([2**64 - 1, 0, 0], np.uint64),
        "empty": np.zeros(0, np.uint64),
    }


def saxpy_case(n: int, seed: int = 0):
    rng = np.random.default_rng(seed)
    return rng.uniform(-1, 1, n).astype(np.float32), rng.uniform(-1, 1, n).astype(np.float32), np.float32(2.5)


# BASELINE config 3 at the reduced shape of tests/golden/mlp_grad.npz: batch 32, 128 -> 512 -> 128.
MLP_GOLDEN_SHAPE = (32, 128, 512, 128)


def mlp_case(B: int, D: int, H: int, O: int, seed: int = 0):
    """Config 3's operands at any shape: x ~ N(0, 1) and w1, w2 ~ N(0, 0.32) as bf16 patterns (config 3's N(0, 0.02)
    scaled by 16, so that products of a few hundred terms keep a spread of signs and sizes), target t ~ N(0, 1)."""
    rng = np.random.default_rng(seed)
    x = encode("bf16", rng.standard_normal(B * D))
    w1 = encode("bf16", rng.standard_normal(D * H) * 0.02 * 16)
    w2 = encode("bf16", rng.standard_normal(H * O) * 0.02 * 16)
    t = rng.standard_normal(B * O).astype(np.float32)
    return x, w1, w2, t


def config1_gemm():
    """BASELINE config 1's f32 GEMM operands: M = N = K = 512, A then B ~ U[-1, 1] from numpy's default_rng(0)."""
    rng = np.random.default_rng(0)
    a = rng.uniform(-1, 1, 512 * 512).astype(np.float32)
    b = rng.uniform(-1, 1, 512 * 512).astype(np.float32)
    return a, b
