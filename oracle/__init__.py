"""TEST INFRASTRUCTURE ONLY: the CPU oracle of the cairn_b200 parity tests.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg (and its reference arm) import this package,
and only as the checker or the timed CPU baseline; the cairn_b200 package never does.

  restated   numpy wrappers of liboracle.so, the C restatement in cairn_oracle.c (each function cites the
             reference file:line it restates)
  reference  numpy wrappers of _ref/libcairn_ref.so, the reference's own header-only host path compiled from its
             sources by the Makefile here, and of _ref/libmlp_grad.so, grad/mlp_grad.cairn built by the reference's
             own compiler (its `derive grad` output for config 3's layers); both present where the reference tree
             was available at build time
  exact_sum_f32_bits  a pure-Python model of the correctly rounded sum (Fraction arithmetic) for small cases
"""

from __future__ import annotations

import ctypes as C
import math
import struct
import subprocess
from fractions import Fraction
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
RESTATED = HERE / "liboracle.so"
REFERENCE = HERE / "_ref" / "libcairn_ref.so"
GRAD = HERE / "_ref" / "libmlp_grad.so"
GRAD_SOURCE = HERE / "grad" / "mlp_grad.cairn"

_z, _p, _f = C.c_size_t, C.c_void_p, C.c_float


def build(reference_tree: str | None = None) -> None:
    """make -C oracle [REF=...]: the restatement always; where the CAIRN reference checkout (the directory holding
    src/cairn) is given, also the reference's host path from its runtime headers, and grad/mlp_grad.cairn through the
    reference's own compiler (`cairn build --kind library --cxx g++`, its host toolchain's flags)."""
    cmd = ["make", "-s", "-C", str(HERE)]
    if reference_tree:
        cmd.append(f"REF={Path(reference_tree) / 'src' / 'cairn' / 'runtime'}")
    subprocess.run(cmd, check=True)
    if reference_tree:
        build_grad(reference_tree)


def build_grad(reference_tree: str) -> Path:
    """grad/mlp_grad.cairn compiled by the reference's compiler into _ref/libmlp_grad.so (and its C header)."""
    import json
    import os
    import shutil
    import sys
    import tempfile

    env = dict(os.environ, PYTHONPATH=str(Path(reference_tree) / "src"))
    with tempfile.TemporaryDirectory(prefix="cairn-grad-") as tmp:
        done = subprocess.run([sys.executable, "-m", "cairn", "build", str(GRAD_SOURCE), "--cxx", "g++", "--kind",
                               "library", "--header", "--out", tmp, "--format", "json"], capture_output=True, text=True,
                              env=env, cwd=tmp, timeout=900)
        if done.returncode != 0:
            raise RuntimeError(f"cairn build mlp_grad.cairn failed:\n{done.stdout[-3000:]}{done.stderr[-3000:]}")
        record = json.loads(done.stdout)
        GRAD.parent.mkdir(exist_ok=True)
        shutil.copy2(record["artifact"], GRAD)
        shutil.copy2(record["header"], GRAD.with_name("mlp_grad.h"))
    return GRAD


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


class _Lib:
    def __init__(self, path: Path, prefix: str):
        self.path, self.prefix, self._h = path, prefix, None

    def available(self) -> bool:
        return self.path.exists()

    def h(self) -> C.CDLL:
        if self._h is None:
            if not self.path.exists():
                if self.path == RESTATED:
                    build()
                else:
                    raise FileNotFoundError(f"{self.path} is not built (it needs the reference source tree)")
            self._h = C.CDLL(str(self.path))
        return self._h

    def fn(self, name: str, res, args):
        f = getattr(self.h(), self.prefix + name)
        f.restype, f.argtypes = res, args
        return f


_rest = _Lib(RESTATED, "oracle_")
_ref = _Lib(REFERENCE, "ref_")
_grad = _Lib(GRAD, "cf_")

MMA_DTYPES = {"bf16": np.uint16, "f16": np.uint16, "f8e4m3": np.uint8, "f8e5m2": np.uint8, "f32": np.float32}


class restated:
    """The C restatement (cairn_oracle.c)."""

    @staticmethod
    def mma(fmt: str, c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        """c (f32, m*n) += a * b in the reference's order; returns a new array."""
        name = {"bf16": "mma_bf16", "f16": "mma_f16", "f8e4m3": "mma_e4m3", "f8e5m2": "mma_e5m2", "f32": "mma_f32"}[fmt]
        out = np.ascontiguousarray(c, dtype=np.float32).copy()
        a = np.ascontiguousarray(a, dtype=MMA_DTYPES[fmt])
        b = np.ascontiguousarray(b, dtype=MMA_DTYPES[fmt])
        _rest.fn(name, None, [_z, _z, _z, _p, _p, _p])(m, n, k, _ptr(out), _ptr(a), _ptr(b))
        return out

    @staticmethod
    def mma_bf16_rows(a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, r0: int, r1: int,
                      c_rows: np.ndarray | None = None) -> np.ndarray:
        out = np.zeros((r1 - r0) * n, np.float32) if c_rows is None else np.ascontiguousarray(c_rows, np.float32).copy()
        a = np.ascontiguousarray(a, np.uint16)
        b = np.ascontiguousarray(b, np.uint16)
        _rest.fn("mma_bf16_rows", None, [_z, _z, _z, _z, _z, _p, _p, _p])(m, n, k, r0, r1, _ptr(out), _ptr(a), _ptr(b))
        return out

    @staticmethod
    def gemm_t16(c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int, trans_a: bool, trans_b: bool,
                 fmt: str = "bf16") -> np.ndarray:
        out = np.ascontiguousarray(c, np.float32).copy()
        a = np.ascontiguousarray(a, np.uint16)
        b = np.ascontiguousarray(b, np.uint16)
        _rest.fn("gemm_t16", None, [_z, _z, _z, _p, _p, _p, C.c_int, C.c_int, C.c_int])(
            m, n, k, _ptr(out), _ptr(a), _ptr(b), int(trans_a), int(trans_b), 1 if fmt == "f16" else 0)
        return out

    @staticmethod
    def bias_act(acc: np.ndarray, bias: np.ndarray | None, relu: bool, m: int, n: int) -> np.ndarray:
        acc = np.ascontiguousarray(acc, np.float32)
        out = np.empty(m * n, np.uint16)
        bias_c = None if bias is None else np.ascontiguousarray(bias, np.float32)
        _rest.fn("bias_act", None, [_z, _z, _p, _p, C.c_int, _p])(
            m, n, _ptr(acc), None if bias_c is None else _ptr(bias_c), int(relu), _ptr(out))
        return out

    @staticmethod
    def mlp_step(x: np.ndarray, w1: np.ndarray, w2: np.ndarray, t: np.ndarray, B: int, D: int, Hd: int, O: int):
        """BASELINE config 3's step at any shape: bf16 patterns x (B x D), w1 (D x Hd), w2 (Hd x O), f32 target t.
        Returns a dict of H, Y, dY, loss, dW2, dH, dW1, dX."""
        x, w1, w2 = (np.ascontiguousarray(v, np.uint16) for v in (x, w1, w2))
        t = np.ascontiguousarray(t, np.float32)
        out = {"H": np.empty(B * Hd, np.uint16), "Y": np.empty(B * O, np.float32), "dY": np.empty(B * O, np.uint16),
               "loss": np.zeros(1, np.float32), "dW2": np.empty(Hd * O, np.float32),
               "dH": np.empty(B * Hd, np.uint16), "dW1": np.empty(D * Hd, np.float32), "dX": np.empty(B * D, np.float32)}
        _rest.fn("mlp_step", None, [_z] * 4 + [_p] * 12)(
            B, D, Hd, O, _ptr(x), _ptr(w1), _ptr(w2), _ptr(t), *(_ptr(out[k]) for k in
                                                                 ("H", "Y", "dY", "loss", "dW2", "dH", "dW1", "dX")))
        return out

    @staticmethod
    def sum_f32(x: np.ndarray) -> np.float32:
        x = np.ascontiguousarray(x, np.float32)
        return np.float32(_rest.fn("sum_f32", _f, [_z, _p])(x.size, _ptr(x)))

    @staticmethod
    def sum_u64(x: np.ndarray) -> tuple[int, bool]:
        x = np.ascontiguousarray(x, np.uint64)
        over = C.c_int(0)
        v = _rest.fn("sum_u64", C.c_uint64, [_z, _p, C.POINTER(C.c_int)])(x.size, _ptr(x), C.byref(over))
        return int(v), bool(over.value)

    @staticmethod
    def saxpy(a: float, x: np.ndarray, y: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        out = np.empty_like(x)
        _rest.fn("saxpy_f32", None, [_z, _p, _p, _p, _f])(x.size, _ptr(out), _ptr(x), _ptr(y), a)
        return out

    @staticmethod
    def scan_u32(x: np.ndarray) -> tuple[np.ndarray, int]:
        x = np.ascontiguousarray(x, np.uint32)
        out = np.empty_like(x)
        total = _rest.fn("scan_u32", C.c_uint32, [_z, _p, _p])(x.size, _ptr(out), _ptr(x))
        return out, int(total)

    @staticmethod
    def runmax_i32(x: np.ndarray) -> tuple[np.ndarray, int]:
        x = np.ascontiguousarray(x, np.int32)
        out = np.empty_like(x)
        total = _rest.fn("runmax_i32", C.c_int32, [_z, _p, _p])(x.size, _ptr(out), _ptr(x))
        return out, int(total)

    @staticmethod
    def widen(fmt: str, bits: np.ndarray) -> np.ndarray:
        name = {"bf16": "bf16_to_f32", "f16": "f16_to_f32", "f8e4m3": "e4m3_to_f32", "f8e5m2": "e5m2_to_f32"}[fmt]
        argt = C.c_uint16 if fmt in ("bf16", "f16") else C.c_uint8
        f = _rest.fn(name, _f, [argt])
        return np.array([f(int(v)) for v in np.asarray(bits).ravel()], np.float32)

    @staticmethod
    def f32_to_bf16(x: np.ndarray) -> np.ndarray:
        f = _rest.fn("f32_to_bf16", C.c_uint16, [_f])
        return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)


class reference:
    """The reference's own host path (ref_shim.cpp over the CAIRN runtime headers)."""

    @staticmethod
    def available() -> bool:
        return _ref.available()

    @staticmethod
    def mma(fmt: str, c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        out = np.ascontiguousarray(c, np.float32).copy()
        a = np.ascontiguousarray(a, MMA_DTYPES[fmt])
        b = np.ascontiguousarray(b, MMA_DTYPES[fmt])
        _ref.fn(f"mma_{fmt}", None, [_z, _z, _z, _p, _p, _p])(m, n, k, _ptr(out), _ptr(a), _ptr(b))
        return out

    @staticmethod
    def mma_bf16_pooled(c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        out = np.ascontiguousarray(c, np.float32).copy()
        _ref.fn("mma_bf16_pooled", None, [_z, _z, _z, _p, _p, _p])(
            m, n, k, _ptr(out), _ptr(np.ascontiguousarray(a, np.uint16)), _ptr(np.ascontiguousarray(b, np.uint16)))
        return out

    @staticmethod
    def gemm_f32_region(c: np.ndarray, a: np.ndarray, b: np.ndarray, m: int, n: int, k: int) -> np.ndarray:
        out = np.ascontiguousarray(c, np.float32).copy()
        _ref.fn("gemm_f32_region", None, [_z, _z, _z, _p, _p, _p])(
            m, n, k, _ptr(out), _ptr(np.ascontiguousarray(a, np.float32)), _ptr(np.ascontiguousarray(b, np.float32)))
        return out

    @staticmethod
    def sum_f32(x: np.ndarray) -> np.float32:
        x = np.ascontiguousarray(x, np.float32)
        return np.float32(_ref.fn("sum_f32", _f, [_z, _p])(x.size, _ptr(x)))

    @staticmethod
    def sum_u64(x: np.ndarray) -> tuple[int, bool]:
        x = np.ascontiguousarray(x, np.uint64)
        over = C.c_int(0)
        v = _ref.fn("sum_u64", C.c_uint64, [_z, _p, C.POINTER(C.c_int)])(x.size, _ptr(x), C.byref(over))
        return int(v), bool(over.value)

    @staticmethod
    def saxpy(a: float, x: np.ndarray, y: np.ndarray, out: np.ndarray | None = None) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        y = np.ascontiguousarray(y, np.float32)
        out = np.empty_like(x) if out is None else out
        _ref.fn("saxpy_f32", None, [_z, _p, _p, _p, _f])(x.size, _ptr(out), _ptr(x), _ptr(y), a)
        return out

    @staticmethod
    def scan_u32(x: np.ndarray, out: np.ndarray | None = None) -> tuple[np.ndarray, int]:
        x = np.ascontiguousarray(x, np.uint32)
        out = np.empty_like(x) if out is None else out
        total = _ref.fn("scan_u32", C.c_uint32, [_z, _p, _p])(x.size, _ptr(out), _ptr(x))
        return out, int(total)

    @staticmethod
    def runmax_i32(x: np.ndarray) -> tuple[np.ndarray, int]:
        x = np.ascontiguousarray(x, np.int32)
        out = np.empty_like(x)
        total = _ref.fn("runmax_i32", C.c_int32, [_z, _p, _p])(x.size, _ptr(out), _ptr(x))
        return out, int(total)

    @staticmethod
    def widen(fmt: str, bits: np.ndarray) -> np.ndarray:
        argt = C.c_uint16 if fmt in ("bf16", "f16") else C.c_uint8
        f = _ref.fn(f"widen_{fmt}", _f, [argt])
        return np.array([f(int(v)) for v in np.asarray(bits).ravel()], np.float32)

    @staticmethod
    def narrow_bf16(x: float) -> int:
        return int(_ref.fn("narrow_bf16", C.c_uint16, [C.c_double])(x))

    @staticmethod
    def lanes() -> int:
        return int(_ref.fn("lanes", _z, [])())

    # ---- derive grad (_ref/libmlp_grad.so: grad/mlp_grad.cairn through the reference's compiler) ----
    @staticmethod
    def grad_available() -> bool:
        return _grad.available()

    @staticmethod
    def dense(x: np.ndarray, w: np.ndarray, b: int, k: int, n: int) -> np.ndarray:
        """cf_dense: out (b x n) = x (b x k) w (k x n) in f32, each output's terms summed in increasing p."""
        x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
        out = np.empty(b * n, np.float32)
        _grad.fn("dense", None, [_z, _z, _z, _z, _p, _z, _p, _z, _p])(b, k, n, b * k, _ptr(x), k * n, _ptr(w), b * n,
                                                                      _ptr(out))
        return out

    @staticmethod
    def dense_grad(x: np.ndarray, w: np.ndarray, d_out: np.ndarray, b: int, k: int, n: int):
        """cf_dense_grad, derive grad's adjoint of `dense`, from zeroed adjoints: returns (d_x, d_w)."""
        x, w = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(w, np.float32)
        d_out = np.ascontiguousarray(d_out, np.float32)
        out, d_x, d_w = np.empty(b * n, np.float32), np.zeros(b * k, np.float32), np.zeros(k * n, np.float32)
        _grad.fn("dense_grad", None, [_z, _z, _z, _z, _p, _z, _p, _z, _p, _p, _p, _p])(
            b, k, n, b * k, _ptr(x), k * n, _ptr(w), b * n, _ptr(out), _ptr(d_x), _ptr(d_w), _ptr(d_out))
        return d_x, d_w

    @staticmethod
    def mse_grad(y: np.ndarray, t: np.ndarray, seed: float = 1.0):
        """cf_mse_grad from a zeroed adjoint: returns (the loss, d_y)."""
        y, t = np.ascontiguousarray(y, np.float32), np.ascontiguousarray(t, np.float32)
        d_y = np.zeros(y.size, np.float32)
        loss = _grad.fn("mse_grad", _f, [_z, _p, _p, _f, _p])(y.size, _ptr(y), _ptr(t), seed, _ptr(d_y))
        return np.float32(loss), d_y

    @staticmethod
    def relu(z: np.ndarray) -> np.ndarray:
        f = _grad.fn("relu", _f, [_f])
        return np.array([f(float(v)) for v in np.asarray(z, np.float32).ravel()], np.float32)

    @staticmethod
    def relu_grad(z: np.ndarray, seed: np.ndarray) -> np.ndarray:
        """cf_relu_grad per element from a zeroed adjoint: d_z = seed where z > 0, else 0."""
        f = _grad.fn("relu_grad", _f, [_f, _f, C.POINTER(C.c_float)])
        out = np.zeros(np.asarray(z).size, np.float32)
        cell = C.c_float(0.0)
        for i, (zv, sv) in enumerate(zip(np.asarray(z, np.float32).ravel(), np.asarray(seed, np.float32).ravel())):
            cell.value = 0.0
            f(float(zv), float(sv), C.byref(cell))
            out[i] = cell.value
        return out

    @staticmethod
    def narrow_bf16_array(x: np.ndarray) -> np.ndarray:
        f = _ref.fn("narrow_bf16", C.c_uint16, [C.c_double])
        return np.array([f(float(v)) for v in np.asarray(x, np.float32).ravel()], np.uint16)

    @staticmethod
    def mlp_step(x: np.ndarray, w1: np.ndarray, w2: np.ndarray, t: np.ndarray, B: int, D: int, Hd: int, O: int):
        """Config 3's step from the reference's own code alone: its dense layers and derive-grad adjoints
        (_ref/libmlp_grad.so), its relu and relu_grad, its mse_grad, and cr::fp::narrow to bf16 where the step
        stores bf16 (H, dY, dH). x, w1, w2 are bf16 patterns, t f32. Returns the same dict as restated.mlp_step."""
        xf = reference.widen("bf16", x)
        w1f = reference.widen("bf16", w1)
        w2f = reference.widen("bf16", w2)
        pre = reference.dense(xf, w1f, B, D, Hd)
        h = reference.narrow_bf16_array(reference.relu(pre))
        hf = reference.widen("bf16", h)
        y = reference.dense(hf, w2f, B, Hd, O)
        loss, dy_f32 = reference.mse_grad(y, t)
        dy = reference.narrow_bf16_array(dy_f32)
        dh_pre, dw2 = reference.dense_grad(hf, w2f, reference.widen("bf16", dy), B, Hd, O)
        dh = reference.narrow_bf16_array(reference.relu_grad(pre, dh_pre))
        dx, dw1 = reference.dense_grad(xf, w1f, reference.widen("bf16", dh), B, D, Hd)
        return {"H": h, "Y": y, "dY": dy, "loss": np.asarray([loss], np.float32), "dW2": dw2, "dH": dh,
                "dW1": dw1, "dX": dx}


# ---- a pure-Python model of the correctly rounded f32 sum (for small cases) ----------------------------------------
def _f32_bits(x: float) -> int:
    return struct.unpack("<I", struct.pack("<f", x))[0]


def exact_sum_f32_bits(terms: list[float]) -> int:
    """The pattern of the f32 exact sum of f32 `terms`, rounded once to nearest-even, with cr::sum::result's rules
    for NaN, infinities and the sign of an exact zero (runtime/cairn_sum.hpp:186-195)."""
    if any(t != t for t in terms) or (math.inf in terms and -math.inf in terms):
        return 0x7FC00000
    if math.inf in terms:
        return 0x7F800000
    if -math.inf in terms:
        return 0xFF800000
    total = sum((Fraction(t) for t in terms), Fraction(0))
    if total == 0:
        return 0x80000000 if terms and all(_f32_bits(t) == 0x80000000 for t in terms) else 0
    sign = 0x80000000 if total < 0 else 0
    mag = abs(total)
    e = mag.numerator.bit_length() - mag.denominator.bit_length()
    while Fraction(2) ** e > mag:
        e -= 1
    while Fraction(2) ** (e + 1) <= mag:
        e += 1
    q = max(e, -126) - 23
    scaled = mag / Fraction(2) ** q
    m, rest = divmod(scaled.numerator, scaled.denominator)
    if 2 * rest > scaled.denominator or (2 * rest == scaled.denominator and m % 2 == 1):
        m += 1
    if m == 1 << 24:
        m >>= 1
        q += 1
    if m < 1 << 23:
        return sign | m
    exponent = q + 23
    if exponent > 127:
        return sign | 0x7F800000
    return sign | ((exponent + 127) << 23) | (m & 0x7FFFFF)
