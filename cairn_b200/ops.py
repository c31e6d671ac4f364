"""Torch-facing forms of CAIRN's hot-path operations, each one call into libcairn_b200.so on the tensors' device and
torch's current stream. PyTorch supplies device memory and streams; the arithmetic is the library's CUDA kernels.

The names and argument meanings follow the reference:
  mma_unordered(m, n, k, c, a, b)   the builtin (compiler/device/tensor.py:35-82 -> cr::tensor::launch,
                                    runtime/cairn_tensor.hpp:206-221): c (f32) += a * b, a and b of one storage float.
  gemm(a, b, ...)                   the same product with transposed operands and a fused epilogue (the dense layer's
                                    forward and its derive-grad backward, compiler/derive/gradients.py:1-11).
  saxpy(a, x, y, out)               `parallel i in n { out[i] = a * x[i] + y[i]; }` (cr::gpu::run,
                                    runtime/cairn_exec.hpp:103-108).
  reduce_sum(x)                     `reduce + parallel i in n yield x[i]` over f32 or u64 (cr::gpu::reduce_on,
                                    runtime/cairn_exec.hpp:163-168); u64 is the checked sum and raises on overflow
                                    where the reference traps.
A guard the reference traps on raises CairnError with the library's status.
"""

from __future__ import annotations

import ctypes as C

import torch

from ._lib import (
    ACT_NONE,
    ACT_RELU,
    BF16,
    ERR_ARG,
    ERR_OVERFLOW,
    F8E4M3,
    F8E5M2,
    F16,
    OUT_ACC_F32,
    OUT_BF16,
    OUT_STORE_F32,
    TF32,
    CairnError,
    check,
    lib,
)

FORMATS = {
    torch.bfloat16: (BF16, "cairn_b200_mma_bf16"),
    torch.float16: (F16, "cairn_b200_mma_f16"),
    torch.float8_e4m3fn: (F8E4M3, "cairn_b200_mma_f8e4m3"),
    torch.float8_e5m2: (F8E5M2, "cairn_b200_mma_f8e5m2"),
    torch.float32: (TF32, "cairn_b200_mma_tf32"),
}


def _stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _dev(*ts: torch.Tensor | None) -> None:
    first = next(t for t in ts if t is not None)
    for t in ts:
        if t is None:
            continue
        if not t.is_cuda or t.device != first.device:
            raise CairnError(ERR_ARG, "every operand must be a CUDA tensor on one device")
        if not t.is_contiguous():
            raise CairnError(ERR_ARG, "operands are contiguous row-major views")
    torch.cuda.set_device(first.device)


def mma_unordered(m: int, n: int, k: int, c: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> None:
    """c (row-major m x n, f32) += a (m x k) * b (k x n); a and b share one storage float (E-MMA,
    compiler/device/tensor.py:47-50). f32 operands run as tf32 (the reference refuses them)."""
    if a.dtype != b.dtype or a.dtype not in FORMATS or c.dtype != torch.float32:
        raise CairnError(ERR_ARG, "mma_unordered: a and b of one storage float, c an f32 view")
    _dev(c, a, b)
    _, name = FORMATS[a.dtype]
    status = getattr(lib(), name)(_stream(c), m, n, k, c.data_ptr(), c.numel(), a.data_ptr(), a.numel(), b.data_ptr(),
                                  b.numel())
    check(status, "mma_unordered")


def gemm(a: torch.Tensor, b: torch.Tensor, *, trans_a: bool = False, trans_b: bool = False,
         out: torch.Tensor | None = None, accumulate: bool = False, bias: torch.Tensor | None = None,
         relu: bool = False, out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """op(a) * op(b) with op(x) = x or x^T (a is m x k, or k x m with trans_a; b is k x n, or n x k with trans_b).

    out_dtype f32: out = product, or out += product with accumulate. out_dtype bf16: out = bf16(act(product + bias)),
    act = ReLU with relu. The tensor cores accumulate in f32 in every case."""
    if a.dtype != b.dtype or a.dtype not in FORMATS:
        raise CairnError(ERR_ARG, "gemm: a and b of one storage float")
    m, k = (a.shape[1], a.shape[0]) if trans_a else (a.shape[0], a.shape[1])
    kb, n = (b.shape[1], b.shape[0]) if trans_b else (b.shape[0], b.shape[1])
    if kb != k:
        raise CairnError(1, "gemm: the inner extents differ")
    if out_dtype == torch.bfloat16:
        kind = OUT_BF16
    elif out_dtype == torch.float32:
        kind = OUT_ACC_F32 if accumulate else OUT_STORE_F32
    else:
        raise CairnError(ERR_ARG, "gemm: out_dtype is f32 or bf16")
    if out is None:
        if accumulate:
            raise CairnError(ERR_ARG, "gemm: accumulate needs out")
        out = torch.empty((m, n), dtype=out_dtype, device=a.device)
    if out.dtype != out_dtype or out.numel() != m * n:
        raise CairnError(1, "gemm: out is m x n of out_dtype")
    if bias is not None and (bias.dtype != torch.float32 or bias.numel() != n):
        raise CairnError(ERR_ARG, "gemm: bias is n f32 values")
    _dev(out, a, b, bias)
    fmt, _ = FORMATS[a.dtype]
    status = lib().cairn_b200_gemm(_stream(out), fmt, m, n, k, a.data_ptr(), int(trans_a), b.data_ptr(), int(trans_b),
                                   out.data_ptr(), kind, bias.data_ptr() if bias is not None else None,
                                   ACT_RELU if relu else ACT_NONE)
    check(status, "gemm")
    return out


def saxpy(a: float, x: torch.Tensor, y: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """out[i] = a * x[i] + y[i] over f32, two roundings (no fused multiply-add)."""
    if x.dtype != torch.float32 or y.dtype != torch.float32 or x.numel() != y.numel():
        raise CairnError(ERR_ARG, "saxpy: x and y are f32 views of one extent")
    if out is None:
        out = torch.empty_like(x)
    if out.dtype != torch.float32 or out.numel() != x.numel():
        raise CairnError(ERR_ARG, "saxpy: out is an f32 view of x's extent")
    _dev(out, x, y)
    check(lib().cairn_b200_saxpy_f32(_stream(out), x.numel(), out.data_ptr(), x.data_ptr(), y.data_ptr(), float(a)),
          "saxpy")
    return out


def reduce_sum(x: torch.Tensor, out: torch.Tensor | None = None, overflow: torch.Tensor | None = None):
    """`reduce + parallel` over x. Without `out`, waits and returns the total as a Python number (the reduce_on form):
    f32 -> float (the exact sum rounded once, to a few f64 ulps); u64 (torch.uint64) -> int, raising CairnError on
    overflow as cr::Sum::checked traps. With `out` (a 1-element device tensor: f32 or f64 for f32 input, u64 for u64
    input, plus `overflow`, a 1-element int32/uint32), queues the sum and returns at once (the reduce_into form)."""
    _dev(x, out, overflow)
    s = _stream(x)
    n = x.numel()
    if x.dtype == torch.float32:
        if out is None:
            result = C.c_float(0.0)
            check(lib().cairn_b200_sum_f32_host(s, n, x.data_ptr(), C.byref(result)), "reduce_sum")
            return result.value
        if out.dtype == torch.float64:
            check(lib().cairn_b200_sum_f32_partial(s, n, x.data_ptr(), out.data_ptr()), "reduce_sum")
        else:
            check(lib().cairn_b200_sum_f32(s, n, x.data_ptr(), out.data_ptr()), "reduce_sum")
        return out
    if x.dtype == torch.uint64:
        if out is None:
            result, over = C.c_uint64(0), C.c_int(0)
            status = lib().cairn_b200_sum_u64_host(s, n, x.data_ptr(), C.byref(result), C.byref(over))
            if status == ERR_OVERFLOW:
                raise CairnError(status, "reduce_sum")
            check(status, "reduce_sum")
            return result.value
        if overflow is None:
            raise CairnError(ERR_ARG, "reduce_sum: a u64 sum into a device cell needs its overflow cell")
        check(lib().cairn_b200_sum_u64(s, n, x.data_ptr(), out.data_ptr(), overflow.data_ptr()), "reduce_sum")
        return out
    raise CairnError(ERR_ARG, "reduce_sum: x is f32 or u64")


def stream_status(device: torch.device | int | None = None) -> None:
    """Waits for the current stream and raises if a CUDA error or a device-side fault (a wait that ran out its
    bound) was recorded."""
    stream = torch.cuda.current_stream(device).cuda_stream
    check(lib().cairn_b200_stream_status(stream), "stream_status")


def watchdog_selftest(device: torch.device | int | None = None) -> None:
    """Runs the device watchdog's self-test on the current stream (a bounded wait on a barrier nothing completes
    must give up and report its fault); raises CairnError if it did not."""
    stream = torch.cuda.current_stream(device).cuda_stream
    check(lib().cairn_b200_watchdog_selftest(stream), "watchdog_selftest")
