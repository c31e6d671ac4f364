"""The multiply from host memory to host memory, with the copies and the products overlapped.

A CAIRN program whose operands live on the host moves them with `transfer` and then calls the device multiply
(`cr::tensor::launch`, runtime/cairn_tensor.hpp:206-221), one step after the other on its context's stream. On a B200
the host link (about 50 GB/s each way) takes ten times longer than the product itself for the 4096^3 case, so
`HostGemm` overlaps them:

  copy-in stream   B (and the bias), then A in row chunks, each chunk's arrival recorded;
  compute stream   each chunk's rows of C = op(A) B as soon as its A rows and B are in (cairn_b200_gemm);
  copy-out stream  each chunk of C back to host memory as soon as it is computed.

Each call uses one of `depth` sets of device buffers, so the next call's copies in run while this one's results are
still coming back; a set is reused only after its previous results have reached the host. Calls return at once with
an event that completes when the result is in host memory. Host buffers should be pinned (torch's pin_memory) for the
copies to run asynchronously at full speed. B and the bias may instead be device tensors that stay resident from call
to call, as a layer's weights do in training: then only A crosses in and C back.

Measured on a B200 (4096^3 bf16 with bias and ReLU, 64 MB in and 32 MB out per product, the link at 55 GB/s each
way and 1.29 ms for both directions at once): 1.36 ms per product in two chunks, 1.45 in four, 1.59 in eight
(each chunk's copies and launches cost more than its finer overlap saves), 1.41 unchunked; the same copies and
product on one stream take 1.96 ms.
"""

from __future__ import annotations

import torch

from ._lib import ERR_ARG, CairnError
from .ops import gemm, saxpy


class HostGemm:
    """out_host = op(a_host) * b_host (+ bias, ReLU, bf16), for fixed m, n, k, on one device."""

    def __init__(self, m: int, n: int, k: int, *, dtype: torch.dtype = torch.bfloat16,
                 out_dtype: torch.dtype = torch.bfloat16, trans_a: bool = False, bias: bool = False,
                 device: torch.device | int | None = None, chunks: int = 2, depth: int = 2):
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index or 0))
        if min(m, n, k) <= 0 or chunks <= 0 or depth <= 0:
            raise CairnError(ERR_ARG, "HostGemm: m, n, k, chunks and depth are positive")
        self.m, self.n, self.k, self.trans_a, self.out_dtype = m, n, k, trans_a, out_dtype
        # row chunks of A and C (A^T's rows are C's columns, so a transposed A is copied and multiplied whole)
        self.chunks = 1 if trans_a else max(1, min(chunks, m))
        bounds = [m * c // self.chunks for c in range(self.chunks + 1)]
        self.rows = [(lo, hi) for lo, hi in zip(bounds[:-1], bounds[1:]) if hi > lo]
        d = self.device
        a_shape = (k, m) if trans_a else (m, k)
        self.sets = [{"a": torch.empty(a_shape, dtype=dtype, device=d), "b": torch.empty((k, n), dtype=dtype, device=d),
                      "bias": torch.empty(n, dtype=torch.float32, device=d) if bias else None,
                      "out": torch.empty((m, n), dtype=out_dtype, device=d),
                      "free": None} for _ in range(depth)]
        self.copy_in = torch.cuda.Stream(d)
        self.compute = torch.cuda.Stream(d)
        self.copy_out = torch.cuda.Stream(d)
        self.calls = 0

    def submit(self, a_host: torch.Tensor, b_host: torch.Tensor, out_host: torch.Tensor,
               bias_host: torch.Tensor | None = None, relu: bool = False) -> torch.cuda.Event:
        """Queues one product; returns an event recorded once out_host holds the result."""
        s = self.sets[self.calls % len(self.sets)]
        self.calls += 1
        if (bias_host is None) != (s["bias"] is None):
            raise CairnError(ERR_ARG, "HostGemm: a bias was declared at construction, and only then is one passed")
        b_resident = b_host.device == self.device
        bias_resident = bias_host is not None and bias_host.device == self.device
        for t, want in ((a_host, s["a"]), (b_host, s["b"]), (out_host, s["out"])):
            where_ok = t.device.type == "cpu" or (t is b_host and b_resident)
            if not where_ok or t.shape != want.shape or t.dtype != want.dtype or not t.is_contiguous():
                raise CairnError(ERR_ARG, "HostGemm: host tensors of the declared shapes and types, contiguous (B may "
                                          "be a resident tensor on the multiply's device)")
        if bias_host is not None and s["bias"] is not None and (bias_host.device.type != "cpu" and not bias_resident
                                                                or bias_host.shape != s["bias"].shape):
            raise CairnError(ERR_ARG, "HostGemm: the bias is n f32 values in host memory or on the multiply's device")
        d_a, d_b, d_out, d_bias = s["a"], s["b"], s["out"], s["bias"]
        if s["free"] is not None:  # this set's previous results have reached the host
            self.copy_in.wait_event(s["free"])
        arrived = []
        with torch.cuda.stream(self.copy_in):
            if b_resident:
                d_b = b_host
            else:
                d_b.copy_(b_host, non_blocking=True)
            if bias_resident:
                d_bias = bias_host
            elif d_bias is not None:
                d_bias.copy_(bias_host, non_blocking=True)
            b_in = torch.cuda.Event()
            b_in.record(self.copy_in)
            for lo, hi in self.rows:
                if self.trans_a:
                    d_a.copy_(a_host, non_blocking=True)
                else:
                    d_a[lo:hi].copy_(a_host[lo:hi], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.copy_in)
                arrived.append(e)
        computed = []
        with torch.cuda.stream(self.compute):
            self.compute.wait_event(b_in)
            for (lo, hi), e in zip(self.rows, arrived):
                self.compute.wait_event(e)
                a_rows = d_a if self.trans_a else d_a[lo:hi]
                gemm(a_rows, d_b, trans_a=self.trans_a, out=d_out[lo:hi], bias=d_bias, relu=relu,
                     out_dtype=self.out_dtype)
                c = torch.cuda.Event()
                c.record(self.compute)
                computed.append(c)
        with torch.cuda.stream(self.copy_out):
            for (lo, hi), c in zip(self.rows, computed):
                self.copy_out.wait_event(c)
                out_host[lo:hi].copy_(d_out[lo:hi], non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.copy_out)
        s["free"] = done
        return done


class HostSaxpy:
    """out_host = a * x_host + y_host over n f32 (the `parallel` saxpy region) from host memory to host memory: x and
    y copied in by chunks on one stream, each chunk's region run as soon as it lands, each chunk's result copied back
    on a third, over `depth` sets of device buffers so that consecutive calls overlap as well."""

    def __init__(self, n: int, *, device: torch.device | int | None = None, chunks: int = 4, depth: int = 2):
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index or 0))
        if n <= 0 or chunks <= 0 or depth <= 0:
            raise CairnError(ERR_ARG, "HostSaxpy: n, chunks and depth are positive")
        self.n = n
        c = max(1, min(chunks, n))
        bounds = [n * i // c for i in range(c + 1)]
        self.ranges = [(lo, hi) for lo, hi in zip(bounds[:-1], bounds[1:]) if hi > lo]
        d = self.device
        self.sets = [{"x": torch.empty(n, dtype=torch.float32, device=d), "y": torch.empty(n, dtype=torch.float32, device=d),
                      "out": torch.empty(n, dtype=torch.float32, device=d), "free": None} for _ in range(depth)]
        self.copy_in, self.compute, self.copy_out = (torch.cuda.Stream(d) for _ in range(3))
        self.calls = 0

    def submit(self, a: float, x_host: torch.Tensor, y_host: torch.Tensor, out_host: torch.Tensor) -> torch.cuda.Event:
        """Queues one region; returns an event recorded once out_host holds the result."""
        for t in (x_host, y_host, out_host):
            if t.device.type != "cpu" or t.dtype != torch.float32 or t.numel() != self.n or not t.is_contiguous():
                raise CairnError(ERR_ARG, "HostSaxpy: contiguous f32 host tensors of n elements")
        s = self.sets[self.calls % len(self.sets)]
        self.calls += 1
        if s["free"] is not None:
            self.copy_in.wait_event(s["free"])
        x_h, y_h, o_h = x_host.view(-1), y_host.view(-1), out_host.view(-1)
        arrived, computed = [], []
        with torch.cuda.stream(self.copy_in):
            for lo, hi in self.ranges:
                s["x"][lo:hi].copy_(x_h[lo:hi], non_blocking=True)
                s["y"][lo:hi].copy_(y_h[lo:hi], non_blocking=True)
                e = torch.cuda.Event()
                e.record(self.copy_in)
                arrived.append(e)
        with torch.cuda.stream(self.compute):
            for (lo, hi), e in zip(self.ranges, arrived):
                self.compute.wait_event(e)
                saxpy(a, s["x"][lo:hi], s["y"][lo:hi], s["out"][lo:hi])
                c = torch.cuda.Event()
                c.record(self.compute)
                computed.append(c)
        with torch.cuda.stream(self.copy_out):
            for (lo, hi), c in zip(self.ranges, computed):
                self.copy_out.wait_event(c)
                o_h[lo:hi].copy_(s["out"][lo:hi], non_blocking=True)
            done = torch.cuda.Event()
            done.record(self.copy_out)
        s["free"] = done
        return done
