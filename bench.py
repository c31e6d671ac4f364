#!/usr/bin/env python
"""Benchmark of CAIRN's data-parallel hot path on B200, one JSON line per run (rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload gemm|gemm5|mlp|saxpy|sum_f32|sum_u64|scan]
                    [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU, NCCL)

Workloads (the default is the one the headline metric is quoted on):
  gemm     config 2: bf16 GEMM M=N=K=4096, f32 accumulate, fused bias (N-vector ~ N(0, 0.1)) + ReLU, bf16 out.
           One step = one product. At N GPUs each rank computes its own 4096-row block of an M = 4096 N product
           with the same B (the M-sharded row-block partition, no collective): weak scaling.
  gemm5    config 5: M-sharded bf16 GEMM, M = 65536, N = K = 8192, f32 out; rank r computes rows [r M/N, (r+1) M/N):
           strong scaling (total work fixed).
  mlp      config 3: a 2-layer MLP's forward + backward (batch 8192, 4096 -> 16384 -> 4096): six products and the
           fused MSE kernel per step; one replica per rank: weak scaling.
  saxpy    config 4: out = 2.5 x + y over n = 2^30 f32, range-sharded: strong scaling.
  sum_f32  config 4: `reduce +` over n = 2^30 f32 (exact sum rounded once), range-sharded; the ranks' parts meet in
           one NCCL all-gather and a combine kernel on every rank.
  sum_u64  config 4: checked `reduce +` over n = 2^30 u64 (data[i] = i), range-sharded, parts all-gathered.
  scan     the next row after reduce: `scan add_wrap parallel i in n yield x[i] into out` over n = 2^30 u32 through
           a CAIRN program built over the drop-in runtime headers (tests/dropin: the reference's own context code on
           this project's B200 machine and scan kernel); one replica per rank: weak scaling. The roofline times the
           machine's scan kernel alone.
Inputs are synthetic (seeded torch generators on the device), larger than L2 across the timed steps: every step
reads a different buffer set, or (2^30 workloads) buffers far larger than the 126 MB L2.

Timing: W untimed steps, then exactly K steps back to back between a barrier and a device synchronize, timed with
CUDA events on the launching stream (nothing recorded between steps); the max over ranks is reported. `value` is
whole-job throughput with inputs resident in HBM; `e2e` is the same metric through the C ABI from pinned host buffers
with the copies inside the timed region; `roofline` divides the dominant kernel's algorithmic work per launch by its
event-timed duration per launch (the region's time over K for a one-kernel step) and by the measured peak
(MEASURED_PEAKS.json: the burst GEMM peak for config 2's short region of 20 products, the sustained one for the long
steps of configs 3 and 5); `cpu_baseline` times the reference's own host path (the CAIRN runtime's
lane-pool code, compiled from its sources into oracle/_ref) on a bounded sample on this box's cores.
`--impl reference` runs only that CPU path, as the reference arm.
"""

from __future__ import annotations

import argparse
import ctypes as C
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

BASELINE_METRIC = "bf16 GEMM TFLOP/s & % tensor peak; reduce/saxpy HBM GB/s at 1/2/4/8 B200"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


# ---------------------------------------------------------------------------------------------------------------------
# plumbing
# ---------------------------------------------------------------------------------------------------------------------
class Dist:
    def __init__(self, gpus: int):
        import torch
        import torch.distributed as dist

        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != gpus:
            raise SystemExit(f"--gpus {gpus} but WORLD_SIZE={self.world}: launch N>1 with torchrun")
        self.dist = dist
        self.device = torch.device("cuda", self.local) if torch.cuda.is_available() else None
        if self.device is not None:
            torch.cuda.set_device(self.device)
        if self.world > 1:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=self.device)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch

        t = torch.tensor([x], dtype=torch.float64, device=self.device)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def measured_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def profile_traffic(name: str) -> int | None:
    """Per-launch DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) recorded from an ncu capture in
    profiles/<name>.md as `traffic_per_launch_bytes: N`."""
    path = ROOT / "profiles" / f"{name}.md"
    if not path.exists():
        return None
    m = re.search(r"traffic_per_launch_bytes:\s*(\d+)", path.read_text())
    return int(m.group(1)) if m else None


class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons every 50 ms; `window` keeps those inside [t0, t1]."""

    QUERY = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-i", str(index),
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (FileNotFoundError, OSError):
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 6:
                self.samples.append((time.time(), parts))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def window(self, t0: float, t1: float) -> dict:
        inside = [s for t, s in self.samples if t0 <= t <= t1]
        note = None
        if not inside and self.samples:  # a timed region shorter than the sampling period: the nearest samples
            nearest = sorted(self.samples, key=lambda ts: min(abs(ts[0] - t0), abs(ts[0] - t1)))[:3]
            inside = [s for _, s in nearest]
            note = "timed region shorter than the 50 ms sampling period: nearest samples of the same run"
        if not inside:
            why = "nvidia-smi unavailable" if self.proc is None else "no nvidia-smi samples in or near the timed region"
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "note": why}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in inside for i in range(4) if s[2 + i].lower().startswith("active")})
        out = {"sm_mhz": statistics.median(float(s[0]) for s in inside), "sm_max_mhz": float(inside[0][1]),
               "reasons": reasons, "samples": len(inside)}
        if note:
            out["note"] = note
        return out


class DeviceClock:
    """The SM clock inside a timed region, from the device itself: cairn_b200_clock_marks before and after the region
    (every SM's %clock64 and %globaltimer), each SM's cycles over nanoseconds, the median over SMs. nvidia-smi samples
    every 50 ms at best, longer than a 20-product region."""

    SLOTS = 256

    def __init__(self, dist: Dist):
        import torch

        self.lib = lib_handle()
        self.marks = [torch.zeros(2 * self.SLOTS, dtype=torch.int64, device=dist.device) for _ in range(2)]

    def mark(self, stream, which: int):
        check(self.lib.cairn_b200_clock_marks(stream.cuda_stream, self.marks[which].data_ptr(), self.SLOTS),
              "cairn_b200_clock_marks")

    def mhz(self) -> float | None:
        a, b = (m.view(-1, 2).cpu().tolist() for m in self.marks)
        rates = [(c1 - c0) / (g1 - g0) * 1000 for (c0, g0), (c1, g1) in zip(a, b) if g0 and g1 > g0 and c1 > c0]
        return statistics.median(rates) if rates else None


def time_steps(dist: Dist, stream, launch, steps: int, warmup: int, clock: DeviceClock | None = None):
    """W warm-up steps, then K steps timed on `stream` with CUDA events (a barrier and a synchronize on both
    sides). Returns (max-over-ranks ms per step, this rank's ms per step, wall t0, wall t1).

    Nothing is recorded between the steps: an event between two products would end the programmatic overlap of one
    product's set-up with the tail of the one before it (each pair kernel is launched as a programmatic dependent),
    and time a way of running the library that no caller's stream of products has (on a B200, 4096^3 with bias and
    ReLU: about 94 us per product back to back against 104-107 us with an event pair around each). The per-launch
    duration of a one-kernel step is therefore the region's time over K."""
    import torch

    for i in range(warmup):
        launch(i)
    torch.cuda.synchronize()
    dist.barrier()
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    t0 = time.time()
    if clock is not None:
        clock.mark(stream, 0)
    start.record(stream)
    for i in range(steps):
        launch(warmup + i)
    end.record(stream)
    if clock is not None:
        clock.mark(stream, 1)
    torch.cuda.synchronize()
    t1 = time.time()
    dist.barrier()
    total = start.elapsed_time(end)
    return dist.max(total) / steps, total / steps, t0, t1


def lib_handle():
    import cairn_b200

    return cairn_b200.lib()


def check(status: int, what: str):
    if status != 0:
        raise SystemExit(f"{what} failed with status {status}")


# ---------------------------------------------------------------------------------------------------------------------
# CPU baseline: the reference's own host path (oracle/_ref), or the C restatement when it was not built
# ---------------------------------------------------------------------------------------------------------------------
def cpu_kind():
    from oracle import reference

    return "reference" if reference.available() else "port"


def cpu_gemm_sample(m_total: int, n: int, k: int, budget_s: float):
    """TFLOP/s of the host multiply (cr::tensor::reference on the reference's lane pool, one lane per row of c) plus
    the bias/ReLU/bf16 epilogue, on a sample of rows sized to take about `budget_s`."""
    import numpy as np

    from oracle import reference, restated

    rng = np.random.default_rng(0)
    b = rng.integers(0, 1 << 16, k * n, dtype=np.uint16) & np.uint16(0xBFFF)  # finite bf16 patterns
    bias = (rng.standard_normal(n) * 0.1).astype(np.float32)
    kind = cpu_kind()
    rows, spent, flops = 4, 0.0, 0.0
    while spent < budget_s:
        a = rng.integers(0, 1 << 16, rows * k, dtype=np.uint16) & np.uint16(0xBFFF)
        c = np.zeros(rows * n, np.float32)
        t = time.perf_counter()
        if kind == "reference":
            acc = reference.mma_bf16_pooled(c, a, b, rows, n, k)
        else:
            acc = restated.mma("bf16", c, a, b, rows, n, k)
        restated.bias_act(acc, bias, True, rows, n)
        spent += time.perf_counter() - t
        flops += 2.0 * rows * n * k
        rows = min(rows * 2, m_total)
    cores = reference.lanes() if kind == "reference" else 1
    return flops / spent / 1e12, cores, kind, f"{int(flops / (2 * n * k))} rows of the {m_total}x{n}x{k} product"


def cpu_stream_sample(workload: str, budget_s: float):
    import numpy as np

    from oracle import reference, restated

    kind = cpu_kind()
    n = 1 << 26
    rng = np.random.default_rng(0)
    x = rng.uniform(-1, 1, n).astype(np.float32)
    y = rng.uniform(-1, 1, n).astype(np.float32)
    u = np.arange(n, dtype=np.uint64)
    w = x.view(np.uint32)
    out = np.empty_like(x)
    lib = reference if kind == "reference" else restated
    per = {"saxpy": 12, "sum_f32": 4, "sum_u64": 8, "scan": 8}[workload]
    spent, done = 0.0, 0
    while spent < budget_s:
        t = time.perf_counter()
        if workload == "scan":
            if kind == "reference":
                reference.scan_u32(w, out.view(np.uint32))
            else:
                restated.scan_u32(w)
        elif workload == "saxpy":
            if kind == "reference":
                reference.saxpy(2.5, x, y, out)
            else:
                restated.saxpy(2.5, x, y)
        elif workload == "sum_f32":
            lib.sum_f32(x)
        else:
            lib.sum_u64(u)
        spent += time.perf_counter() - t
        done += n
    cores = reference.lanes() if kind == "reference" else 1
    return done * per / spent / 1e9, cores, kind, f"{done // n} passes over 2^26 elements"


# ---------------------------------------------------------------------------------------------------------------------
# workloads
# ---------------------------------------------------------------------------------------------------------------------
class Gemm:
    """bf16 GEMM with the fused bias + ReLU + bf16 epilogue (config 2), or the M-sharded f32-out product (config 5)."""

    def __init__(self, dist: Dist, config5: bool):
        import torch

        self.torch, self.dist, self.config5 = torch, dist, config5
        if config5:
            self.m_total, self.n, self.k = 65536, 8192, 8192
            self.m = self.m_total // dist.world
            self.scaling = "strong"
        else:
            self.m, self.n, self.k = 4096, 4096, 4096
            self.m_total = self.m * dist.world
            self.scaling = "weak"
        dev = dist.device
        row0 = dist.rank * self.m
        # Enough buffer sets that consecutive steps never find their operands in the 126 MB L2.
        per_set = (self.m * self.k + self.k * self.n) * 2 + self.m * self.n * (4 if config5 else 2)
        self.sets = max(2, -(-3 * 126 * 2**20 // per_set))
        gb = torch.Generator(device=dev).manual_seed(0)
        b_std = 0.02 if config5 else 1.0
        self.a, self.b, self.out = [], [], []
        for s in range(self.sets):
            ga = torch.Generator(device=dev).manual_seed(1_000_003 * (s + 1) + row0)
            self.a.append(torch.randn(self.m, self.k, device=dev, generator=ga).to(torch.bfloat16))
            self.b.append((torch.randn(self.k, self.n, device=dev, generator=gb) * b_std).to(torch.bfloat16))
            self.out.append(torch.empty(self.m, self.n, device=dev,
                                        dtype=torch.float32 if config5 else torch.bfloat16))
        self.bias = (torch.randn(self.n, device=dev, generator=gb) * 0.1).float()
        self.lib = lib_handle()
        self.stream = torch.cuda.current_stream(dev)
        self.flops = 2.0 * self.m * self.n * self.k

    def launch(self, i: int):
        s = i % self.sets
        if self.config5:
            st = self.lib.cairn_b200_gemm(self.stream.cuda_stream, 0, self.m, self.n, self.k, self.a[s].data_ptr(), 0,
                                          self.b[s].data_ptr(), 0, self.out[s].data_ptr(), 1, None, 0)
        else:
            st = self.lib.cairn_b200_gemm(self.stream.cuda_stream, 0, self.m, self.n, self.k, self.a[s].data_ptr(), 0,
                                          self.b[s].data_ptr(), 0, self.out[s].data_ptr(), 2, self.bias.data_ptr(), 1)
        if st:
            raise SystemExit(f"cairn_b200_gemm failed with status {st}")

    def e2e(self, steps: int, warmup: int):
        """The same product from pinned host memory through cairn_b200.HostGemm (the library's host-buffer multiply:
        A's row chunks copied in, each chunk's rows of C computed as they land and copied back), every step's A in
        and its whole bf16 (or f32) result out; B and the bias stay resident on the device, as a layer's weights do
        from step to step. Steps overlap as a stream of products would. Also returns each GPU's host-link rates."""
        torch = self.torch
        from cairn_b200 import HostGemm

        a_h = [self.a[s].cpu().pin_memory() for s in range(2)]
        out_h = torch.empty(self.out[0].shape, dtype=self.out[0].dtype).pin_memory()
        hg = HostGemm(self.m, self.n, self.k, out_dtype=self.out[0].dtype, bias=not self.config5,
                      device=self.dist.device)
        bias = None if self.config5 else self.bias

        def step(i):
            done = hg.submit(a_h[i % 2], self.b[0], out_h, bias, relu=not self.config5)
            self.stream.wait_event(done)  # the timed region ends when the last result is in host memory

        ms, _, _, _ = time_steps(self.dist, self.stream, step, steps, warmup)
        h2d = a_h[0].numel() * 2
        d2h = out_h.numel() * out_h.element_size()
        self.link = {"h2d_GBps_per_gpu": h2d / (ms * 1e-3) / 1e9, "d2h_GBps_per_gpu": d2h / (ms * 1e-3) / 1e9,
                     "resident": "B and the bias (uploaded once, as weights are)"}
        return self.dist.world * self.flops / (ms * 1e-3) / 1e12, h2d, d2h


class Stream:
    """saxpy and the two `reduce +` collectors over n = 2^30 elements, range-sharded across the ranks."""

    def __init__(self, dist: Dist, workload: str, log2n: int = 30):
        import torch

        self.torch, self.dist, self.workload = torch, dist, workload
        self.n_total = 1 << log2n
        lo = self.n_total * dist.rank // dist.world
        hi = self.n_total * (dist.rank + 1) // dist.world
        self.n = hi - lo
        dev = dist.device
        g = torch.Generator(device=dev).manual_seed(0 + dist.rank)
        self.lib = lib_handle()
        self.stream = torch.cuda.current_stream(dev)
        if workload == "saxpy":
            self.x = torch.rand(self.n, device=dev, generator=g) * 2 - 1
            self.y = torch.rand(self.n, device=dev, generator=g) * 2 - 1
            self.o = torch.empty_like(self.x)
            self.bytes = 12
        elif workload == "sum_f32":
            self.x = torch.rand(self.n, device=dev, generator=g) * 2 - 1
            self.part = torch.zeros(3, dtype=torch.float64, device=dev)
            self.parts = torch.zeros(dist.world * 3, dtype=torch.float64, device=dev)
            self.total = torch.zeros(1, dtype=torch.float32, device=dev)
            self.bytes = 4
        else:
            self.x = torch.arange(lo, hi, device=dev, dtype=torch.int64).view(torch.uint64)
            self.cell = torch.zeros(1, dtype=torch.int64, device=dev)
            self.flag = torch.zeros(1, dtype=torch.int32, device=dev)
            self.cells = torch.zeros(dist.world, dtype=torch.int64, device=dev)
            self.flags = torch.zeros(dist.world, dtype=torch.int32, device=dev)
            self.bytes = 8

    def launch(self, i: int):
        lib, st, dist = self.lib, self.stream.cuda_stream, self.dist
        if self.workload == "saxpy":
            check(lib.cairn_b200_saxpy_f32(st, self.n, self.o.data_ptr(), self.x.data_ptr(), self.y.data_ptr(), 2.5),
                  "saxpy")
        elif self.workload == "sum_f32":
            if dist.world == 1:
                check(lib.cairn_b200_sum_f32(st, self.n, self.x.data_ptr(), self.total.data_ptr()), "sum")
            else:
                check(lib.cairn_b200_sum_f32_partial(st, self.n, self.x.data_ptr(), self.part.data_ptr()), "sum")
                dist.dist.all_gather_into_tensor(self.parts, self.part)
                check(lib.cairn_b200_sum_f32_combine_device(st, self.parts.data_ptr(), dist.world,
                                                            self.total.data_ptr()), "combine")
        else:
            check(lib.cairn_b200_sum_u64(st, self.n, self.x.data_ptr(), self.cell.data_ptr(), self.flag.data_ptr()),
                  "sum_u64")
            if dist.world > 1:
                dist.dist.all_gather_into_tensor(self.cells, self.cell)
                dist.dist.all_gather_into_tensor(self.flags, self.flag)

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        lib, st = self.lib, self.stream.cuda_stream
        chunk = min(self.n, 1 << 26)  # the e2e sample: 2^26 elements per rank from pinned host memory
        x_h = self.x[:chunk].cpu().pin_memory()
        x_d = self.x[:chunk]
        if self.workload == "saxpy":  # through cairn_b200.HostSaxpy: copies in, regions and copies out overlapped
            from cairn_b200 import HostSaxpy

            y_h, o_h = self.y[:chunk].cpu().pin_memory(), torch.empty(chunk, dtype=torch.float32).pin_memory()
            hs = HostSaxpy(chunk, device=self.dist.device)

            def step(i):
                self.stream.wait_event(hs.submit(2.5, x_h, y_h, o_h))

            h2d, d2h = 8 * chunk, 4 * chunk
        else:
            res = torch.empty(1, dtype=torch.int64).pin_memory()
            cell = torch.zeros(1, dtype=torch.int64, device=self.dist.device)
            flag = torch.zeros(1, dtype=torch.int32, device=self.dist.device)

            def step(i):
                x_d.copy_(x_h, non_blocking=True)
                if self.workload == "sum_f32":
                    check(lib.cairn_b200_sum_f32(st, chunk, x_d.data_ptr(), cell.data_ptr()), "sum")
                else:
                    check(lib.cairn_b200_sum_u64(st, chunk, x_d.data_ptr(), cell.data_ptr(), flag.data_ptr()), "sum")
                res.copy_(cell, non_blocking=True)

            h2d, d2h = x_h.numel() * x_h.element_size(), 8
        ms, _, _, _ = time_steps(self.dist, self.stream, step, steps, warmup)
        return self.dist.world * chunk * self.bytes / (ms * 1e-3) / 1e9, h2d, d2h


EMITTED = ROOT / "tests" / "dropin" / "_build" / "libhotpath.so"
SCAN_PROBE = ROOT / "tests" / "dropin" / "_build" / "libscanprobe.so"


class Scan:
    """The drop-in machine's device scan over n = 2^30 u32 (add_wrap), through the compiler-emitted CAIRN library
    built over include/cairn_b200/runtime (cf_wscan: `scan add_wrap out parallel i in n yield x[i]`, the reference's
    scan_into, which scans into its arena and copies to out, then waits for its stream), and the machine's scan kernel
    alone (tests/dropin/scan_probe.cu's b200_scan_u32) for the roofline. 8 algorithmic bytes per element."""

    def __init__(self, dist: Dist, log2n: int = 30):
        import torch

        self.torch, self.dist = torch, dist
        self.n = 1 << log2n
        dev = dist.device
        g = torch.Generator(device=dev).manual_seed(0 + dist.rank)
        self.x = torch.randint(-2**31, 2**31 - 1, (self.n,), device=dev, dtype=torch.int32, generator=g)
        self.out = torch.empty_like(self.x)
        lib_handle()  # the program links libcairn_b200.so: load it from the tree first
        h = C.CDLL(str(EMITTED))
        h.cf_wscan.restype, h.cf_wscan.argtypes = None, [C.c_size_t, C.c_void_p, C.c_void_p]
        h.cairn_hotpath_device_stream.restype, h.cairn_hotpath_device_stream.argtypes = None, [C.c_void_p]
        probe = C.CDLL(str(SCAN_PROBE))
        probe.b200_scan_u32_scratch.restype, probe.b200_scan_u32_scratch.argtypes = C.c_size_t, [C.c_size_t]
        probe.b200_scan_u32.restype = None
        probe.b200_scan_u32.argtypes = [C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p, C.c_void_p]
        self.h, self.probe = h, probe
        self.temp = torch.empty(probe.b200_scan_u32_scratch(self.n), dtype=torch.uint8, device=dev)
        self.stream = torch.cuda.current_stream(dev)
        h.cairn_hotpath_device_stream(self.stream.cuda_stream)  # the program's work on the bench's stream
        self.bytes = 8
        self.scaling = "weak"

    def launch(self, i: int):
        self.h.cf_wscan(self.n, self.out.data_ptr(), self.x.data_ptr())

    def kernel_alone(self, i: int):
        self.probe.b200_scan_u32(self.stream.cuda_stream, self.n, self.out.data_ptr(), self.x.data_ptr(),
                                 self.temp.data_ptr())

    def e2e(self, steps: int, warmup: int):
        torch = self.torch
        chunk = min(self.n, 1 << 26)  # the e2e sample: 2^26 elements from pinned host memory
        x_h = self.x[:chunk].cpu().pin_memory()
        o_h = torch.empty(chunk, dtype=torch.int32).pin_memory()
        x_d, o_d = self.x[:chunk], self.out[:chunk]

        def step(i):
            x_d.copy_(x_h, non_blocking=True)
            self.h.cf_wscan(chunk, o_d.data_ptr(), x_d.data_ptr())
            o_h.copy_(o_d, non_blocking=True)

        ms, _, _, _ = time_steps(self.dist, self.stream, step, steps, warmup)
        return self.dist.world * chunk * self.bytes / (ms * 1e-3) / 1e9, 4 * chunk, 4 * chunk


class Mlp:
    """Config 3: one forward + backward of a 2-layer MLP (batch 8192, 4096 -> 16384 -> 4096, bf16 weights ~ N(0, 0.02),
    inputs ~ N(0, 1), ReLU, MSE against an N(0, 1) target): six products and the fused loss kernel per step.
    Replicas only at N GPUs (each rank runs its own step): weak scaling."""

    def __init__(self, dist: Dist):
        import torch

        from cairn_b200 import mlp

        self.torch, self.dist, self.mlp = torch, dist, mlp
        self.B, self.D, self.H, self.O = 8192, 4096, 16384, 4096
        dev = dist.device
        g = torch.Generator(device=dev).manual_seed(0 + dist.rank)
        self.x = torch.randn(self.B, self.D, device=dev, generator=g).bfloat16()
        self.w1 = (torch.randn(self.D, self.H, device=dev, generator=g) * 0.02).bfloat16()
        self.w2 = (torch.randn(self.H, self.O, device=dev, generator=g) * 0.02).bfloat16()
        self.t = torch.randn(self.B, self.O, device=dev, generator=g)
        self.ws = mlp.MLPWorkspace(self.B, self.D, self.H, self.O, dev)
        self.stream = torch.cuda.current_stream(dev)
        self.flops = mlp.mlp_flops(self.B, self.D, self.H, self.O)
        self.scaling = "weak"

    def launch(self, i: int):
        self.mlp.mlp_step(self.x, self.w1, self.w2, self.t, self.ws, self.stream.cuda_stream)

    def e2e(self, steps: int, warmup: int):
        """The step through mlp.step_from_host: this step's batch and target copied in from pinned host memory (on the
        feed's stream, while the step before computes) and the loss read back; the weights stay resident as in
        training."""
        torch = self.torch
        x_h, t_h = self.x.cpu().pin_memory(), self.t.cpu().pin_memory()
        loss_h = torch.empty(1, dtype=torch.float32).pin_memory()
        feed = self.mlp.HostFeed(self.B, self.D, self.O, self.dist.device)

        def step(i):
            self.mlp.step_from_host(feed, x_h, t_h, self.w1, self.w2, self.ws, loss_h, self.stream)

        ms, _, _, _ = time_steps(self.dist, self.stream, step, steps, warmup)
        return self.dist.world * self.flops / (ms * 1e-3) / 1e12, x_h.numel() * 2 + t_h.numel() * 4, 4


def cpu_mlp_sample(budget_s: float):
    """TFLOP/s of config 3's step on the host by the reference's own code, at a reduced shape (batch 32,
    256 -> 1024 -> 256): its dense layers and the adjoints `derive grad` writes for them and for mse
    (oracle/_ref/libmlp_grad.so, oracle/grad/mlp_grad.cairn through the reference's compiler; sequential f32 loops,
    one core, the only backward the reference has), timed around those compiled calls; the relu and bf16 roundings
    between them run in numpy outside the clock. Credited with the step's six products (the reference's adjoints
    run each layer's forward again, which the credit leaves out). Without the reference build, the C restatement."""
    import numpy as np

    from oracle import reference, restated

    def narrow(v):  # nearest-even bf16 of finite f32 values as f32 patterns, as cr::fp::narrow rounds
        u = np.asarray(v, np.float32).view(np.uint32).astype(np.uint64)
        return (((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint32) << 16).view(np.float32)

    B, D, H, O = 32, 256, 1024, 256
    rng = np.random.default_rng(0)
    xf = narrow(rng.standard_normal(B * D))
    w1f = narrow(rng.standard_normal(D * H) * 0.02)
    w2f = narrow(rng.standard_normal(H * O) * 0.02)
    t = rng.standard_normal(B * O).astype(np.float32)
    flops_step = 2.0 * B * H * (3 * D + 3 * O)
    spent, flops = 0.0, 0.0
    if reference.grad_available():

        while spent < budget_s:
            t0 = time.perf_counter()
            pre = reference.dense(xf, w1f, B, D, H)
            spent += time.perf_counter() - t0
            hf = narrow(np.maximum(pre, 0))
            t0 = time.perf_counter()
            y = reference.dense(hf, w2f, B, H, O)
            _, dyf = reference.mse_grad(y, t)
            spent += time.perf_counter() - t0
            dy = narrow(dyf)
            t0 = time.perf_counter()
            dh_pre, _ = reference.dense_grad(hf, w2f, dy, B, H, O)
            spent += time.perf_counter() - t0
            dh = narrow(np.where(pre > 0, dh_pre, np.float32(0)))
            t0 = time.perf_counter()
            reference.dense_grad(xf, w1f, dh, B, D, H)
            spent += time.perf_counter() - t0
            flops += flops_step
        kind = "reference"
    else:
        bits = [(v.view(np.uint32) >> 16).astype(np.uint16) for v in (xf, w1f, w2f)]
        while spent < budget_s:
            t0 = time.perf_counter()
            restated.mlp_step(*bits, t, B, D, H, O)
            spent += time.perf_counter() - t0
            flops += flops_step
        kind = "port"
    return flops / spent / 1e12, 1, kind, f"{int(flops / flops_step)} steps at batch 32, 256 -> 1024 -> 256"


def scaling_legs(dist: Dist) -> dict:
    """The sharded designs of BASELINE configs 5 and 4, run by every rank after the headline at every N so that the
    scaling run records them: config 5's M-sharded product (M = 65536 split into N row blocks, N = K = 8192, f32 out;
    strong scaling, no collective) with its optional all-gather of C timed apart, and the range-sharded f32 and u64
    sums over n = 2^30 with their all-gather of the ranks' parts inside each step. Times are device times, the max
    over ranks (CUDA events between barriers, as the headline's)."""
    import torch

    from cairn_b200 import shard

    out: dict = {}
    g5 = Gemm(dist, config5=True)
    ms, launch_ms, _, _ = time_steps(dist, g5.stream, g5.launch, 5, 3)
    out["config5"] = {"rows_per_gpu": g5.m, "ms_per_product": ms, "TFLOP/s": dist.world * g5.flops / (ms * 1e-3) / 1e12,
                      "per_gpu_TFLOP/s": g5.flops / (launch_ms * 1e-3) / 1e12, "scaling": "strong"}
    if dist.world > 1:
        whole = torch.empty(g5.m_total, g5.n, dtype=torch.float32, device=dist.device)
        gms, _, _, _ = time_steps(dist, g5.stream, lambda i: shard.gather_rows(g5.out[0], g5.m_total, out=whole), 3, 1)
        received = (g5.m_total - g5.m) * g5.n * 4
        out["config5"]["allgather_ms"] = gms
        out["config5"]["allgather_GBps_per_gpu"] = received / (gms * 1e-3) / 1e9
        out["config5"]["allgather_note"] = "NCCL all-gather of the f32 C row blocks, received bytes per GPU"
        del whole
    del g5
    torch.cuda.empty_cache()
    for w in ("sum_f32", "sum_u64"):
        st = Stream(dist, w, 30)
        ms, _, _, _ = time_steps(dist, st.stream, st.launch, 10, 3)
        out[w] = {"n": st.n_total, "ms_per_step": ms, "GB/s": st.n_total * st.bytes / (ms * 1e-3) / 1e9,
                  "scaling": "strong", "exchange": "parts all-gathered every step" if dist.world > 1 else "none"}
        del st
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------------------------------------------------
REF_DEVICE = ROOT / "baseline" / "_ref" / "libhotpath_ref.so"

# The compiler-emitted entries of tests/dropin/programs/hotpath.cairn timed on each machine, with their C types and
# algorithmic bytes per element (regions and collectors) or None (the multiply).
MACHINE_ENTRIES = {
    "cq_saxpy": (None, ["p", "z", "p", "p", "p", "f"], 12), "cq_saxpy4": (None, ["p", "z", "p", "p", "p", "f"], 12),
    "cq_blur": (None, ["p", "z", "p", "p"], 8), "cf_dsum": ("f", ["z", "p"], 4), "cf_usum": ("u64", ["z", "p"], 8),
    "cf_wscan": (None, ["z", "p", "p"], 8), "cq_gemm": (None, ["p", "z", "z", "z", "z", "p", "z", "p", "z", "p"], None),
    "cairn_hotpath_device_stream": (None, ["p"], None),
}


def machine_measure(args) -> dict:
    """One machine's timings of the compiler-emitted program (tests/dropin/programs/hotpath.cairn): `args.machine` is
    tests/dropin/_build/libhotpath.so (this project's B200 machine under the drop-in headers) or
    baseline/_ref/libhotpath_ref.so (the same emitted source over the reference's own headers: its lane kernels, CUB
    collectors and WMMA multiply). Runs in a process of its own (two builds of one program would share template
    symbols). Inputs resident in HBM, n = 2^log2n; every entry runs on the bench's stream (bound with
    cairn_hotpath_device_stream for the cf_ ones), each timed over 10 calls with CUDA events after 2 untimed ones.
    cf_ entries wait for their stream and copy their total back, on either machine alike."""
    import torch

    types = {"p": C.c_void_p, "z": C.c_size_t, "f": C.c_float, "u64": C.c_uint64, None: None}
    h = C.CDLL(str(args.machine))
    for name, (res, argt, _) in MACHINE_ENTRIES.items():
        f = getattr(h, name)
        f.restype, f.argtypes = types[res], [types[a] for a in argt]
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    h.cairn_hotpath_device_stream(stream.cuda_stream)
    st = stream.cuda_stream
    g = torch.Generator(device=dev).manual_seed(0)

    def events(fn, steps: int = 10, warmup: int = 2) -> float:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    out: dict = {"n": 1 << args.log2n}
    n = 1 << args.log2n
    x = torch.rand(n, device=dev, generator=g) * 2 - 1
    y = torch.rand(n, device=dev, generator=g) * 2 - 1
    o = torch.empty_like(x)
    runs = {
        "saxpy": lambda: h.cq_saxpy(st, n, o.data_ptr(), x.data_ptr(), y.data_ptr(), 2.5),
        "saxpy4": lambda: h.cq_saxpy4(st, n, o.data_ptr(), x.data_ptr(), y.data_ptr(), 2.5),
        "blur": lambda: h.cq_blur(st, n, o.data_ptr(), x.data_ptr()),
        "dsum": lambda: h.cf_dsum(n, x.data_ptr()),
        "wscan": lambda: h.cf_wscan(n, o.data_ptr(), x.data_ptr()),
    }
    per = {"saxpy": 12, "saxpy4": 12, "blur": 8, "dsum": 4, "wscan": 8}
    for name, fn in runs.items():
        ms = events(fn)
        out[name] = {"GB/s": n * per[name] / (ms * 1e-3) / 1e9, "ms": ms}
    del y
    u = torch.arange(n, device=dev, dtype=torch.int64)
    ms = events(lambda: h.cf_usum(n, u.data_ptr()))
    out["usum"] = {"GB/s": n * 8 / (ms * 1e-3) / 1e9, "ms": ms}
    del u, x, o
    if args.workload in ("gemm", "gemm5"):
        m, nn, k = (4096, 4096, 4096) if args.workload == "gemm" else (65536, 8192, 8192)
        a = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        b = (torch.randn(k, nn, device=dev, generator=g) * (1.0 if args.workload == "gemm" else 0.02)).to(torch.bfloat16)
        c = torch.zeros(m, nn, device=dev)
        ms = events(lambda: h.cq_gemm(st, m, nn, k, m * nn, c.data_ptr(), m * k, a.data_ptr(), k * nn, b.data_ptr()),
                    3 if args.workload == "gemm5" else 10, 1)
        out["gemm"] = {"TFLOP/s": 2.0 * m * nn * k / (ms * 1e-3) / 1e12, "ms": ms, "shape": [m, nn, k]}
    h.cairn_hotpath_device_stream(None)
    return out


def machine_leg(args, lib: Path) -> dict:
    """machine_measure in a fresh process (python bench.py --machine-measure LIB ...), or why there is none."""
    if not lib.exists():
        return {"unavailable": f"{lib.relative_to(ROOT)} is not built (it needs the CAIRN reference's compiler)"}
    cmd = [sys.executable, str(Path(__file__).resolve()), "--machine-measure", str(lib), "--workload", args.workload,
           "--log2n", str(args.log2n)]
    try:
        done = subprocess.run(cmd, capture_output=True, text=True, timeout=900)
    except subprocess.TimeoutExpired:
        return {"unavailable": f"{lib.name} did not finish within 900 s"}
    lines = [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
    if done.returncode != 0 or not lines:
        return {"unavailable": f"{lib.name} exited {done.returncode}: {done.stderr[-300:]}"}
    return json.loads(lines[-1])


def dropin_report(args) -> tuple[dict, dict | None]:
    """The compiler-emitted program on both machines, and the reference machine's figure for this workload (the
    reference's own CUDA path on this GPU: its WMMA multiply, lane kernel, CUB collectors), or None."""
    ours, ref = machine_leg(args, EMITTED), machine_leg(args, REF_DEVICE)
    report = {"program": "tests/dropin/programs/hotpath.cairn, emitted by the reference's compiler; the same "
                         "emitted C++ built over the drop-in headers (b200) and over the reference's own (reference)",
              "b200": ours, "reference": ref}
    if "unavailable" in ref:
        return report, ref
    key = {"gemm": "gemm", "gemm5": "gemm", "saxpy": "saxpy", "sum_f32": "dsum", "sum_u64": "usum",
           "scan": "wscan"}.get(args.workload)
    if key is None or key not in ref:
        return report, {"unavailable": "the reference's derive-grad backward runs on the host only, and its device "
                                       "multiply takes no transposed operand"}
    unit = "TFLOP/s" if key == "gemm" else "GB/s"
    what = {"gemm": "the reference's mma_unordered (cr::tensor::launch: WMMA 16x16x16, 64 x 64 tiles), f32 C += A B "
                    "(it has no fused bias/ReLU epilogue)",
            "saxpy": "cr::gpu::run of out[i] = a x[i] + y[i] (the reference's lane kernel)",
            "dsum": "reduce_on<float> over CUB's DeviceReduce (total copied back and awaited)",
            "usum": "reduce_on<Sum<u64>> over CUB's DeviceReduce (total copied back and awaited)",
            "wscan": "scan_into over CUB's DeviceScan (the reference context's scan, then its copy pass)"}[key]
    return report, {"value": ref[key][unit], "unit": unit, "ms": ref[key]["ms"], "what": what}


def reference_arm(args, dist: Dist) -> None:
    """The reference's own CPU implementation of the path (the CAIRN runtime's host code, oracle/_ref) on this box's
    host cores, rank 0 only, each step a bounded sample of the workload."""
    if dist.rank != 0:
        return
    from oracle import reference

    budget = max(0.2, min(5.0, 90.0 / max(1, args.steps + args.warmup)))
    if args.workload == "mlp":
        for _ in range(args.warmup):
            cpu_mlp_sample(budget / 4)
        vals = [cpu_mlp_sample(budget) for _ in range(args.steps)]
        unit, sample = "TFLOP/s", vals[-1][3]
    elif args.workload in ("gemm", "gemm5"):
        m, n, k = (4096, 4096, 4096) if args.workload == "gemm" else (65536, 8192, 8192)
        for _ in range(args.warmup):
            cpu_gemm_sample(m, n, k, budget / 4)
        vals = [cpu_gemm_sample(m, n, k, budget) for _ in range(args.steps)]
        unit, sample = "TFLOP/s", vals[-1][3]
    else:
        for _ in range(args.warmup):
            cpu_stream_sample(args.workload, budget / 4)
        vals = [cpu_stream_sample(args.workload, budget) for _ in range(args.steps)]
        unit, sample = "GB/s", vals[-1][3]
    value = statistics.median(v[0] for v in vals)
    cores, kind = vals[-1][1], vals[-1][2]
    line = {"metric": BASELINE_METRIC, "value": value, "unit": unit, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": None, "higher_is_better": True,
            "scaling": "weak" if args.workload in ("gemm", "mlp") else "strong", "vs_baseline": None,
            "dtype": "bf16" if args.workload in ("gemm", "gemm5", "mlp") else
                     ("f32" if args.workload != "sum_u64" else "u64"),
            "data": "synthetic", "config": config_of(args, dist),
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": kind,
                             "sample": f"per step: {sample}"},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    if args.workload == "scan":
        line["scaling"], line["dtype"] = "weak", "u32"
    if not reference.available():
        line["note"] = "oracle/_ref not built on this box: the C restatement of the reference's host path ran"
    print(json.dumps(line), flush=True)


def config_of(args, dist: Dist) -> dict:
    w = args.workload
    if w == "gemm":
        return {"workload": "config 2: bf16 GEMM 4096^3, fused bias + ReLU, bf16 out", "m": 4096 * dist.world,
                "n": 4096, "k": 4096, "rows_per_gpu": 4096, "parallelism": f"row-block x{dist.world}",
                "l2": "inputs rotate over buffer sets larger than L2"}
    if w == "mlp":
        return {"workload": "config 3: 2-layer MLP forward + backward (6 products + fused MSE)", "batch": 8192,
                "dims": [4096, 16384, 4096], "parallelism": f"replicas x{dist.world}",
                "l2": "operands far larger than L2"}
    if w == "gemm5":
        return {"workload": "config 5: M-sharded bf16 GEMM, f32 out", "m": 65536, "n": 8192, "k": 8192,
                "parallelism": f"row-block x{dist.world}", "l2": "inputs rotate over buffer sets larger than L2"}
    if w == "scan":
        return {"workload": f"drop-in scan: add_wrap over n = 2^{args.log2n} u32 (next row after reduce)",
                "n": 1 << args.log2n, "parallelism": f"replicas x{dist.world}", "l2": "inputs larger than L2"}
    return {"workload": f"config 4: {w} over n = 2^{args.log2n}", "n": 1 << args.log2n,
            "parallelism": f"range x{dist.world}", "l2": "inputs larger than L2"}


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--workload", default="gemm",
                    choices=["gemm", "gemm5", "mlp", "saxpy", "sum_f32", "sum_u64", "scan"])
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--log2n", type=int, default=30, help="saxpy/sum size 2^log2n (BASELINE: 30; smaller for ncu)")
    ap.add_argument("--no-reference-device", action="store_true",
                    help="skip the drop-in legs (the emitted program on both machines, timed in subprocesses)")
    ap.add_argument("--no-scaling-legs", action="store_true",
                    help="skip the default line's config-5 and sharded-sum legs (run at every N)")
    ap.add_argument("--machine-measure", default=None, help=argparse.SUPPRESS)  # that subprocess
    args = ap.parse_args()
    if args.machine_measure:
        args.machine = args.machine_measure
        print(json.dumps(machine_measure(args)), flush=True)
        return
    defaults = {"gemm": (20, 5), "gemm5": (50, 5), "mlp": (40, 5), "saxpy": (100, 5), "sum_f32": (200, 5),
                "sum_u64": (100, 5), "scan": (50, 5)}
    d_steps, d_warm = defaults[args.workload] if args.impl == "ours" else (5, 1)
    args.steps = args.steps if args.steps is not None else d_steps
    args.warmup = args.warmup if args.warmup is not None else d_warm
    if args.impl == "ours" and args.warmup < 3:
        args.warmup = 3  # the contract's least warm-up

    dist = Dist(args.gpus)
    if args.impl == "reference":
        reference_arm(args, dist)
        dist.close()
        return
    import torch

    sampler = ClockSampler(dist.local)  # started before the set-up, so it is sampling when the timed region begins
    if args.workload.startswith("gemm"):
        wl = Gemm(dist, args.workload == "gemm5")
    elif args.workload == "mlp":
        wl = Mlp(dist)
    elif args.workload == "scan":
        if not EMITTED.exists():
            sampler.stop()
            if dist.rank == 0:
                print(json.dumps({"metric": BASELINE_METRIC, "workload": "scan", "unavailable":
                                  "tests/dropin/_build/libhotpath.so is not built (it needs the CAIRN reference's "
                                  "compiler, present where __graft_entry__.build() ran)"}), flush=True)
            dist.close()
            return
        wl = Scan(dist, args.log2n)
    else:
        wl = Stream(dist, args.workload, args.log2n)
    peaks, peak_source = measured_peaks()
    device_clock = DeviceClock(dist)
    ms, launch_ms, t0, t1 = time_steps(dist, wl.stream, wl.launch, args.steps, args.warmup, device_clock)
    clocks = sampler.window(t0, t1)
    sampler.stop()
    clocks["sm_mhz_in_region"] = device_clock.mhz()
    clocks["in_region_note"] = "each SM's %clock64 cycles over %globaltimer ns across the timed region, median over SMs"
    if isinstance(wl, Scan):  # the roofline's kernel: the machine's scan alone, without the context's copy pass
        _, launch_ms, _, _ = time_steps(dist, wl.stream, wl.kernel_alone, args.steps, args.warmup)
    stat = lib_handle().cairn_b200_stream_status(wl.stream.cuda_stream)
    if stat:
        raise SystemExit(f"device status {stat} after the timed steps")
    e2e_val, h2d, d2h = wl.e2e(max(3, min(args.steps, 20)), 3)

    if isinstance(wl, (Gemm, Mlp)):
        value = dist.world * wl.flops / (ms * 1e-3) / 1e12
        unit, bound, dtype = "TFLOP/s", "tensor", "bf16"
        # an MLP step is six equal products and a short loss kernel: the products are credited with the whole step
        achieved = wl.flops / (launch_ms * 1e-3) / 1e12
        long_step = isinstance(wl, Mlp) or args.workload == "gemm5"
        peak = peaks.get("bf16_tflops_sustained" if long_step else "bf16_tflops", FALLBACK_PEAKS["bf16_tflops"])
        kernel = "tc_gemm_pair_kernel"
        traffic = profile_traffic({"gemm": "gemm_pair_bf16_4096_bias_relu", "gemm5": "gemm_bf16_config5",
                                   "mlp": "mlp_step_config3"}[args.workload])
    else:
        per_rank_bytes = wl.n * wl.bytes
        value = dist.world * per_rank_bytes / (ms * 1e-3) / 1e9
        unit, bound = "GB/s", "hbm"
        dtype = {"saxpy": "f32", "sum_f32": "f32", "sum_u64": "u64", "scan": "u32"}[args.workload]
        achieved = per_rank_bytes / (launch_ms * 1e-3) / 1e9
        peak = peaks.get("hbm_gbs", FALLBACK_PEAKS["hbm_gbs"])
        kernel = {"saxpy": "saxpy_vec_kernel", "sum_f32": "sum_f32_kernel", "sum_u64": "sum_u64_kernel",
                  "scan": "scan_kernel"}[args.workload]
        traffic = profile_traffic(f"{args.workload}_2p30")

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        if isinstance(wl, Mlp):
            v, cores, kind, sample = cpu_mlp_sample(12.0)
        elif isinstance(wl, Gemm):
            v, cores, kind, sample = cpu_gemm_sample(wl.m, wl.n, wl.k, 12.0)
        else:
            v, cores, kind, sample = cpu_stream_sample(args.workload, 12.0)
        cpu = {"value": v, "unit": unit, "cores": cores, "kind": kind, "sample": sample}

    refdev = dropin = None
    if dist.rank == 0 and dist.world == 1 and not args.no_reference_device:
        dropin, refdev = dropin_report(args)
    link = getattr(wl, "link", None)
    launches = args.steps * (7 if isinstance(wl, Mlp) else 2 if isinstance(wl, Scan) else
                             1 if isinstance(wl, Gemm) or args.workload != "sum_f32" or dist.world == 1 else 2)
    scaling_kind = wl.scaling if isinstance(wl, (Gemm, Mlp, Scan)) else "strong"
    long_step = isinstance(wl, Mlp) or args.workload == "gemm5"
    scaling = None
    if args.workload == "gemm" and not args.no_scaling_legs:
        del wl
        torch.cuda.empty_cache()
        scaling = scaling_legs(dist)

    line = {
        "metric": BASELINE_METRIC, "value": value, "unit": unit, "n_gpus": dist.world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
        "scaling": scaling_kind, "vs_baseline": None,
        "dtype": dtype,
        "data": "synthetic (seeded device generators; random-init operands of the configs' shapes and distributions)",
        "config": config_of(args, dist),
        "roofline": {"bound": bound, "kernel": kernel, "achieved": achieved, "peak": peak, "unit": unit,
                     "frac": achieved / peak,
                     "peak_source": f"{peak_source} ({'hbm_gbs' if bound == 'hbm' else ('bf16_tflops_sustained: a long step' if long_step else 'bf16_tflops burst')})",
                     "traffic": traffic},
        "cpu_baseline": cpu,
        "reference_on_b200": refdev,
        "dropin_machines": dropin,
        "clocks": clocks,
        "e2e": {"value": e2e_val, "unit": unit, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                **({"link": link} if link else {})},
        "gpu_launches": launches,
    }
    if scaling is not None:
        line["scaling_legs"] = scaling
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    dist.close()


if __name__ == "__main__":
    main()
