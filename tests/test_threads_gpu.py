"""The C ABI from several host threads at once, each on a stream of its own: the library's per-thread, per-device
state (the stream-K workspace, the reductions' scratch) and its per-device state (the SM count, the plans, the
tensor-map encoder) must hold under concurrent calls. Each thread runs the exact f32 sum, the checked u64 sum,
saxpy, a bf16 product with bias and ReLU over the planned cover, and a stream-K product (few tiles, long k), ten
rounds; every result equals the one a single thread computed first (the kernels are deterministic), and the sums
equal the oracle's."""

from __future__ import annotations

import threading

import numpy as np
import pytest
import torch

import cairn_b200
import inputs
from oracle import restated

pytestmark = pytest.mark.gpu

THREADS, ROUNDS = 4, 10


def _case(t: int, cuda):
    rng = np.random.default_rng(400 + t)
    n = 2_000_003
    x = (rng.uniform(-1, 1, n) * 2.0 ** rng.integers(-20, 20, n)).astype(np.float32)
    u = rng.integers(0, 1 << 40, n, dtype=np.uint64)
    sx, sy, a = inputs.saxpy_case(n, seed=500 + t)
    g = torch.Generator(device=cuda).manual_seed(600 + t)
    pa = torch.randn(3072, 4096, device=cuda, generator=g).bfloat16()  # planned cover (4096 columns, 12 bands)
    pb = torch.randn(4096, 4096, device=cuda, generator=g).bfloat16()
    bias = torch.randn(4096, device=cuda, generator=g) * 0.1
    ka = torch.randn(512, 8192, device=cuda, generator=g).bfloat16()  # 2 tiles, 128 k-blocks: stream-K
    kb = torch.randn(8192, 512, device=cuda, generator=g).bfloat16()
    return dict(x=torch.from_numpy(x).to(cuda), u=torch.from_numpy(u.view(np.int64)).to(cuda).view(torch.uint64),
                sx=torch.from_numpy(sx).to(cuda), sy=torch.from_numpy(sy).to(cuda), a=float(a), pa=pa, pb=pb,
                bias=bias, ka=ka, kb=kb, want_f32=np.float32(restated.sum_f32(x)).view(np.uint32),
                want_u64=int(u.sum(dtype=np.uint64)), want_saxpy=restated.saxpy(float(a), sx, sy).view(np.uint32))


def _run(c: dict) -> tuple:
    f32 = cairn_b200.reduce_sum(c["x"])
    u64 = cairn_b200.reduce_sum(c["u"])
    s = cairn_b200.saxpy(c["a"], c["sx"], c["sy"])
    p = cairn_b200.gemm(c["pa"], c["pb"], bias=c["bias"], relu=True, out_dtype=torch.bfloat16)
    k = cairn_b200.gemm(c["ka"], c["kb"], out_dtype=torch.float32)
    cairn_b200.stream_status()
    return f32, u64, s, p, k


def test_the_c_abi_from_several_threads_at_once(cuda):
    cases = [_case(t, cuda) for t in range(THREADS)]
    torch.cuda.synchronize()
    first = [_run(c) for c in cases]  # one thread, one after another: the reference bits
    for c, (f32, u64, s, _, _) in zip(cases, first):
        assert np.float32(f32).view(np.uint32) == c["want_f32"] and u64 == c["want_u64"]
        assert np.array_equal(s.cpu().numpy().view(np.uint32), c["want_saxpy"])
    failures: list[str] = []

    def work(t: int):
        c, ref = cases[t], first[t]
        stream = torch.cuda.Stream(cuda)
        try:
            with torch.cuda.stream(stream):
                for r in range(ROUNDS):
                    f32, u64, s, p, k = _run(c)
                    same = (f32 == ref[0] and u64 == ref[1] and torch.equal(s, ref[2]) and torch.equal(p, ref[3])
                            and torch.equal(k, ref[4]))
                    if not same:
                        failures.append(f"thread {t} round {r}")
        except Exception as e:  # noqa: BLE001 - reported below
            failures.append(f"thread {t}: {e!r}")

    threads = [threading.Thread(target=work, args=(t,)) for t in range(THREADS)]
    for th in threads:
        th.start()
    for th in threads:
        th.join(timeout=600)
    assert not any(th.is_alive() for th in threads)
    assert not failures, failures[:4]
