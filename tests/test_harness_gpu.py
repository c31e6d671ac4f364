"""KernelBench submissions that the reference compiler exported over the drop-in headers (`cairn export --harness
kernelbench`, built by tests/dropin/build_emitted.py build_harnesses from tests/dropin/harness/): each
tests/dropin/_build/harness/<name>/model_new.py embeds the runtime headers it was exported with, checks their hashes,
and builds the program and its torch binding with load_inline when it is first imported.

Each submission runs in a child process of its own (the three build side by side): the child imports it, checks that
the embedded region header is this machine's, calls ModelNew.forward on seeded inputs and saves its outputs;
the test compares them with the oracle, bit for bit. The u64 sum's child ends by summing past 2^64, which the
reference's checked sum (cr::Sum::checked, cairn_runtime.hpp:158-166) turns into std::abort on the host once its
kernels have finished."""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
HARNESS = ROOT / "tests" / "dropin" / "_build" / "harness"
NAMES = ("saxpy4", "blur", "usum")

SAXPY_SIZES = (0, 1, 3, 4, 5, 1023, 4096 * 37 + 3, 4_194_307)
BLUR_SIZES = (1, 4, 5, 129, 100_003, 4_194_305)
USUM_SIZES = (0, 1, 2049, 1_000_003)


def saxpy_case(n: int, shifted: bool):
    rng = np.random.default_rng(n * 2 + shifted)
    x = rng.uniform(-4, 4, n + 1).astype(np.float32)
    y = rng.uniform(-4, 4, n).astype(np.float32)
    return (x[1:] if shifted else x[:n]), y, float(np.float32(rng.uniform(-3, 3)))


def blur_case(n: int):
    return np.random.default_rng(n + 70).uniform(-1, 1, n).astype(np.float32)


def usum_random(n: int):
    return np.random.default_rng(n).integers(0, 1 << 40, n, dtype=np.uint64)


def _child(name: str, out: str) -> None:
    """Imports one submission, runs its cases on cuda:0 and saves what it returned to `out` (an .npz)."""
    import importlib.util

    import torch

    spec = importlib.util.spec_from_file_location(f"kb_{name}", HARNESS / name / "model_new.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    model = module.ModelNew().cuda()
    dev = torch.device("cuda", 0)
    saved = {"machine": np.array(["CAIRN_B200_MACHINE" in module._HEADERS["cairn_gpu.hpp"]]),
             "extension": np.array([module._cairn.__file__])}
    if name == "saxpy4":
        for n in SAXPY_SIZES:
            for shifted in (False, True):
                x, y, a = saxpy_case(n, shifted)
                buf = torch.zeros(n + 1, dtype=torch.float32, device=dev)
                xd = buf[1:] if shifted else buf[:n]  # shifted: 4 bytes past a 16-byte boundary
                xd.copy_(torch.from_numpy(x.copy()))
                saved[f"{n}/{int(shifted)}"] = model(xd, torch.from_numpy(y).to(dev), a).cpu().numpy()
    elif name == "blur":
        for n in BLUR_SIZES:
            saved[str(n)] = model(torch.from_numpy(blur_case(n)).to(dev)).cpu().numpy()
    else:
        def total(x: np.ndarray) -> int:
            t = torch.from_numpy(x.view(np.int64)).to(dev).view(torch.uint64)
            return int(model(t).view(torch.int64).cpu().numpy().view(np.uint64)[0])

        for n in USUM_SIZES:
            saved[f"iota/{n}"] = np.array([total(np.arange(n, dtype=np.uint64))], np.uint64)
        saved["random"] = np.array([total(usum_random(3_000_001))], np.uint64)
        np.savez(out, **saved)
        torch.cuda.synchronize()
        print("overflow next", flush=True)
        total(np.array([1 << 63, 1 << 63, 5], np.uint64))  # aborts on the host
        print("no trap", flush=True)
        return
    torch.cuda.synchronize()
    np.savez(out, **saved)


@pytest.fixture(scope="module")
def runs(tmp_path_factory, cuda):
    missing = [n for n in NAMES if not (HARNESS / n / "model_new.py").is_file()]
    if missing:
        pytest.skip(f"tests/dropin/_build/harness is not built (it needs the CAIRN reference's compiler): {missing}")
    tmp = tmp_path_factory.mktemp("harness")
    procs = {}
    for name in NAMES:
        env = dict(os.environ, TORCH_EXTENSIONS_DIR=str(tmp / "ext" / name))
        procs[name] = subprocess.Popen([sys.executable, __file__, name, str(tmp / f"{name}.npz")], cwd=str(tmp),
                                       env=env, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)
    done = {}
    for name, p in procs.items():
        try:
            stdout, stderr = p.communicate(timeout=900)
        except subprocess.TimeoutExpired:
            p.kill()
            stdout, stderr = p.communicate()
        done[name] = (p.returncode, stdout, stderr, tmp / f"{name}.npz")
    return done


def _load(runs, name: str, rc: int = 0):
    code, stdout, stderr, path = runs[name]
    assert code == rc, (name, code, stdout[-2000:], stderr[-4000:])
    saved = np.load(path)
    assert bool(saved["machine"][0]), f"{name}: the embedded cairn_gpu.hpp is not the B200 machine"
    assert str(saved["extension"][0]).endswith(".so")
    return saved


def test_exported_vector_region_matches_the_oracle(runs):
    from oracle import restated

    saved = _load(runs, "saxpy4")
    for n in SAXPY_SIZES:
        for shifted in (False, True):
            x, y, a = saxpy_case(n, shifted)
            got = saved[f"{n}/{int(shifted)}"]
            assert got.shape == (n,)
            assert np.array_equal(got.view(np.uint32), restated.saxpy(a, x, y).view(np.uint32)), (n, shifted)


def _blur(x: np.ndarray) -> np.ndarray:
    """blur's body (tests/dropin/harness/regions.cairn) in f32, in source order and with no fused multiply-add."""
    want = x.copy()
    if x.size >= 5:
        two, three = np.float32(2.0), np.float32(3.0)
        mid = x[:-4] + x[1:-3] * two
        mid = mid + x[2:-2] * three
        mid = mid + x[3:-1]
        want[2:-2] = mid + x[4:]
    return want


def test_exported_staged_region_matches_the_oracle(runs):
    saved = _load(runs, "blur")
    for n in BLUR_SIZES:
        assert np.array_equal(saved[str(n)].view(np.uint32), _blur(blur_case(n)).view(np.uint32)), n


def test_exported_checked_sum_and_its_trap(runs):
    code, stdout, _, _ = runs["usum"]
    saved = _load(runs, "usum", rc=-6)
    assert "overflow next" in stdout and "no trap" not in stdout
    for n in USUM_SIZES:
        assert int(saved[f"iota/{n}"][0]) == n * (n - 1) // 2, n
    assert int(saved["random"][0]) == int(sum(int(v) for v in usum_random(3_000_001)))


if __name__ == "__main__":
    _child(sys.argv[1], sys.argv[2])
