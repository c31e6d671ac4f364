"""Builds tests/dropin/emitted_program.cu into tests/dropin/_build/libemitted.so: the CAIRN runtime headers from the
reference tree given on the command line, with include/cairn_b200/runtime ahead of them, so the program's runtime
calls land on the B200 machine and libcairn_b200.so. The flags are the reference toolchain's device flags
(projects/toolchain.py:184-200: C++20, -O3, --fmad=false, --extended-lambda, --expt-relaxed-constexpr), for sm_100a.

    python tests/dropin/build_emitted.py <cairn source tree>/src/cairn/runtime

It also builds the same program over the reference's headers alone into baseline/_ref/libemitted_ref.so (see
REF_DEVICE_OUT).
"""

from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build" / "libemitted.so"
# The same program over the reference's runtime headers alone: the reference's own CUDA machine (its lane kernels,
# CUB collectors and WMMA multiply) compiled for sm_100a, the reference-on-B200 baseline that bench.py times beside
# this project's kernels. Built from the reference tree where it lies into baseline/_ref/, which never enters the
# history.
REF_DEVICE_OUT = ROOT / "baseline" / "_ref" / "libemitted_ref.so"


def _flags(nvcc: str) -> list[str]:
    return [nvcc, "-std=c++20", "-O3", "--fmad=false", "-gencode", "arch=compute_100a,code=sm_100a",
            "--extended-lambda", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
            "-shared"]


def build_reference_device(runtime_dir: str) -> Path:
    REF_DEVICE_OUT.parent.mkdir(parents=True, exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = _flags(nvcc) + [f"-I{runtime_dir}", str(HERE / "emitted_program.cu"), "-o", str(REF_DEVICE_OUT)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"nvcc failed on the reference's device build:\n{done.stderr[-6000:]}")
    return REF_DEVICE_OUT


def build(runtime_dir: str) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = _flags(nvcc) + [f"-I{ROOT / 'include' / 'cairn_b200' / 'runtime'}", f"-I{runtime_dir}",
           str(HERE / "emitted_program.cu"), f"-L{ROOT / 'cairn_b200'}", "-lcairn_b200",
           "-Xlinker", "-rpath,$ORIGIN/../../../cairn_b200", "-o", str(OUT)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{done.stderr[-6000:]}")
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1]))
    print(build_reference_device(sys.argv[1]))
