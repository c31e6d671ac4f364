"""Builds tests/dropin/emitted_program.cu into tests/dropin/_build/libemitted.so: the CAIRN runtime headers from the
reference tree given on the command line, with include/cairn_b200/runtime ahead of them, so the program's runtime
calls land on the B200 machine and libcairn_b200.so. The flags are the reference toolchain's device flags
(projects/toolchain.py:184-200: C++20, -O3, --fmad=false, --extended-lambda, --expt-relaxed-constexpr), for sm_100a.

    python tests/dropin/build_emitted.py <cairn source tree>/src/cairn/runtime
"""

from __future__ import annotations

import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
OUT = HERE / "_build" / "libemitted.so"


def build(runtime_dir: str) -> Path:
    OUT.parent.mkdir(exist_ok=True)
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    cmd = [nvcc, "-std=c++20", "-O3", "--fmad=false", "-gencode", "arch=compute_100a,code=sm_100a",
           "--extended-lambda", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-ffp-contract=off,-fno-fast-math",
           "-shared", f"-I{ROOT / 'include' / 'cairn_b200' / 'runtime'}", f"-I{runtime_dir}",
           str(HERE / "emitted_program.cu"), f"-L{ROOT / 'cairn_b200'}", "-lcairn_b200",
           "-Xlinker", "-rpath,$ORIGIN/../../../cairn_b200", "-o", str(OUT)]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"nvcc failed:\n{done.stderr[-6000:]}")
    return OUT


if __name__ == "__main__":
    print(build(sys.argv[1]))
