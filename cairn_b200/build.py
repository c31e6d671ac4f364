"""Builds libcairn_b200.so in-tree from cairn_b200/csrc for sm_100a with nvcc.

Each translation unit compiles to an object under cairn_b200/_build (in parallel), then nvcc links the shared
library next to this file, with the CUDA runtime linked statically so the library carries no dependency on the
toolkit's libcudart. `python -m cairn_b200.build [--verbose]` rebuilds it; `--ptxas` prints ptxas' resource usage
(registers, spills, shared memory) for every kernel.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
BUILD = HERE / "_build"
LIB = HERE / "libcairn_b200.so"
INCLUDE = HERE.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-std=c++17",
    "-O3",
    "-lineinfo",
    "-DNDEBUG",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC,-O3,-Wall,-Wno-unused-function",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build libcairn_b200.so")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    built = target.stat().st_mtime
    return any(d.stat().st_mtime > built for d in deps)


def _compile(src: Path, ptxas: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas:
        cmd += ["-Xptxas", "-v"]
    done = subprocess.run(cmd, capture_output=True, text=True)
    if done.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{done.stderr[-6000:]}")
    return obj, done.stderr


def build(force: bool = False, verbose: bool = False, ptxas: bool = False) -> Path:
    """Compiles every stale translation unit and relinks the library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "cairn_b200.h"]
    srcs = sources()
    todo = [s for s in srcs if force or ptxas or _stale(BUILD / (s.stem + ".o"), [s, *headers])]
    if todo:
        workers = min(len(todo), os.cpu_count() or 1)
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            for obj, log in pool.map(lambda s: _compile(s, ptxas), todo):
                if verbose or ptxas:
                    print(f"[cairn_b200] built {obj.name}", file=sys.stderr)
                    if log.strip():
                        print(log, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or todo or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        done = subprocess.run(cmd, capture_output=True, text=True)
        if done.returncode != 0:
            raise RuntimeError(f"link failed:\n{done.stderr[-4000:]}")
    return LIB


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    parser.add_argument("--ptxas", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas=args.ptxas))


if __name__ == "__main__":
    main()
