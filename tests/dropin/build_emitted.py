"""Builds the drop-in test programs: CAIRN source compiled by the reference's own compiler, then the emitted C++ built
twice with the reference toolchain's exact device command.

For every program under tests/dropin/programs/ (CAIRN source):

1. `python -m cairn build PROGRAM --kind library --header --device-target sm_100a --cxx g++` runs the reference's
   compiler on it. That writes the emitted C++ (program.cpp), its C header and a library built over the reference's
   own runtime headers (its lane kernels, CUB collectors and WMMA multiply), with the command line the reference
   toolchain used (projects/toolchain.py device_prefix: C++20, -O3, --fmad=false, --extended-lambda,
   --expt-relaxed-constexpr, -Werror all-warnings -diag-suppress 177,550, and the host flags -Wall -Wextra -Werror
   ...). That library is the reference-on-B200 baseline, copied to baseline/_ref/lib<NAME>_ref.so.
2. The same program.cpp, unchanged, is compiled again by that same command with include/cairn_b200/runtime ahead
   of the reference's runtime directory on the include path, and linked against libcairn_b200.so, into
   tests/dropin/_build/lib<NAME>.so. Its regions, collectors and multiply then run on the B200 machine.

tests/dropin/scan_probe.cu, which exposes the B200 scan kernel alone (entries no CAIRN program emits), is built over
the drop-in headers with the same device flags into tests/dropin/_build/libscanprobe.so.

Kernel-benchmark submissions: each function of tests/dropin/harness/regions.cairn is exported with
`cairn export --harness kernelbench --mapping kb_<name>.toml` by the reference compiler run from a copy of the
reference's source tree whose runtime directory holds this project's drop-in region and collector headers
(cairn_gpu.hpp, cairn_kernels.hpp, cairn_cub.hpp), so the submission (a KernelBench ModelNew that embeds the runtime
headers it was exported with and builds them with torch's load_inline) runs the B200 machine. They land in
tests/dropin/_build/harness/<name>/.

The reference tree is named by the CAIRN_REFERENCE environment variable (the directory holding src/cairn), or by
the first command-line argument. Nothing here is needed on a GPU box: the built libraries travel with the tree.

    CAIRN_REFERENCE=<cairn checkout> python tests/dropin/build_emitted.py
"""

from __future__ import annotations

import concurrent.futures
import json
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
PROGRAMS = HERE / "programs"
BUILD = HERE / "_build"
DROPIN_HEADERS = ROOT / "include" / "cairn_b200" / "runtime"
REF_OUT = ROOT / "baseline" / "_ref"
ARCH = "sm_100a"


def reference_tree(arg: str | None = None) -> Path | None:
    """The CAIRN reference checkout (the directory holding src/cairn), or None when it is not present."""
    given = arg or os.environ.get("CAIRN_REFERENCE")
    if not given:
        return None
    tree = Path(given)
    return tree if (tree / "src" / "cairn" / "runtime").is_dir() else None


def programs() -> list[Path]:
    return sorted(PROGRAMS.glob("*.cairn"))


def _run(cmd: list[str], what: str, **kw) -> subprocess.CompletedProcess:
    done = subprocess.run(cmd, capture_output=True, text=True, **kw)
    if done.returncode != 0:
        raise RuntimeError(f"{what} failed ({done.returncode}):\n{' '.join(cmd)}\n{done.stdout[-4000:]}{done.stderr[-6000:]}")
    return done


def emit(tree: Path, program: Path, out: Path) -> dict:
    """The reference compiler's build of one program; returns its JSON record (command, directory, artifact, ...)."""
    env = dict(os.environ, PYTHONPATH=str(tree / "src"))
    cmd = [sys.executable, "-m", "cairn", "build", str(program), "--cxx", "g++", "--kind", "library", "--header",
           "--device-target", ARCH, "--out", str(out), "--format", "json"]
    done = _run(cmd, f"cairn build {program.name}", env=env, cwd=str(out), timeout=1800)
    record = json.loads(done.stdout)
    if record.get("status") != "native-built":
        raise RuntimeError(f"cairn build {program.name}: {record}")
    return record


def dropin_command(record: dict, source: Path, output: Path, runtime: Path) -> list[str]:
    """The reference toolchain's own command for `record`, on `source`, with the drop-in headers first."""
    cmd = list(record["command"])
    src = cmd.index(str(Path(record["directory"]) / "program.cpp"))
    out = cmd.index("-o")
    cmd[out + 1] = str(output)
    cmd[src] = str(source)
    cmd[src:src] = [f"-I{DROPIN_HEADERS}", f"-I{runtime}"]
    return cmd + [f"-L{ROOT / 'cairn_b200'}", "-lcairn_b200", "-Xlinker", "-rpath,$ORIGIN/../../../cairn_b200"]


def build_program(tree: Path, program: Path) -> tuple[Path, Path]:
    name = program.stem
    runtime = tree / "src" / "cairn" / "runtime"
    BUILD.mkdir(parents=True, exist_ok=True)
    REF_OUT.mkdir(parents=True, exist_ok=True)
    with tempfile.TemporaryDirectory(prefix=f"cairn-{name}-") as tmp:
        record = emit(tree, program, Path(tmp))
        built = Path(record["directory"])
        ref_lib = REF_OUT / f"lib{name}_ref.so"
        shutil.copy2(record["artifact"], ref_lib)
        # the emitted source alone, with no runtime header beside it (a quoted include would find those first)
        own = BUILD / name
        own.mkdir(exist_ok=True)
        shutil.copy2(built / "program.cpp", own / "program.cpp")
        shutil.copy2(record["header"], BUILD / f"{name}.h")
        (own / "reference_command.json").write_text(json.dumps(record["command"], indent=1))
        lib = BUILD / f"lib{name}.so"
        _run(dropin_command(record, own / "program.cpp", lib, runtime), f"drop-in build of {name}", timeout=1800)
    return lib, ref_lib


def build_probe(tree: Path) -> Path:
    """tests/dropin/scan_probe.cu over the drop-in headers, with the reference toolchain's device flags."""
    runtime = tree / "src" / "cairn" / "runtime"
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    out = BUILD / "libscanprobe.so"
    BUILD.mkdir(parents=True, exist_ok=True)
    cmd = [nvcc, "-std=c++20", "-O3", "--fmad=false", f"-arch={ARCH}", "--extended-lambda", "--expt-relaxed-constexpr",
           "-Werror", "all-warnings", "-diag-suppress", "177,550", "-x", "cu", "-shared", "-Xcompiler",
           "-ffp-contract=off,-fno-fast-math,-fno-finite-loops,-fexceptions,-fno-rtti,-Wall,-Wextra,-Werror,"
           "-Wno-unused-parameter,-Wno-unused-variable,-Wno-unused-but-set-variable,-fPIC,-Wno-unused-function",
           f"-I{DROPIN_HEADERS}", f"-I{runtime}", str(HERE / "scan_probe.cu"), "-o", str(out)]
    _run(cmd, "scan probe build", timeout=1800)
    return out


HARNESS = HERE / "harness"
HARNESS_OUT = BUILD / "harness"
DROPIN_RUNTIME = ("cairn_gpu.hpp", "cairn_kernels.hpp", "cairn_cub.hpp")


def build_harnesses(tree: Path) -> list[Path]:
    """Every function of harness/regions.cairn exported as a KernelBench submission over the drop-in headers."""
    done: list[Path] = []
    with tempfile.TemporaryDirectory(prefix="cairn-overlay-") as tmp:
        overlay = Path(tmp) / "src" / "cairn"
        shutil.copytree(tree / "src" / "cairn", overlay, ignore=shutil.ignore_patterns("__pycache__"))
        for name in DROPIN_RUNTIME:
            shutil.copy2(DROPIN_HEADERS / name, overlay / "runtime" / name)
        env = dict(os.environ, PYTHONPATH=str(Path(tmp) / "src"))
        for mapping in sorted(HARNESS.glob("kb_*.toml")):
            symbol = mapping.stem[3:]
            out = HARNESS_OUT / symbol
            if out.exists():
                shutil.rmtree(out)
            out.parent.mkdir(parents=True, exist_ok=True)
            cmd = [sys.executable, "-m", "cairn", "export", str(HARNESS / "regions.cairn"), "--harness", "kernelbench",
                   "--symbol", symbol, "--mapping", str(mapping), "--device-target", ARCH, "--cxx", "g++", "--out",
                   str(out), "--format", "json"]
            record = json.loads(_run(cmd, f"cairn export --harness of {symbol}", env=env, cwd=tmp, timeout=900).stdout)
            if record.get("status") != "exported-harness":
                raise RuntimeError(f"cairn export {symbol}: {record}")
            done.append(out / record["file"])
    return done


def build(arg: str | None = None) -> list[Path]:
    """Builds every program both ways and the probe; returns the libraries written. Needs the reference tree."""
    tree = reference_tree(arg)
    if tree is None:
        raise RuntimeError("the CAIRN reference tree is not available (set CAIRN_REFERENCE)")
    done: list[Path] = []
    with concurrent.futures.ThreadPoolExecutor(4) as pool:
        jobs = [pool.submit(build_program, tree, p) for p in programs()] + [pool.submit(build_probe, tree),
                                                                             pool.submit(build_harnesses, tree)]
        for job in jobs:
            r = job.result()
            done.extend(r if isinstance(r, (tuple, list)) else [r])
    return done


if __name__ == "__main__":
    for path in build(sys.argv[1] if len(sys.argv) > 1 else None):
        print(path)
