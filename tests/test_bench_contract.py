"""bench.py's JSON line, as the driver reads it: the reference arm on the CPU (the reference's host path, one bounded
step), and this project's arm on a B200 (config 2, three products after three warm-up ones)."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
BASE_KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
             "vs_baseline", "dtype", "data", "config", "e2e", "cpu_baseline"}


def _line(args: list[str], timeout: int) -> dict:
    done = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], cwd=ROOT, capture_output=True, text=True,
                          timeout=timeout)
    assert done.returncode == 0, done.stderr[-3000:]
    lines = [ln for ln in done.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, done.stdout[-3000:]
    return json.loads(lines[0])


def test_reference_arm_line():
    d = _line(["--impl", "reference", "--workload", "saxpy", "--steps", "1", "--warmup", "0"], timeout=600)
    assert BASE_KEYS <= d.keys() and d["impl"] == "reference"
    assert d["unit"] == "GB/s" and d["value"] > 0 and d["higher_is_better"] is True
    assert d["e2e"] == {"value": d["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    cpu = d["cpu_baseline"]
    assert cpu["value"] == d["value"] and cpu["cores"] >= 1 and cpu["kind"] in ("reference", "port")
    assert d["config"]["workload"].startswith("config 4")


@pytest.mark.gpu
def test_our_arm_line_on_config_2(cuda):
    d = _line(["--steps", "3", "--warmup", "3", "--no-cpu-baseline", "--no-reference-device", "--no-scaling-legs"],
              timeout=900)
    assert BASE_KEYS <= d.keys() and "impl" not in d
    assert (d["unit"], d["dtype"], d["scaling"], d["n_gpus"], d["steps"], d["warmup"]) == \
        ("TFLOP/s", "bf16", "weak", 1, 3, 3)
    assert 200 < d["value"] < 2500  # a B200's dense bf16 range
    r = d["roofline"]
    assert r["bound"] == "tensor" and r["unit"] == "TFLOP/s" and 0.1 < r["frac"] < 1.5
    assert abs(r["frac"] - r["achieved"] / r["peak"]) < 1e-9
    e = d["e2e"]
    assert e["unit"] == "TFLOP/s" and 0 < e["value"] < d["value"]
    assert e["h2d_bytes_per_step"] == 4096 * 4096 * 2 and e["d2h_bytes_per_step"] == 4096 * 4096 * 2
    assert d["gpu_launches"] == 3
    assert {"sm_mhz", "sm_max_mhz", "reasons"} <= d["clocks"].keys()
    assert 300 < d["clocks"]["sm_mhz_in_region"] < 2100
