"""The benchmark's reference arm on the host (no GPU): `bench.py --impl
reference` runs the reference's own CPU code for the config-2 block (the
product-flag build of ops.c under oracle/_ref when the build could compile
it, else the C restatement) and prints the same JSON line as the GPU arm,
with `impl` set, its CPU baseline described and no host<->device bytes."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_bench(*args):
    env = dict(os.environ)
    env.pop("WORLD_SIZE", None)
    env.pop("RANK", None)
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), *args], cwd=ROOT,
                         env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    return json.loads(lines[0])


def test_reference_arm_prints_the_contract_line():
    line = _run_bench("--impl", "reference", "--headline-only", "--steps", "2", "--warmup", "3")
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config",
                "impl", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference"
    assert line["unit"] == "TOPS" and line["higher_is_better"] is True
    assert line["n_gpus"] == 1 and line["steps"] == 2 and line["warmup"] == 3
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["config"]["M"] == 2048 and line["config"]["D"] == 1024
    assert line["config"]["H"] == 2816
    cpu = line["cpu_baseline"]
    assert cpu["kind"] in ("reference", "port") and cpu["cores"] >= 1
    assert cpu["value"] == line["value"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bench_rejects_short_warmup():
    """The timing rules ask for at least three warm-up steps."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--warmup", "2"], cwd=ROOT, capture_output=True, text=True,
                         timeout=120)
    assert out.returncode != 0
    assert "warmup" in (out.stderr + out.stdout)
