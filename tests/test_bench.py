"""``bench.py`` on the CPU: the reference arm (the NumPy path of the same configuration, which
needs no GPU) prints one JSON line with the contract's keys, for the default workload and a
GEMM, and the CPU baseline covers every configuration."""

from __future__ import annotations

import json
import subprocess
import sys

import pytest
from conftest import ROOT

KEYS = {"metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
        "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config", "impl",
        "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload", [None, "c5b_matmul_splitk"])
def test_reference_arm_prints_one_contract_line(workload: str | None) -> None:
    cmd = [sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1",
           "--warmup", "1", "--cpu-seconds", "0.5"]
    if workload:
        cmd += ["--workload", workload]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert KEYS <= set(line), KEYS - set(line)
    assert line["impl"] == "reference" and line["n_gpus"] == 1 and line["value"] > 0
    import bench

    assert line["config"] == bench.config_of(workload or "c2_gelu_chain", 1, "strong")
    assert line["unit"] == ("TFLOP/s" if workload else "GB/s")
    assert line["e2e"]["h2d_bytes_per_step"] == line["e2e"]["d2h_bytes_per_step"] == 0
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["value"] == line["value"]


def test_cpu_baseline_covers_every_configuration() -> None:
    import bench  # the repository root is on sys.path (conftest)

    from ptxgen import problems, shard

    for name in problems.CONFIGS:
        plan = shard.local_problem(name, 1)
        r = bench.cpu_baseline(name, plan, 0.05, 2)
        assert r["value"] > 0 and r["cores"] >= 1 and r["sample"], name
