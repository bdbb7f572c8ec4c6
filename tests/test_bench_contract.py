"""The JSON line of ``bench.py --impl reference`` (the reference's torch path on the
host cores), checked on the CPU: one step, keys and units as the benchmark
driver reads them, and the same metric, unit and workload as the GPU arm."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def test_reference_arm_prints_one_contract_line():
    proc = subprocess.run(
        [sys.executable, "bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"],
        cwd=ROOT, capture_output=True, text=True, timeout=600, check=True,
    )
    lines = [line for line in proc.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    assert line["impl"] == "reference"
    assert line["metric"] == "NS matrices/s" and line["unit"] == "matrices/s"
    assert line["higher_is_better"] is True and line["n_gpus"] == 1
    assert line["steps"] == 1 and line["warmup"] == 1
    assert line["value"] > 0 and line["ms_per_step"] > 0
    assert line["config"]["batch_per_gpu"] == 64
    assert (line["config"]["rows"], line["config"]["cols"]) == (1024, 4096)
    cpu = line["cpu_baseline"]
    assert cpu["value"] == line["value"] and cpu["unit"] == line["unit"]
    assert cpu["kind"] in ("port", "reference") and cpu["cores"] >= 1 and cpu["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
