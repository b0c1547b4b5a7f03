"""The benchmark's reference arm (`bench.py --impl reference`) runs on host
cores only: this checks, without a GPU, that it prints the one JSON line the
benchmark contract asks for (the metric of BASELINE.json, a positive
per-layer time, the CPU baseline it describes, an end-to-end entry with no
host-device copies)."""
from __future__ import annotations

import json
import os
import subprocess
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, os.path.join(REPO, "bench.py"), "--impl", "reference",
                        "--steps", "1", "--warmup", "3"], cwd=REPO, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads(r.stdout.strip().splitlines()[-1])
    with open(os.path.join(REPO, "BASELINE.json")) as f:
        metric = json.load(f)["metric"]
    assert line["impl"] == "reference"
    assert line["metric"] == metric
    assert line["value"] > 0 and line["unit"] == "us/layer"
    assert line["higher_is_better"] is False
    assert (line["n_gpus"], line["steps"], line["warmup"]) == (1, 1, 3)
    assert abs(line["ms_per_step"] * 1000 - line["value"]) < 1e-3 * line["value"]
    cb = line["cpu_baseline"]
    assert cb["value"] == line["value"] and cb["kind"] in ("port", "reference")
    assert cb["cores"] >= 1 and cb["sample"]
    e2e = line["e2e"]
    assert e2e["value"] == line["value"] and e2e["unit"] == line["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert line["config"]["workload"]
