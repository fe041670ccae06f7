"""bench.py --impl reference on the host: one JSON line with the contract's keys.

The reference arm times the oracle's CPU restatement of the reference path on the host cores,
so it runs without a GPU; this checks the line it prints (impl, metric and unit of our arm, a
cpu_baseline describing the run, an e2e object with no host-device copies).
"""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_the_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference",
                          "--steps", "1", "--warmup", "1"], cwd=ROOT, capture_output=True, text=True,
                         timeout=600, check=True)
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["metric"] == "OABF dequant-GEMV HBM GB/s and decode tokens/s at 1/2/4/8 B200"
    assert line["unit"] == "GB/s" and line["higher_is_better"] is True
    assert line["value"] > 0 and line["steps"] == 1 and line["warmup"] == 1
    cb = line["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert cb["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert "workload" in line["config"]
