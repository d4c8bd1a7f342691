"""bench.py's reference arm on the CPU: one JSON line in the benchmark contract.

The arm times the CPU restatement of the reference's Q8 engine on the host
cores (no GPU involved), for both workloads, on the tiny model so the test
takes seconds.
"""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("extra", [["--requests", "40"], ["--workload", "longtext", "--docs", "2"]])
def test_reference_arm_prints_one_contract_line(extra):
    cmd = [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--model", "tiny_self",
           "--steps", "1", "--warmup", "1", "--cpu-seconds", "1"] + extra
    out = subprocess.run(cmd, capture_output=True, text=True, timeout=300, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["unit"] == "tokens/s" and d["higher_is_better"] is True
    assert d["metric"] == "target tokens/sec per box (greedy)" and d["value"] > 0
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]
    assert d["e2e"] == {"value": d["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    want = "long-text stream" if "longtext" in extra else "continuous-batching stream"
    assert d["config"]["workload"].startswith(want)
