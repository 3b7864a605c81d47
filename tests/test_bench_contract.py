"""bench.py's reference arm on the CPU: one JSON line with the fields the benchmark contract asks for (the
reference's CPU path of the Lloyd pass, timed on this host's cores, on the same metric and configuration as the
GPU arm).  CPU tier: the NumPy restatement runs on a bounded row sample, one warm-up and one timed step."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "1",
                          "--warmup", "1"], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1
    j = json.loads(lines[0])
    base = json.load(open(os.path.join(ROOT, "BASELINE.json")))
    assert j["impl"] == "reference" and j["metric"] == base["metric"]
    assert j["unit"] == "rows/s" and j["higher_is_better"] is True and j["value"] > 0
    assert j["n_gpus"] == 1 and j["steps"] == 1 and j["warmup"] == 1
    assert j["e2e"]["value"] == j["value"] and j["e2e"]["unit"] == j["unit"]
    assert j["e2e"]["h2d_bytes_per_step"] == 0 and j["e2e"]["d2h_bytes_per_step"] == 0
    cb = j["cpu_baseline"]
    assert cb["value"] == j["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["sample"]
    assert "config3" in j["config"]["workload"]
