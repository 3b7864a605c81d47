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


def test_clock_sampler_waits_for_its_first_sample(tmp_path, monkeypatch):
    """The clock record of a short timed region: sampling starts before the region (nvidia-smi may take a
    while to start) and takes one more sample after it.  A stand-in nvidia-smi prints the query's CSV rows."""
    import importlib.util
    import time
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/bash\nsleep 0.3\nwhile true; do\n"
                    "  echo '0, 1965, 1965, 700.0, 0x0, Not Active, Not Active, Not Active, Active'\n"
                    "  sleep 0.05\ndone\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ.get('PATH', '')}")
    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    c = bench.Clocks("0")
    c.start()
    time.sleep(0.01)                                    # a timed region shorter than the sampling interval
    rec = c.stop()
    assert rec["samples"] >= 2 and rec["sm_mhz"] == 1965.0 and rec["sm_max_mhz"] == 1965.0
    assert rec["reasons"] == ["sw_power_cap"]
