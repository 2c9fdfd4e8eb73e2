"""bench.py's output contract, checked through its reference arm (the CPU
implementation of the path timed on host cores, so it runs without a GPU):
one JSON line with the metric, unit and direction the GPU arm reports, the
base keys, a cpu_baseline describing the run and an e2e object with no
host-device traffic.  The GPU arm prints the same keys plus roofline, clocks
and gpu_launches; it is exercised on the B200."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_reference_arm_prints_one_contract_line():
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--steps", "2",
                          "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    rec = json.loads(lines[0])
    sys.path.insert(0, ROOT)
    import bench

    assert rec["impl"] == "reference"
    assert rec["metric"] == bench.METRIC and rec["unit"] == bench.UNIT and rec["unit"] == "GB/s"
    assert rec["higher_is_better"] is True and rec["scaling"] == "weak"
    assert rec["n_gpus"] == 1 and rec["steps"] == 2 and rec["warmup"] == 1
    assert rec["value"] > 0 and rec["ms_per_step"] > 0
    assert rec["data"] == "synthetic" and rec["vs_baseline"] is None
    assert rec["config"]["workload"].startswith("configs[0]")
    cb = rec["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == rec["value"]
    assert cb["unit"] == rec["unit"] and cb["sample"]
    e2e = rec["e2e"]
    assert e2e["value"] == rec["value"] and e2e["unit"] == rec["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
