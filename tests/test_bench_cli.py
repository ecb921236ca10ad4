"""The benchmark's command-line contract on the host (no GPU): the reference arm prints exactly one
JSON line with the keys the round-end driver reads, and the vendor arm declines the workloads it
does not cover with an `unavailable` line and exit status 0."""
import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def run_bench(*args):
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), *args], capture_output=True, text=True,
                       cwd=ROOT, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip()]
    assert len(lines) == 1, r.stdout  # the JSON line is the only thing on stdout
    return json.loads(lines[0])


def test_reference_arm_line():
    line = run_bench("--impl", "reference", "--config", "c1", "--steps", "1", "--warmup", "1")
    assert line["impl"] == "reference"
    assert line["unit"] == "residues/s" and line["value"] > 0 and line["higher_is_better"] is True
    assert line["steps"] == 1 and line["warmup"] == 1 and line["n_gpus"] == 1
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "residues/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}


def test_vendor_arm_declines_the_scan():
    line = run_bench("--impl", "vendor", "--config", "c3")
    assert line["impl"] == "vendor" and "unavailable" in line
