"""`bench.py --impl reference` (the CPU reference arm the driver times beside ours) prints one JSON line
with the same metric, unit and direction as our arm, `impl: reference`, a `cpu_baseline` describing the
run and an `e2e` object with no host<->device traffic. Runs on the CPU (one 2,208-token document through
the oracle, a few seconds)."""
import json
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_json_line():
    r = subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", "--steps", "1", "--warmup", "0"],
                       capture_output=True, text=True, timeout=600, cwd=str(ROOT))
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [ln for ln in r.stdout.splitlines() if ln.strip().startswith("{")]
    assert len(lines) == 1, r.stdout
    d = json.loads(lines[0])
    assert d["impl"] == "reference"
    assert d["metric"] == "bf16 docs/sec @2,208 tok (24-layer text backbone + pool)"
    assert d["unit"] == "docs/s" and d["higher_is_better"] is True
    assert d["value"] > 0 and d["steps"] == 1
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("port", "reference") and cb["cores"] >= 1 and cb["value"] == d["value"]
    e = d["e2e"]
    assert e["value"] == d["value"] and e["h2d_bytes_per_step"] == 0 and e["d2h_bytes_per_step"] == 0
