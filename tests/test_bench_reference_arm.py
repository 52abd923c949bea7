"""bench.py's reference arm on the host: the JSON line keeps the benchmark
contract, and the process never loads libautdot (the arm times the
reference's own CPU code, or the oracle's restatement of it when the
reference's host library was not built)."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_RUNNER = r"""
import runpy, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "3", "--warmup", "3"]
try:
    runpy.run_path("bench.py", run_name="__main__")
except SystemExit as e:
    if e.code not in (None, 0):
        raise
with open("/proc/self/maps") as f:
    maps = f.read()
print("LOADED_LIBAUTDOT=%d" % ("libautdot" in maps))
"""


def test_reference_arm_line_and_no_product_library():
    r = subprocess.run([sys.executable, "-c", _RUNNER], cwd=ROOT, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [l for l in r.stdout.splitlines() if l.strip()]
    assert lines[-1] == "LOADED_LIBAUTDOT=0", lines[-1]
    d = json.loads(next(l for l in reversed(lines) if l.startswith("{")))
    assert d["impl"] == "reference"
    if "unavailable" in d:
        return
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in d, key
    assert d["steps"] == 3 and d["warmup"] == 3 and d["n_gpus"] == 1
    assert d["value"] > 0 and d["unit"] == "GB/s" and d["higher_is_better"] is True
    cb = d["cpu_baseline"]
    assert cb["kind"] in ("reference", "port") and cb["cores"] >= 1 and cb["value"] == d["value"]
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0
    assert "workload" in d["config"]
