"""bench.py's reference arm on the CPU: it times the reference's own C++
fused attention and engine (built from the reference's sources into
oracle/_ref) without importing this package, and prints one JSON line with
the contract's keys and the same `config` object as the GPU arm."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SCRIPT = r'''
import json, sys
sys.argv = ["bench.py", "--impl", "reference", "--steps", "1", "--warmup", "1"]
import bench
bench.main()
loaded = sorted(m for m in sys.modules if m.startswith("tritiercache_b200"))
print("LOADED " + json.dumps(loaded))
'''


def test_reference_arm_runs_without_the_package():
    ref = os.path.join(ROOT, "oracle", "_ref")
    if not (os.path.isdir(ref) and any(f.startswith("_C") and f.endswith(".so") for f in os.listdir(ref))):
        pytest.skip("the reference build (oracle/_ref) is not here")
    out = subprocess.run([sys.executable, "-c", SCRIPT], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["higher_is_better"] is False and d["value"] > 0
    for k in ("metric", "unit", "n_gpus", "steps", "warmup", "config", "cpu_baseline", "e2e"):
        assert k in d, k
    assert d["e2e"]["h2d_bytes_per_step"] == 0 and d["e2e"]["d2h_bytes_per_step"] == 0
    assert d["cpu_baseline"]["kind"] == "reference" and d["cpu_baseline"]["cores"] >= 1
    assert d["config"]["workload"].startswith("config2")
    loaded = json.loads([l for l in out.stdout.splitlines() if l.startswith("LOADED ")][0][7:])
    assert loaded == [], loaded
