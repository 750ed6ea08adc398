"""The repeat-N stress driver (bench/stress.py) on CPU programs."""
import json
import os
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _stress(*args):
    p = subprocess.run([sys.executable, os.path.join(ROOT, "bench", "stress.py"), *args], cwd=ROOT,
                       capture_output=True, text=True, timeout=300)
    return p.returncode, json.loads(p.stdout.strip().splitlines()[-1])


def test_stress_counts_passes_and_summarises_a_json_key():
    rc, out = _stress("-n", "2", "--repeat", "2", "--json-key", "v", "--", sys.executable, "-c",
                      "import json; print('PASS'); print(json.dumps({'v': 3.5}))")
    assert rc == 0 and out["passed"] == 2 and out["v"]["mean"] == 3.5


def test_stress_reports_failures():
    rc, out = _stress("-n", "1", "--repeat", "2", "--", sys.executable, "-c", "print('FAIL'); raise SystemExit(3)")
    assert rc == 1 and out["passed"] == 0 and len(out["failed"]) == 2 and out["failed"][0]["rc"] != 0
