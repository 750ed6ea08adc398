"""Every benchmark script imports and parses its command line on a machine without a GPU
(`--help`), so a script that only runs on the GPU box cannot rot unnoticed."""
import glob
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SCRIPTS = sorted(glob.glob(os.path.join(ROOT, "bench", "*.py"))) + [os.path.join(ROOT, "bench.py")]
NO_ARGPARSE = {"profile_kernels.py"}  # positional case names, no --help


@pytest.mark.parametrize("script", [s for s in SCRIPTS if os.path.basename(s) not in NO_ARGPARSE],
                         ids=os.path.basename)
def test_help(script):
    p = subprocess.run([sys.executable, script, "--help"], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert p.returncode == 0, p.stderr[-2000:]
    assert "usage" in p.stdout.lower()


def test_profile_kernels_imports():
    p = subprocess.run([sys.executable, "-c", "import ast,sys; ast.parse(open(sys.argv[1]).read())",
                        os.path.join(ROOT, "bench", "profile_kernels.py")], capture_output=True, text=True, timeout=60)
    assert p.returncode == 0, p.stderr
