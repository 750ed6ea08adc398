"""The native C++ programs (opengda_b200/bin/*) run under the local launcher."""
import os
import subprocess
import sys

import pytest

from opengda_b200.parallel.launch import free_port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "opengda_b200", "bin")

pytestmark = pytest.mark.gpu


def _launch(n, prog, *args):
    cmd = [sys.executable, "-m", "opengda_b200.parallel.launch", "-n", str(n), "--port", str(free_port()),
           "--timeout", "120", os.path.join(BIN, prog)] + [str(a) for a in args]
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=180,
                          env=dict(os.environ, GICC_TIMEOUT_MS="5000"))


def test_barrier_test_single_rank():
    p = _launch(1, "gicc_barrier_test", 1000)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "PASS" in p.stdout


@pytest.mark.multigpu
def test_barrier_test_all_gpus():
    import torch
    n = min(torch.cuda.device_count(), 8)
    p = _launch(n, "gicc_barrier_test", 10000)
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count("PASS") == n


@pytest.mark.multigpu
def test_pingpong_two_ranks():
    p = _launch(2, "gicc_pingpong", 200)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "PASS" in p.stdout


def test_gda_api_example_single_rank():
    p = _launch(1, "gda_api_example")
    assert p.returncode == 0, p.stdout + p.stderr
    assert "rank 0: PASS" in p.stdout


@pytest.mark.multigpu
def test_gda_api_example_all_gpus():
    import torch
    n = min(torch.cuda.device_count(), 8)
    p = _launch(n, "gda_api_example")
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count("PASS") == n


def test_gicc_api_example_single_rank():
    p = _launch(1, "gicc_api_example")
    assert p.returncode == 0, p.stdout + p.stderr
    assert "rank 0 of 1: PASS" in p.stdout


@pytest.mark.multigpu
def test_gicc_api_example_all_gpus():
    import torch
    n = min(torch.cuda.device_count(), 8)
    p = _launch(n, "gicc_api_example")
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count("PASS") == n


def test_gicc_jacobi_single_rank():
    p = _launch(1, "gicc_jacobi", "-nx", 1024, "-ny", 1024, "-niter", 50, "-nccheck", 10)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "PASS" in p.stdout


@pytest.mark.multigpu
def test_gicc_jacobi_all_gpus_matches_single_gpu():
    import torch
    n = min(torch.cuda.device_count(), 8)
    p = _launch(n, "gicc_jacobi", "-nx", 2048, "-ny", 2051, "-niter", 100, "-csv")
    assert p.returncode == 0, p.stdout + p.stderr
    assert ",PASS" in p.stdout


@pytest.mark.multigpu
def test_gicc_mm_all_gpus_analytic_check():
    import torch
    n = min(torch.cuda.device_count(), 8)
    p = _launch(n, "gicc_mm", "-n", 4096, "-iters", 5, "-samples", 128)
    assert p.returncode == 0, p.stdout + p.stderr
    assert "PASS" in p.stdout
