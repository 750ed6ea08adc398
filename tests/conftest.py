import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")
    config.addinivalue_line("markers", "multigpu: needs 2 or more GPUs")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        have_gpu = torch.cuda.is_available()
        ngpu = torch.cuda.device_count() if have_gpu else 0
    except Exception:  # pragma: no cover
        have_gpu, ngpu = False, 0
    for item in items:
        if "gpu" in item.keywords and not have_gpu:
            item.add_marker(pytest.mark.skip(reason="no CUDA device"))
        if "multigpu" in item.keywords and ngpu < 2:
            item.add_marker(pytest.mark.skip(reason="needs >= 2 GPUs"))


def run_native(n, prog, *args, timeout=180, env=None):
    """Run opengda_b200/bin/<prog> on n ranks under the local launcher; returns the
    CompletedProcess (stdout/stderr captured)."""
    import subprocess

    from opengda_b200.parallel.launch import free_port
    cmd = [sys.executable, "-m", "opengda_b200.parallel.launch", "-n", str(n), "--port", str(free_port()),
           "--timeout", str(max(30, timeout - 60)), os.path.join(ROOT, "opengda_b200", "bin", prog)]
    cmd += [str(a) for a in args]
    return subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True, timeout=timeout,
                          env=dict(os.environ, GICC_TIMEOUT_MS="5000", **(env or {})))


@pytest.fixture
def native_app():
    return run_native
