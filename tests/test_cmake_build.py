"""The CMake build of the native runtime (CMakeLists.txt at the repository root): it
configures with the default options, lists the library and every example program as
targets, and rejects any architecture other than sm_100a."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.skipif(shutil.which("cmake") is None or not os.path.exists("/usr/local/cuda/bin/nvcc"),
                                reason="cmake or nvcc not available")


def _configure(build_dir, *extra):
    env = dict(os.environ, CUDACXX="/usr/local/cuda/bin/nvcc")
    return subprocess.run(["cmake", "-S", ROOT, "-B", str(build_dir), *extra], capture_output=True, text=True,
                          timeout=300, env=env)


def test_configure_defaults_lists_library_and_apps(tmp_path):
    res = _configure(tmp_path / "b")
    assert res.returncode == 0, res.stdout[-2000:] + res.stderr[-2000:]
    assert "arch sm_100a" in res.stdout
    targets = subprocess.run(["cmake", "--build", str(tmp_path / "b"), "--target", "help"], capture_output=True,
                             text=True, timeout=120).stdout
    apps = [f[:-3] for f in os.listdir(os.path.join(ROOT, "csrc", "apps")) if f.endswith(".cu")]
    for t in ["gicc"] + apps:
        assert t in targets, (t, targets[-2000:])


def test_configure_rejects_other_architectures(tmp_path):
    res = _configure(tmp_path / "b", "-DGICC_ARCH=90a")
    assert res.returncode != 0
    assert "only" in (res.stdout + res.stderr) or "not supported" in (res.stdout + res.stderr)
