"""CPU multi-process tests of the socket bootstrap: collectives, fd passing and failure
detection (a rank that leaves, aborts or never arrives).  No GPU involved."""
import os
import sys

import pytest

from opengda_b200.parallel.launch import launch

WORKER = os.path.join(os.path.dirname(__file__), "workers", "boot_worker.py")


def _run(n, mode, tmp_path, env=None, timeout=60):
    out = str(tmp_path / mode)
    rc = launch(n, [sys.executable, WORKER, mode, out], timeout=timeout, extra_env=env)
    res = {}
    for r in range(n):
        p = f"{out}.{r}"
        res[r] = open(p).read() if os.path.exists(p) else None
    return rc, res


@pytest.mark.parametrize("n", [1, 2, 4])
def test_collectives(n, tmp_path):
    rc, res = _run(n, "collectives", tmp_path)
    assert rc == 0, res
    assert all(v == "ok" for v in res.values()), res


@pytest.mark.parametrize("n", [2, 3])
def test_fd_passing(n, tmp_path):
    rc, res = _run(n, "fds", tmp_path)
    assert rc == 0, res
    assert all(v == "ok" for v in res.values()), res


@pytest.mark.parametrize("how", ["die", "kill"])
def test_rank_that_leaves_is_detected(how, tmp_path):
    rc, res = _run(3, how, tmp_path, env={"GICC_BOOTSTRAP_TIMEOUT_MS": "20000"})
    for r in (0, 2):
        assert res[r] is not None and res[r].startswith("err:") and "left the job" in res[r], res
        assert float(res[r].rsplit(":", 1)[1]) < 5.0, res  # well before the timeout


def test_abort_fails_the_job(tmp_path):
    rc, res = _run(3, "abort", tmp_path, env={"GICC_BOOTSTRAP_TIMEOUT_MS": "20000"})
    assert rc == 3  # the aborting rank's code
    for r in (0, 2):
        assert res[r] is not None and "aborted the job" in res[r] and "injected failure" in res[r], res


def test_barrier_timeout(tmp_path):
    rc, res = _run(2, "timeout", tmp_path, env={"GICC_BOOTSTRAP_TIMEOUT_MS": "1000"})
    assert res[0] is not None and res[0].startswith("err:") and "timed out" in res[0], res
    assert float(res[0].rsplit(":", 1)[1]) < 3.0, res


def test_native_host_collectives_cpu():
    """gicc::coll::allreduce_sum/min/max, allgather, broadcast and sendrecv from C++
    (opengda_b200/bin/gicc_coll_test), 3 CPU ranks through the local launcher."""
    import subprocess
    from opengda_b200.parallel.launch import free_port
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    p = subprocess.run([sys.executable, "-m", "opengda_b200.parallel.launch", "-n", "3", "--port", str(free_port()),
                        "--timeout", "60", os.path.join(root, "opengda_b200", "bin", "gicc_coll_test")],
                       cwd=root, capture_output=True, text=True, timeout=120)
    assert p.returncode == 0, p.stdout + p.stderr
    assert p.stdout.count("PASS") == 3


@pytest.mark.parametrize("mode,needle", [("exchange_count", "registered"), ("exchange_kind", "different kind")])
def test_exchange_table_mismatch_fails_on_every_rank(mode, needle, tmp_path):
    rc, res = _run(3, mode, tmp_path)
    for r in range(3):
        assert res[r] is not None and res[r].startswith("err:BootstrapError") and needle in res[r], res


def test_exchange_tables_that_match_pass(tmp_path):
    rc, res = _run(3, "exchange_ok", tmp_path)
    assert rc == 0, res
    assert all(v == "ok" for v in res.values()), res
