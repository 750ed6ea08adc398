"""The local multi-rank launcher: rank environment, failure propagation (the other ranks
are terminated, then killed after the grace period) and the overall timeout."""
import sys
import time

from opengda_b200.parallel.launch import launch

PY = sys.executable


def test_ranks_get_their_environment(tmp_path):
    out = tmp_path / "env"
    code = ("import os; r = os.environ['GICC_RANK']; "
            f"open(r'{out}.' + r, 'w').write(' '.join(os.environ[k] for k in "
            "('GICC_RANK', 'GICC_SIZE', 'GICC_LOCAL_RANK', 'RANK', 'WORLD_SIZE', 'GICC_BOOTSTRAP_ADDR')))")
    assert launch(3, [PY, "-c", code], timeout=60) == 0
    vals = [open(f"{out}.{r}").read().split() for r in range(3)]
    assert [v[:5] for v in vals] == [[str(r), "3", str(r), str(r), "3"] for r in range(3)]
    assert len({v[5] for v in vals}) == 1 and vals[0][5].startswith("127.0.0.1:")


def test_failing_rank_ends_the_job_with_its_code():
    code = "import os, time; r = int(os.environ['GICC_RANK']); time.sleep(0.5) if r == 1 else None; " \
           "raise SystemExit(7) if r == 1 else time.sleep(60)"
    t0 = time.time()
    assert launch(3, [PY, "-c", code], timeout=120) == 7
    assert time.time() - t0 < 30


def test_rank_ignoring_sigterm_is_killed_after_grace():
    code = ("import os, signal, time; r = int(os.environ['GICC_RANK']); "
            "signal.signal(signal.SIGTERM, signal.SIG_IGN); "
            "raise SystemExit(5) if r == 0 else time.sleep(60)")
    t0 = time.time()
    assert launch(2, [PY, "-c", code], timeout=120, grace=1.0) == 5
    assert time.time() - t0 < 30


def test_timeout_returns_124():
    t0 = time.time()
    assert launch(2, [PY, "-c", "import time; time.sleep(60)"], timeout=2) == 124
    assert time.time() - t0 < 30
