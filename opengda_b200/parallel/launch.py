"""Local multi-rank launcher: ``python -m opengda_b200.parallel.launch -n N prog args...``.

Forks N ranks on this host with GICC_RANK / GICC_SIZE / GICC_LOCAL_RANK / GICC_LOCAL_SIZE
and GICC_BOOTSTRAP_ADDR set (the reference relies on ``srun``/``mpirun``,
scripts/LC/run.sh:45-50).  If one rank exits non-zero the launcher terminates the rest
(their process groups; SIGKILL after `grace` seconds if one ignores SIGTERM) and returns
that rank's exit code.  With `timeout`, every rank still running after that many seconds is
killed and the launcher returns 124.
"""
from __future__ import annotations

import argparse
import os
import signal
import socket
import subprocess
import sys
import time
from typing import List, Optional


def free_port(host: str = "127.0.0.1") -> int:
    s = socket.socket()
    s.bind((host, 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _kill_groups(procs, ranks, sig) -> None:
    for q in ranks:
        try:
            os.killpg(procs[q].pid, sig)
        except ProcessLookupError:
            pass


def launch(n: int, cmd: List[str], host: str = "127.0.0.1", port: Optional[int] = None,
           timeout: Optional[float] = None, extra_env: Optional[dict] = None, grace: float = 10.0) -> int:
    port = port or free_port(host)
    procs = []
    for r in range(n):
        env = dict(os.environ)
        env.update(extra_env or {})
        env.update({
            "GICC_RANK": str(r), "GICC_SIZE": str(n), "GICC_LOCAL_RANK": str(r), "GICC_LOCAL_SIZE": str(n),
            "GICC_BOOTSTRAP_ADDR": f"{host}:{port}",
            "RANK": str(r), "WORLD_SIZE": str(n), "LOCAL_RANK": str(r), "LOCAL_WORLD_SIZE": str(n),
        })
        procs.append(subprocess.Popen(cmd, env=env, start_new_session=True))
    t0 = time.time()
    rc = 0
    term_at = None  # when the surviving ranks were sent SIGTERM
    alive = set(range(n))
    try:
        while alive:
            for r in list(alive):
                c = procs[r].poll()
                if c is None:
                    continue
                alive.discard(r)
                if c != 0 and rc == 0:
                    rc = c
                    _kill_groups(procs, alive, signal.SIGTERM)
                    term_at = time.time()
            if alive and term_at is not None and time.time() - term_at > grace:
                _kill_groups(procs, alive, signal.SIGKILL)
                term_at = float("inf")  # sent once
            if timeout is not None and time.time() - t0 > timeout:
                _kill_groups(procs, alive, signal.SIGKILL)
                for q in alive:
                    procs[q].wait()
                return 124
            time.sleep(0.02)
    except KeyboardInterrupt:
        _kill_groups(procs, range(n), signal.SIGTERM)
        raise
    return rc


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("-n", "--nranks", type=int, required=True)
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=None)
    ap.add_argument("--timeout", type=float, default=None)
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    a = ap.parse_args(argv)
    if not a.cmd:
        ap.error("missing command")
    return launch(a.nranks, a.cmd, a.host, a.port, a.timeout)


if __name__ == "__main__":
    sys.exit(main())
