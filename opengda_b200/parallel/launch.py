"""Local multi-rank launcher: ``python -m opengda_b200.parallel.launch -n N prog args...``.

Forks N ranks on this host with GICC_RANK / GICC_SIZE / GICC_LOCAL_RANK / GICC_LOCAL_SIZE
and GICC_BOOTSTRAP_ADDR set (the reference relies on ``srun``/``mpirun``,
scripts/LC/run.sh:45-50).  If one rank exits non-zero the launcher terminates the rest
(their process groups) and returns that rank's exit code.
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


def launch(n: int, cmd: List[str], host: str = "127.0.0.1", port: Optional[int] = None,
           timeout: Optional[float] = None, extra_env: Optional[dict] = None) -> int:
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
                    for q in alive:
                        try:
                            os.killpg(procs[q].pid, signal.SIGTERM)
                        except ProcessLookupError:
                            pass
            if timeout is not None and time.time() - t0 > timeout:
                for q in alive:
                    try:
                        os.killpg(procs[q].pid, signal.SIGKILL)
                    except ProcessLookupError:
                        pass
                return 124
            time.sleep(0.02)
    except KeyboardInterrupt:
        for p in procs:
            try:
                os.killpg(p.pid, signal.SIGTERM)
            except ProcessLookupError:
                pass
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
