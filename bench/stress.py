"""Repeat a multi-rank program N times and summarise pass/fail and run-to-run jitter (the
reference's legacy/ofi/prototype/test_barrier.sh and stress_test.sh: repeat-N loops over
srun that grep "PASS" and summarise JSON results).

    python bench/stress.py -n 2 --repeat 20 -- opengda_b200/bin/gicc_barrier_test 10000
    python bench/stress.py -n 8 --repeat 5 --json-key barrier_us -- python tests/workers/...

Each run goes through opengda_b200.parallel.launch (one process per GPU, 127.0.0.1
bootstrap, per-run timeout).  A run passes when it exits 0 and, if the program prints
"PASS"/"FAIL" lines, every rank printed PASS.  With --json-key, the last JSON object that a
run prints is searched for that key and its values are summarised too.  Prints one JSON
object: runs, passed, failed (with exit codes), wall seconds and key stats (mean / std /
min / max / p50 / p90 / p99).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def last_json(text: str):
    for line in reversed(text.splitlines()):
        line = line.strip()
        if line.startswith("{") and line.endswith("}"):
            try:
                return json.loads(line)
            except ValueError:
                continue
    return None


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("-n", type=int, default=1, help="ranks per run")
    ap.add_argument("--repeat", type=int, default=10)
    ap.add_argument("--timeout", type=float, default=300.0)
    ap.add_argument("--json-key", default=None)
    ap.add_argument("cmd", nargs=argparse.REMAINDER)
    args = ap.parse_args()
    cmd = args.cmd[1:] if args.cmd and args.cmd[0] == "--" else args.cmd
    if not cmd:
        raise SystemExit("give the program after --")
    from opengda_b200.parallel.launch import free_port
    from opengda_b200.utils.timing import summarize

    walls, values, failed = [], [], []
    for i in range(args.repeat):
        launch = [sys.executable, "-m", "opengda_b200.parallel.launch", "-n", str(args.n), "--port", str(free_port()),
                  "--timeout", str(args.timeout)] + cmd
        t0 = time.time()
        p = subprocess.run(launch, cwd=ROOT, capture_output=True, text=True, timeout=args.timeout + 60)
        walls.append(time.time() - t0)
        npass, nfail = p.stdout.count("PASS"), p.stdout.count("FAIL")
        ok = p.returncode == 0 and nfail == 0 and (npass in (0, args.n) or npass >= args.n)
        if not ok:
            failed.append({"run": i, "rc": p.returncode, "tail": (p.stdout + p.stderr)[-400:]})
        if args.json_key:
            j = last_json(p.stdout)
            if j is not None and args.json_key in j:
                values.append(float(j[args.json_key]))
    out = {"runs": args.repeat, "ranks": args.n, "passed": args.repeat - len(failed), "failed": failed,
           "wall_s": summarize(walls)}
    if values:
        out[args.json_key] = summarize(values)
    print(json.dumps(out))
    return 0 if not failed else 1


if __name__ == "__main__":
    sys.exit(main())
