"""Structured benchmark result records and resumable sweeps.

``record(...)`` builds one JSON-ready result with the fields every benchmark of this
package reports: metric, value, unit, n_gpus, shape, dtype, seed, whether the number is the
maximum over ranks, the roofline fraction against the measured peaks of this machine
(``MEASURED_PEAKS.json`` at the repository root when present, else the stated fallbacks),
the verification status, the git commit and a UTC timestamp.

``ResultStore(path)`` is an append-only JSON-lines file keyed by a configuration string:
a sweep calls ``store.done(key)`` to skip configurations finished by an earlier run (after
a crash or a timeout) and ``store.add(key, rec)`` after each one -- resume at the harness
level, since the runtime itself keeps no state worth checkpointing.
"""
from __future__ import annotations

import json
import os
import subprocess
import time
from typing import Any, Dict, Iterable, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

# Used only when MEASURED_PEAKS.json is absent: an earlier measurement on this kind of node.
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0,
                  "nvlink_gbs": 770.0}


def measured_peaks(path: Optional[str] = None) -> Dict[str, Any]:
    """The roofline denominators: measured copy bandwidth (GB/s), cuBLAS bf16 burst and
    sustained TFLOP/s, and the per-direction NVLink peer-copy bandwidth (GB/s)."""
    p = path or os.path.join(ROOT, "MEASURED_PEAKS.json")
    peaks = dict(FALLBACK_PEAKS)
    src = "fallback"
    try:
        with open(p) as f:
            m = json.load(f)
        for k in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained"):
            if isinstance(m.get(k), (int, float)):
                peaks[k] = float(m[k])
        src = "measured"
    except (OSError, ValueError):
        pass
    peaks["source"] = src
    return peaks


def roofline_fraction(achieved: float, kind: str, peaks: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    """achieved / peak for kind in {"hbm_gbs", "bf16_tflops", "bf16_tflops_sustained",
    "nvlink_gbs"}, labelled "of measured" or "of fallback"."""
    peaks = peaks or measured_peaks()
    if kind not in peaks:
        raise ValueError(f"unknown peak kind {kind!r}")
    return {"fraction": achieved / peaks[kind], "of": f"{peaks['source']} {kind} = {peaks[kind]}"}


def _git_commit() -> Optional[str]:
    try:
        out = subprocess.run(["git", "-C", ROOT, "rev-parse", "--short", "HEAD"], capture_output=True, text=True,
                             timeout=10)
        return out.stdout.strip() or None
    except (OSError, subprocess.SubprocessError):
        return None


def record(metric: str, value: float, unit: str, n_gpus: int, shape: Any = None, dtype: Optional[str] = None,
           seed: Optional[int] = None, max_over_ranks: bool = True, verified: Optional[bool] = None,
           roofline: Optional[Dict[str, Any]] = None, **extra) -> Dict[str, Any]:
    rec = {"metric": metric, "value": value, "unit": unit, "n_gpus": n_gpus, "shape": shape, "dtype": dtype,
           "seed": seed, "max_over_ranks": max_over_ranks, "verified": verified, "roofline": roofline,
           "commit": _git_commit(), "utc": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime())}
    rec.update(extra)
    return rec


class ResultStore:
    """Append-only JSON-lines store of finished configurations."""

    def __init__(self, path: str):
        self.path = path
        self._done: Dict[str, Dict[str, Any]] = {}
        if os.path.exists(path):
            with open(path) as f:
                for line in f:
                    line = line.strip()
                    if not line:
                        continue
                    try:
                        row = json.loads(line)
                    except ValueError:  # a line cut short by a crash: that config reruns
                        continue
                    if isinstance(row, dict) and "key" in row:
                        self._done[row["key"]] = row.get("record", {})

    def done(self, key: str) -> bool:
        return key in self._done

    def get(self, key: str) -> Optional[Dict[str, Any]]:
        return self._done.get(key)

    def add(self, key: str, rec: Dict[str, Any]) -> None:
        d = os.path.dirname(os.path.abspath(self.path))
        os.makedirs(d, exist_ok=True)
        with open(self.path, "a") as f:
            f.write(json.dumps({"key": key, "record": rec}) + "\n")
            f.flush()
            os.fsync(f.fileno())
        self._done[key] = rec

    def records(self) -> Iterable[Dict[str, Any]]:
        return list(self._done.values())
