"""Sample SM clocks / throttle reasons with nvidia-smi while a timed region runs."""
from __future__ import annotations

import shutil
import statistics
import subprocess
import tempfile
import time
from typing import List, Optional

QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
REASONS = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]


class ClockSampler:
    """``with ClockSampler(gpus) as cs: ...`` then ``cs.summary()``.

    ``__enter__`` returns only after nvidia-smi has written its first sample (it takes a
    fraction of a second to start), and the summary keeps only the samples written after
    that point, so a timed region of a few hundred milliseconds still gets samples of its
    own.  ``__exit__`` waits for one more sample when the region produced none."""

    def __init__(self, gpus: Optional[List[int]] = None, period_ms: int = 50, start_timeout_s: float = 5.0):
        self.gpus = gpus
        self.period_ms = period_ms
        self.start_timeout_s = start_timeout_s
        self.proc = None
        self.file = None
        self.skip = 0

    def _lines(self) -> int:
        self.file.flush()
        with open(self.file.name) as f:
            return sum(1 for _ in f)

    def _wait_lines(self, n: int, timeout_s: float) -> None:
        t0 = time.monotonic()
        while self._lines() < n and time.monotonic() - t0 < timeout_s and self.proc.poll() is None:
            time.sleep(0.01)

    def __enter__(self):
        if shutil.which("nvidia-smi") is None:
            return self
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        cmd = ["nvidia-smi", f"--query-gpu={QUERY}", "--format=csv,noheader,nounits", f"-lms={self.period_ms}"]
        if self.gpus is not None:
            cmd.insert(1, "-i=" + ",".join(str(g) for g in self.gpus))
        self.proc = subprocess.Popen(cmd, stdout=self.file, stderr=subprocess.DEVNULL)
        per_round = len(self.gpus) if self.gpus is not None else 1
        self._wait_lines(per_round, self.start_timeout_s)
        self.skip = self._lines()
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            if self._lines() <= self.skip:
                self._wait_lines(self.skip + 1, 4 * self.period_ms / 1000 + 0.5)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        if self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.file.flush()
        rows = []
        with open(self.file.name) as f:
            for i, line in enumerate(f):
                if i < self.skip:
                    continue
                parts = [p.strip() for p in line.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    rows.append((int(parts[0]), float(parts[1]), float(parts[2]), parts[3], parts[5:9]))
                except ValueError:
                    continue
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        mx = max(r[2] for r in rows)
        loaded = [r for r in rows if r[1] > 0.3 * mx] or rows
        reasons = set()
        for r in loaded:
            for name, v in zip(REASONS, r[4]):
                if v.lower() == "active":
                    reasons.add(name)
        watts = []
        for r in loaded:
            try:
                watts.append(float(r[3]))
            except ValueError:
                pass
        out = {"sm_mhz": statistics.median(r[1] for r in loaded), "sm_max_mhz": mx,
               "reasons": sorted(reasons), "samples": len(rows)}
        if watts:
            out["power_w"] = round(statistics.median(watts), 1)
        return out


def gather_clock_summary(summary: dict) -> dict:
    """Combine every rank's ``ClockSampler.summary()`` (collective over the default
    torch.distributed group when it is initialised): the lowest per-rank median SM clock,
    the union of throttle reasons and the per-rank medians."""
    try:
        import torch.distributed as dist
        multi = dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1
    except Exception:  # pragma: no cover
        multi = False
    if not multi:
        return summary
    allc = [None] * dist.get_world_size()
    dist.all_gather_object(allc, summary)
    sm = [c.get("sm_mhz") for c in allc]
    known = [v for v in sm if v]
    return {"sm_mhz": min(known) if known else None, "sm_max_mhz": allc[0].get("sm_max_mhz"),
            "reasons": sorted({r for c in allc for r in c.get("reasons", [])}), "per_rank_sm_mhz": sm}


class BenchClocks:
    """Clock record for a whole benchmark run: ``clk = BenchClocks(local_gpu)`` starts
    sampling; ``clk.finish()`` (a collective when several ranks run) stops it and returns
    the combined record, to be embedded in the benchmark's JSON."""

    def __init__(self, gpu: int, period_ms: int = 100):
        self._cs = ClockSampler([gpu], period_ms=period_ms)
        self._cs.__enter__()

    def finish(self) -> dict:
        self._cs.__exit__(None, None, None)
        return gather_clock_summary(self._cs.summary())
