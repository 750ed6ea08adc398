"""Device-side timing: CUDA events on the launching stream, L2 flush between samples,
max over ranks for multi-GPU numbers (the reference times on rank 0 only,
examples/gicc/mm.cu:230-243; here every multi-GPU figure is the slowest rank)."""
from __future__ import annotations

import statistics
from typing import Callable, List

import torch

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2 of B200

_flush_buf = {}


def flush_l2(device=None) -> None:
    """Overwrite a buffer twice the size of L2 so the next kernel starts cold."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    buf = _flush_buf.get(dev)
    if buf is None:
        buf = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
        _flush_buf[dev] = buf
    buf.fill_(1)


def time_device(fn: Callable[[], None], iters: int = 10, warmup: int = 3, flush: bool = True) -> List[float]:
    """Per-iteration device time (ms) of ``fn`` measured with CUDA events."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        if flush:
            flush_l2()
        s = torch.cuda.Event(enable_timing=True)
        e = torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e))
    return out


def summarize(samples: List[float]) -> dict:
    s = sorted(samples)

    def pct(p):
        return s[min(len(s) - 1, int(round(p / 100.0 * (len(s) - 1))))]

    return {
        "mean": statistics.fmean(s),
        "std": statistics.pstdev(s) if len(s) > 1 else 0.0,
        "min": s[0],
        "max": s[-1],
        "p50": pct(50),
        "p90": pct(90),
        "p99": pct(99),
    }


def max_over_ranks(value: float) -> float:
    """Max of a scalar over all ranks of the default process group (identity if none)."""
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    dev = "cuda" if dist.get_backend() == "nccl" else "cpu"
    t = torch.tensor([value], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
