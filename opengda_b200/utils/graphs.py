"""CUDA-graph capture guard.

The ops of this package pass their call counters (epochs) to the kernels as arguments, so
a call captured in a CUDA graph would replay with a stale counter: its waits would be
satisfied by the previous call's signals.  Entry points that are not capturable call
``refuse_capture`` first; ``Allreduce(graph_safe=True)`` keeps its counter on the device and
is capturable.
"""
from __future__ import annotations


def capturing() -> bool:
    try:
        import torch
        return bool(torch.cuda.is_available() and torch.cuda.is_current_stream_capturing())
    except Exception:  # no CUDA runtime here
        return False


def refuse_capture(what: str) -> None:
    if capturing():
        raise RuntimeError(f"{what} cannot be captured in a CUDA graph: its call counter is a kernel argument "
                           "and a replay would reuse it")
