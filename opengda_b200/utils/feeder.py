"""Double-buffered host -> device input feeding: the pinned-memory copy of step i+1 runs
on a side stream while step i computes, so PCIe transfers overlap the kernels."""
from __future__ import annotations

from collections import deque

import torch


class HostFeeder:
    def __init__(self, shape, dtype, device, depth: int = 2):
        self.bufs = [torch.empty(tuple(shape), dtype=dtype, device=device) for _ in range(depth)]
        self.ready = [torch.cuda.Event() for _ in range(depth)]
        self.free = [torch.cuda.Event() for _ in range(depth)]
        for e in self.free:
            e.record()
        self.stream = torch.cuda.Stream(device=device)
        self.depth = depth
        self.head = 0  # next buffer to fill
        self.queue: deque = deque()
        self.current = None

    def submit(self, host: torch.Tensor) -> None:
        """Enqueue the copy of `host` (pinned) into the next free device buffer."""
        j = self.head % self.depth
        with torch.cuda.stream(self.stream):
            self.stream.wait_event(self.free[j])
            self.bufs[j].copy_(host, non_blocking=True)
            self.ready[j].record(self.stream)
        self.queue.append(j)
        self.head += 1

    def next(self) -> torch.Tensor:
        """Device buffer of the oldest submitted copy, ordered on the current stream."""
        j = self.queue.popleft()
        torch.cuda.current_stream().wait_event(self.ready[j])
        self.current = j
        return self.bufs[j]

    def release(self) -> None:
        """The current stream's work enqueued so far no longer needs the buffer from next()."""
        self.free[self.current].record()
