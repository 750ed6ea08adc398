"""Double-buffered host -> device input feeding: the pinned-memory copy of step i+1 runs
on a side stream while step i computes, so PCIe transfers overlap the kernels.

The device buffers can be the consumer's own input slots (``bufs=``), e.g. the two
symmetric A slots of a fused ``DistGemm`` in the order of its next calls
(``DistGemm.input_slots()``): the copy then lands where the kernel reads it, with no
device-to-device copy that could queue behind the next step's host copy."""
from __future__ import annotations

from collections import deque

import torch


class HostFeeder:
    def __init__(self, shape, dtype, device, depth: int = 2, bufs=None):
        if bufs is not None:
            bufs = list(bufs)
            if len(bufs) < 2 or any(tuple(b.shape) != tuple(shape) or b.dtype != dtype for b in bufs):
                raise ValueError("HostFeeder: bufs must be two or more device tensors of the given shape and dtype")
            depth = len(bufs)
        self.bufs = bufs or [torch.empty(tuple(shape), dtype=dtype, device=device) for _ in range(depth)]
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
