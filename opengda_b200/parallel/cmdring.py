"""``gicc::CmdRing`` from Python: host-queued transfers executed by a persistent kernel.

    ring = CmdRing(rt)            # one CTA, 64 slots, exits after 10 s without commands
    ring.start()
    seq = ring.put(src.data_ptr(), dst_rank, buf.index, offset, nbytes)
    ring.signal(dst_rank, word, value)
    ring.wait(seq); ring.stop()

While the ring kernel is resident, the first launch of a kernel this process has not yet
loaded (CUDA lazy module loading) waits until the ring exits -- warm such kernels up before
``start()`` or set ``CUDA_MODULE_LOADING=EAGER``.

The reference has the same component, unused, for its NIC path
(src/gicc/platform/mlx5/persistent.cuh:27-47, 239-311).
"""
from __future__ import annotations

from .. import native
from .runtime import Runtime


class CmdRing:
    def __init__(self, rt: Runtime, nslots: int = 64, threads: int = 256, idle_timeout_ms: int = 10000):
        self.rt = rt
        self._r = native().CmdRing(rt.native, nslots, threads, idle_timeout_ms)

    def start(self) -> None:
        self._r.start()

    def put(self, src_ptr: int, dst_rank: int, dst_buf: int, dst_off: int, size: int, user: int = 0) -> int:
        return self._r.put(src_ptr, dst_rank, dst_buf, dst_off, size, user)

    def get(self, dst_ptr: int, src_rank: int, src_buf: int, src_off: int, size: int, user: int = 0) -> int:
        return self._r.get(dst_ptr, src_rank, src_buf, src_off, size, user)

    def signal(self, dst_rank: int, word: int, value: int) -> int:
        return self._r.signal(dst_rank, word, value)

    def add(self, dst_rank: int, word: int, value: int) -> int:
        return self._r.add(dst_rank, word, value)

    def fence(self) -> int:
        return self._r.fence()

    def wait(self, seq: int) -> None:
        self._r.wait(seq)

    def completed(self) -> int:
        return self._r.completed()

    def stop(self) -> None:
        self._r.stop()

    def status(self) -> int:
        return self._r.status()

    @property
    def running(self) -> bool:
        return self._r.running
