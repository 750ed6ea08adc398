"""Active messages (reference: src/gicc/platform/ofi/internal/am.hpp:70-373 host class,
platform/mlx5/am_device.cuh device ops) over NVLink symmetric rings.

Handler ids: NOOP=0, COUNTER_ADD=1 (counter += args[0]), CHECKSUM=2 (checksum += sum of
payload bytes), ECHO=3 (requests are answered with args[0]), USER_BASE=100.
"""
from __future__ import annotations

from typing import Sequence

from .. import native

NOOP, COUNTER_ADD, CHECKSUM, ECHO, USER_BASE = 0, 1, 2, 3, 100


class Am:
    def __init__(self, rt, nslots: int = 128, max_payload: int = 8192):
        self.rt = rt
        self._a = native().Am(rt.native, nslots, max_payload)

    def send_handle(self, dst: int, handler: int, args: Sequence[int] = (), request: bool = False) -> int:
        return self._a.send_handle(dst, handler, list(args), request)

    def send_payload(self, dst: int, handler: int, args: Sequence[int], payload: bytes) -> int:
        return self._a.send_payload(dst, handler, list(args), payload)

    def check_can_send(self, dst: int) -> bool:
        return self._a.check_can_send(dst)

    def poll_once(self, max_per_peer: int = 64) -> int:
        return self._a.poll_once(max_per_peer)

    def reply(self, src: int, seq: int, value: int) -> None:
        self._a.reply(src, seq, value)

    def wait_reply(self, dst: int, seq: int) -> int:
        return self._a.wait_reply(dst, seq)

    def trigger_and_wait(self) -> None:
        self._a.trigger_and_wait()

    def counter(self) -> int:
        return self._a.counter()

    def checksum(self) -> int:
        return self._a.checksum()

    def device_view(self) -> int:
        return self._a.device_view()

    def pingpong(self, peer: int, iters: int, mode: str, initiator: bool, out_ptr: int) -> None:
        """Device-driven AM round trips (mode "reqrep": 64-B request, 8-B reply; "reqreq")."""
        native().k_am_pingpong(self._a.device_view(), peer, iters, 0 if mode == "reqrep" else 1, initiator, out_ptr)
