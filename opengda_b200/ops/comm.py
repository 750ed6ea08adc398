"""Torch-facing one-sided communication over symmetric tensors (the device API of
``csrc/include/gicc/device/comm.cuh`` as stream-ordered kernels):

    x = rt.alloc_tensor((n,), torch.float32)          # symmetric
    put(x, src, peer)                                  # src -> x on `peer`
    put_signal(x, src, peer, rt, word)                 # ... then +1 per block on peer's word
    wait_signal(rt, word, expected)                    # bounded; raises on timeout
    get(dst, x, peer)                                  # x on `peer` -> dst

Every call is enqueued on the current CUDA stream and ends with fence.acq_rel.sys, so the
stores are performed system-wide when the kernel completes.  Offsets and sizes are in
bytes of the symmetric buffer.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import native

CMP = {"eq": 0, "ne": 1, "ge": 2, "gt": 3, "lt": 4, "le": 5}


def _nbytes(t: torch.Tensor) -> int:
    if not t.is_contiguous():
        raise ValueError("tensor must be contiguous")
    return t.numel() * t.element_size()


def _check_range(sym, offset: int, nbytes: int) -> None:
    total = _nbytes(sym.local)
    if offset < 0 or nbytes < 0 or offset + nbytes > total:
        raise ValueError(f"bytes [{offset}, {offset + nbytes}) outside the symmetric buffer of {total} bytes")


def put(dst_sym, src: torch.Tensor, peer: int, offset: int = 0, blocks: int = 0) -> None:
    """Copy ``src`` into ``dst_sym`` on rank ``peer`` at byte ``offset`` (NVLink stores)."""
    n = _nbytes(src)
    _check_range(dst_sym, offset, n)
    native().k_copy(dst_sym.ptr(peer) + offset, src.data_ptr(), n, 1, blocks, 0)


def get(dst: torch.Tensor, src_sym, peer: int, offset: int = 0, blocks: int = 0) -> torch.Tensor:
    """Copy ``src_sym`` on rank ``peer`` (from byte ``offset``) into the local ``dst``."""
    n = _nbytes(dst)
    _check_range(src_sym, offset, n)
    native().k_copy(dst.data_ptr(), src_sym.ptr(peer) + offset, n, 1, blocks, 0)
    return dst


def put_signal(dst_sym, src: torch.Tensor, peer: int, rt, word: int, offset: int = 0, blocks: int = 0) -> int:
    """Put, then every block adds 1 (release) to signal word ``word`` on ``peer`` once its
    slice is visible.  Returns how much the word grows (the number of blocks)."""
    n = _nbytes(src)
    _check_range(dst_sym, offset, n)
    if blocks <= 0:
        blocks = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
    native().k_put_signal(dst_sym.ptr(peer) + offset, src.data_ptr(), n, rt.signal_peer(peer, word), blocks)
    return blocks


def signal(rt, peer: int, word: int, value: int, op: str = "set") -> None:
    """Set or add ``value`` on signal word ``word`` of ``peer`` (release)."""
    if op not in ("set", "add"):
        raise ValueError("op must be 'set' or 'add'")
    native().k_signal(rt.signal_peer(peer, word), int(value), 0 if op == "set" else 1)


def wait_signal(rt, word: int, value: int, cmp: str = "ge", timeout_ns: Optional[int] = None,
                sync: bool = True) -> Optional[torch.Tensor]:
    """Stream-ordered bounded wait until this rank's signal word satisfies ``cmp value``.
    With sync=True the host waits and raises on timeout; otherwise the int32 status tensor
    (0 = ok) is returned for the caller to check later."""
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    native().k_wait_signal(rt.signal_local(word), CMP[cmp], int(value), int(timeout_ns or rt.timeout_ns),
                           status.data_ptr())
    if not sync:
        return status
    if int(status.item()) != 0:
        raise TimeoutError(f"signal word {word} did not reach {cmp} {value} in time")
    return None
