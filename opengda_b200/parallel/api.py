"""NVSHMEM-style API (reference src/gicc/platform/mlx5/gicc_api.hpp:42-129):
``init``, collective ``malloc``, ``free``, ``context``, ``remote_ptr``, ``barrier``,
``my_pe``, ``n_pes``, ``runtime``, ``finalize``.

``remote_ptr`` returns an address that device code dereferences directly (the peer
buffer is mapped into this process), so no translation happens on the device.
"""
from __future__ import annotations

from typing import Optional

import torch

from .runtime import Runtime

_rt: Optional[Runtime] = None
_ctx: Optional[int] = None
_dirty = True
_allocs = {}


def init(runtime: Optional[Runtime] = None) -> Runtime:
    global _rt, _dirty
    if _rt is None:
        _rt = runtime or Runtime()
        _dirty = True
    return _rt


def runtime() -> Runtime:
    if _rt is None:
        raise RuntimeError("gicc: call init() first")
    return _rt


def malloc(nbytes: int, multicast: bool = False) -> int:
    """Collective: symmetric allocation (zeroed), registered and exchanged; returns the local address."""
    global _dirty
    rt = runtime()
    b = rt.native.alloc(nbytes, multicast)
    rt.native.exchange()
    _allocs[b["ptr"]] = b["index"]
    _dirty = True
    return b["ptr"]


def malloc_tensor(shape, dtype=torch.bfloat16, multicast: bool = False):
    global _dirty
    t = runtime().alloc_tensor(shape, dtype, multicast)
    _allocs[t.ptr()] = t.index
    _dirty = True
    return t


def free(ptr: int) -> None:
    """Local: forget the allocation.  Its memory is released at finalize() (VMM mappings
    of peers may still reference it until every rank is done)."""
    _allocs.pop(ptr, None)


def context() -> int:
    """Device address of the GiccContext (rebuilt when allocations changed)."""
    global _ctx, _dirty
    if _ctx is None or _dirty:
        _ctx = runtime().build_context()
        _dirty = False
    return _ctx


def remote_ptr(local_ptr: int, pe: int) -> int:
    return runtime().native.translate(int(local_ptr), pe)


def barrier() -> None:
    runtime().barrier()


def my_pe() -> int:
    return runtime().rank


def n_pes() -> int:
    return runtime().size


def finalize() -> None:
    global _rt, _ctx, _dirty
    if _rt is not None:
        torch.cuda.synchronize()
        _rt.finalize()
    _rt, _ctx, _dirty = None, None, True
    _allocs.clear()
