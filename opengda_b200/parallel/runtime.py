"""Python face of ``gicc::Runtime`` (csrc/src/runtime.cpp) and ``gicc::Barrier``.

Adds torch conveniences on top of the reference method set (register_buffer, exchange,
remote_buffer, prepare, build_context, reset, barrier, put_no_db / prepare_trigger /
wait): symmetric tensors (``alloc_tensor``) whose peer copies and NVLS multicast views
are ordinary torch tensors.
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .. import native
from .bootstrap import Bootstrap

_DTYPE_NAMES = {
    torch.bfloat16: "bfloat16", torch.float16: "float16", torch.float32: "float32", torch.float64: "float64",
    torch.int32: "int32", torch.int64: "int64", torch.uint8: "uint8", torch.int8: "int8",
}


def tensor_at(ptr: int, shape: Sequence[int], dtype: torch.dtype, device: int) -> torch.Tensor:
    """Zero-copy tensor over device memory owned elsewhere (peer mapping, multicast VA)."""
    return native().tensor_from_ptr(int(ptr), list(shape), _DTYPE_NAMES[dtype], int(device))


class SymmetricTensor:
    """A tensor allocated at the same index on every rank, with its peers' views."""

    def __init__(self, rt: "Runtime", index: int, shape, dtype):
        self.rt = rt
        self.index = index
        self.shape = tuple(shape)
        self.dtype = dtype
        self.local = tensor_at(rt.native.buffer(index)["ptr"], shape, dtype, rt.gpu_id)
        self._peers: dict = {}

    def peer(self, rank: int) -> torch.Tensor:
        """This buffer on ``rank``, mapped into this process (NVLink loads/stores)."""
        if rank == self.rt.rank:
            return self.local
        t = self._peers.get(rank)
        if t is None:
            t = tensor_at(self.rt.native.remote_ptr(rank, self.index, 0), self.shape, self.dtype, self.rt.gpu_id)
            self._peers[rank] = t
        return t

    def peers(self) -> List[torch.Tensor]:
        return [self.peer(r) for r in range(self.rt.size)]

    def multicast(self) -> Optional[torch.Tensor]:
        """NVLS multicast view (multimem.* only -- plain loads/stores through it are invalid)."""
        p = self.rt.native.multicast_ptr(self.index)
        return None if p == 0 else tensor_at(p, self.shape, self.dtype, self.rt.gpu_id)

    def ptr(self, rank: Optional[int] = None) -> int:
        if rank is None or rank == self.rt.rank:
            return self.rt.native.buffer(self.index)["ptr"]
        return self.rt.native.remote_ptr(rank, self.index, 0)

    @property
    def mc_ptr(self) -> int:
        return self.rt.native.multicast_ptr(self.index)


class Runtime:
    def __init__(self, boot: Optional[Bootstrap] = None, device: int = -1, signal_heap_bytes: int = 4 << 20,
                 enable_multicast: bool = True):
        if boot is None:
            import torch.distributed as dist

            boot = Bootstrap.from_torch() if dist.is_available() and dist.is_initialized() else Bootstrap.from_env()
        self.boot = boot
        opt = native().RuntimeOptions()
        opt.device = device
        opt.signal_heap_bytes = signal_heap_bytes
        opt.enable_multicast = enable_multicast
        self.native = native().Runtime(boot.native, opt)
        torch.cuda.set_device(self.gpu_id)

    # reference API -------------------------------------------------------------------------
    @property
    def rank(self) -> int:
        return self.native.rank

    @property
    def size(self) -> int:
        return self.native.size

    @property
    def gpu_id(self) -> int:
        return self.native.gpu_id

    def clock_rate_khz(self) -> float:
        return self.native.clock_rate_khz()

    def gpu_name(self) -> str:
        return self.native.gpu_name()

    def register_buffer(self, t_or_ptr, size: Optional[int] = None, is_device: bool = True) -> dict:
        if isinstance(t_or_ptr, torch.Tensor):
            return self.native.register_buffer(t_or_ptr.data_ptr(), t_or_ptr.numel() * t_or_ptr.element_size(),
                                               t_or_ptr.is_cuda)
        return self.native.register_buffer(int(t_or_ptr), int(size), is_device)

    def exchange(self) -> None:
        self.native.exchange()

    def remote_buffer(self, rank: int, index: int):
        return self.native.remote_buffer(rank, index)

    def prepare(self, peer: int = -1, remote_buf_index: int = 0) -> int:
        return self.native.prepare(peer, remote_buf_index)

    def build_context(self) -> int:
        return self.native.build_context()

    def reset(self) -> None:
        self.native.reset()

    def barrier(self) -> None:
        self.native.barrier()

    def put_no_db(self, src_index: int, dest_rank: int, dest_index: int, size: int, src_off: int = 0,
                  dst_off: int = 0):
        return self.native.put_no_db(src_index, dest_rank, dest_index, size, src_off, dst_off)

    def prepare_trigger(self, token) -> int:
        return self.native.prepare_trigger(*token)

    def wait(self, token) -> None:
        self.native.wait(*token)

    # additions -----------------------------------------------------------------------------
    @property
    def multicast_supported(self) -> bool:
        return self.native.multicast_supported

    def alloc_tensor(self, shape, dtype=torch.bfloat16, multicast: bool = False, exchange: bool = True
                     ) -> SymmetricTensor:
        """Collective: a symmetric tensor (same shape/dtype on every rank)."""
        n = 1
        for s in shape:
            n *= int(s)
        nbytes = n * torch.empty((), dtype=dtype).element_size()
        b = self.native.alloc(max(nbytes, 1), multicast)
        if exchange:
            self.native.exchange()
        return SymmetricTensor(self, b["index"], shape, dtype)

    def signal_alloc(self, nwords: int) -> int:
        return self.native.signal_alloc(nwords)

    def signal_local(self, word: int = 0) -> int:
        return self.native.signal_local(word)

    def signal_peer(self, rank: int, word: int = 0) -> int:
        return self.native.signal_peer(rank, word)

    def signal_multicast(self, word: int = 0) -> int:
        return self.native.signal_multicast(word)

    @property
    def timeout_ns(self) -> int:
        return self.native.timeout_ns

    def check_device_errors(self, clear: bool = True) -> None:
        self.native.check_device_errors(clear)

    def finalize(self) -> None:
        self.native.finalize()


class Barrier:
    """``gicc::Barrier`` (reference: platform/ofi/internal/gicc_barrier.hpp:57-300)."""

    def __init__(self, rt: Runtime, nvls: bool = False):
        self.rt = rt
        self._b = native().Barrier(rt.native, nvls)

    def init(self):
        self._b.init()

    def finalize(self):
        self._b.finalize()

    def setup(self):
        self._b.setup()

    def wait_completion(self):
        self._b.wait_completion()

    def reset(self):
        self._b.reset()

    def start_continuous(self, n: int):
        self._b.start_continuous(n)

    def wait_continuous(self):
        self._b.wait_continuous()

    def device_ctx(self) -> int:
        return self._b.device_ctx()

    def count(self) -> int:
        return self._b.count()

    @property
    def uses_nvls(self) -> bool:
        return self._b.uses_nvls

    # failure detection tests ---------------------------------------------------------------
    SKIP_SIGNAL, STALE_EPOCH = 1, 2

    def inject_fault(self, mode: int, after: int = 0, timeout_ms: int = 0) -> int:
        """Make this rank misbehave in the barrier ``after`` barriers from now: leave its
        signal out (``SKIP_SIGNAL``) or send the previous epoch (``STALE_EPOCH``).  The peers
        (and possibly this rank) end that barrier with ETIMEDOUT after ``timeout_ms``;
        nothing faults or hangs.  Returns the epoch of the affected barrier."""
        epoch = self._b.next_epoch + after
        self._b.inject_fault(mode, epoch, timeout_ms)
        return epoch

    # kernels -------------------------------------------------------------------------------
    def run_single(self, flag_ptr: int = 0) -> None:
        """setup() + one device barrier kernel (reference examples/ofi/barrier_test.cpp:20-24)."""
        self._b.setup()
        native().k_barrier_single(self._b.device_ctx(), flag_ptr)

    def device_barrier(self, n: int = 1) -> None:
        """Enqueue n barriers on the current stream; the kernel advances the epoch itself,
        so no host memory copy is involved (CUDA-graph capturable)."""
        self._b.advance(n)
        native().k_barrier_continuous(self._b.device_ctx(), n, 0)

    def run_continuous(self, n: int, counter_ptr: int = 0) -> None:
        """start_continuous(n) + one kernel running n barriers (barrier_test.cpp:32-41)."""
        self._b.start_continuous(n)
        native().k_barrier_continuous(self._b.device_ctx(), n, counter_ptr)
