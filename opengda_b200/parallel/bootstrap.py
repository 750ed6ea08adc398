"""Process-plane bootstrap (native ``gicc::Bootstrap``: a socket key-value store).

Three ways to get one:

* ``Bootstrap.from_env()`` -- GICC_RANK/GICC_SIZE/GICC_BOOTSTRAP_ADDR (set by
  ``opengda_b200.parallel.launch``) or torchrun's RANK/WORLD_SIZE/MASTER_ADDR/MASTER_PORT;
* ``Bootstrap.create(rank, size, addr)`` -- explicit; rank 0 serves at ``addr``;
* ``Bootstrap.from_torch()`` -- next to an initialised ``torch.distributed`` group: rank 0
  binds a free port and publishes it through the group's store.

The method set follows the reference's MPI/PMI2 bootstrap
(src/gicc/bootstrap/detail/bootstrap_mpi.hpp:70-159).
"""
from __future__ import annotations

import pickle
import struct
from typing import Any, List

from .. import native


def BootstrapError():  # noqa: N802 - exception class accessor
    return native().BootstrapError


class Bootstrap:
    def __init__(self, impl):
        self._b = impl

    # ---- construction ------------------------------------------------------------------
    @classmethod
    def from_env(cls) -> "Bootstrap":
        return cls(native().Bootstrap())

    @classmethod
    def create(cls, rank: int, size: int, addr: str, timeout_s: float = -1.0, setup: bool = True) -> "Bootstrap":
        b = native().Bootstrap(rank, size, addr, timeout_s)
        if setup:
            b.setup()
        return cls(b)

    @classmethod
    def from_torch(cls, timeout_s: float = -1.0) -> "Bootstrap":
        import os

        import torch.distributed as dist

        if not dist.is_initialized():
            raise RuntimeError("Bootstrap.from_torch needs an initialised torch.distributed process group")
        rank, size = dist.get_rank(), dist.get_world_size()
        host = os.environ.get("MASTER_ADDR", "127.0.0.1")
        if rank == 0:
            b = native().Bootstrap(0, size, f"{host}:0", timeout_s)
            obj = [f"{host}:{b.server_port}"]
        else:
            obj = [None]
        dist.broadcast_object_list(obj, src=0)
        if rank != 0:
            b = native().Bootstrap(rank, size, obj[0], timeout_s)
        local_rank = int(os.environ.get("LOCAL_RANK", "-1"))
        local_size = int(os.environ.get("LOCAL_WORLD_SIZE", "-1"))
        b.setup(local_rank, local_size)
        return cls(b)

    # ---- reference API -----------------------------------------------------------------
    @property
    def native(self):
        return self._b

    def rank(self) -> int:
        return self._b.rank

    def size(self) -> int:
        return self._b.size

    def local_rank(self) -> int:
        return self._b.local_rank

    def local_size(self) -> int:
        return self._b.local_size

    def locality_map(self) -> List[bool]:
        return list(self._b.locality_map())

    def barrier(self) -> None:
        self._b.barrier()

    def allgather(self, data: bytes) -> List[bytes]:
        return list(self._b.allgather(bytes(data)))

    def allgather_obj(self, obj: Any) -> List[Any]:
        return [pickle.loads(x) for x in self._b.allgather(pickle.dumps(obj))]

    def allgather_fixed(self, fmt: str, value) -> list:
        """``allgather_fixed<T>``: every rank contributes one struct of format ``fmt``."""
        raw = self._b.allgather(struct.pack(fmt, value))
        sz = struct.calcsize(fmt)
        for r in raw:
            if len(r) != sz:
                raise BootstrapError()("allgather_fixed: size mismatch across ranks")
        return [struct.unpack(fmt, r)[0] for r in raw]

    def broadcast(self, data: bytes | None, root: int = 0) -> bytes:
        return self._b.broadcast(data if data is not None else b"", root)

    def broadcast_obj(self, obj: Any, root: int = 0) -> Any:
        return pickle.loads(self._b.broadcast(pickle.dumps(obj) if self.rank() == root else b"", root))

    def send(self, data: bytes, dst: int, tag: int = 0) -> None:
        self._b.send(bytes(data), dst, tag)

    def recv(self, nbytes: int, src: int, tag: int = 0) -> bytes:
        return self._b.recv(nbytes, src, tag)

    def sendrecv(self, data: bytes, dst: int, nbytes: int, src: int, tag: int = 0) -> bytes:
        return self._b.sendrecv(bytes(data), dst, nbytes, src, tag)

    def wtime(self) -> float:
        return self._b.wtime()

    def check(self) -> None:
        self._b.check()

    def abort(self, code: int, msg: str) -> None:
        """Fail the job for every rank and exit this process (reference gicc::abort)."""
        self._b.abort_job(code, msg)

    def fail_job(self, code: int, msg: str) -> None:
        self._b.fail_job(code, msg)

    def kv_put(self, key: str, value: bytes) -> None:
        self._b.kv_put(key, value)

    def kv_get(self, key: str, consume: int = 0) -> bytes:
        return self._b.kv_get(key, consume)


# ---- host reductions (reference src/gicc/coll.hpp:15-39) ------------------------------------
def allreduce_sum(boot: Bootstrap, value: float, fmt: str = "d"):
    return sum(boot.allgather_fixed(fmt, value))


def allreduce_min(boot: Bootstrap, value: float, fmt: str = "d"):
    return min(boot.allgather_fixed(fmt, value))


def allreduce_max(boot: Bootstrap, value: float, fmt: str = "d"):
    return max(boot.allgather_fixed(fmt, value))
