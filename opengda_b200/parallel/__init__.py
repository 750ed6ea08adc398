"""Process plane and NVLink transport: bootstrap, Runtime, Barrier, active messages,
the NVSHMEM-style API and the local launcher."""
from .bootstrap import Bootstrap, allreduce_max, allreduce_min, allreduce_sum  # noqa: F401
from .runtime import Barrier, Runtime, SymmetricTensor, tensor_at  # noqa: F401
