"""opengda_b200 -- a Blackwell-native (sm_100a) GPU-initiated communication runtime.

It offers the capabilities and API of GICC/OpenGDA (lwshanbd/OpenGDA), rebuilt for one
8xB200 NVLink 5 / NVSwitch node:

* ``opengda_b200.parallel`` -- socket bootstrap, ``Runtime`` (symmetric memory over CUDA
  VMM, NVLS multicast), ``Barrier`` (incl. continuous mode), active messages, the
  NVSHMEM-style ``init/malloc/remote_ptr`` API and a local multi-rank launcher;
* ``opengda_b200.ops`` -- the sm_100a kernels (tcgen05 GEMM, put/get, barrier,
  allreduce, Jacobi, MoE routing/dispatch/combine) as torch-facing functions;
* ``opengda_b200.models`` -- the workloads: distributed GEMM (AG->GEMM, GEMM->RS),
  the fp32 ring-stripe matmul, Jacobi with fused halo puts (per-iteration or persistent),
  the MoE expert-parallel layer, the CPU matmul;
* ``opengda_b200.baselines`` -- NCCL(+cuBLAS) and host-driven restatements used as the
  comparison arm;
* ``opengda_b200.utils`` -- config, logging, device timing, clock sampling, result
  records, litmus tests, the topology / environment probe, the CUDA-graph capture guard.

The native code lives in ``lib/libgicc.so`` (no torch dependency) and the binding
``_C``; ``python -m opengda_b200._build`` compiles both in place.
"""
from __future__ import annotations

__version__ = "0.1.0"

_native_mod = None


def native():
    """Return the loaded native module, failing loudly if it was not built."""
    global _native_mod
    if _native_mod is None:
        import importlib

        try:
            import torch  # noqa: F401  (loads libc10/libtorch before the binding)

            mod = importlib.import_module(__name__ + "._C")
        except ImportError as e:  # pragma: no cover - exercised only on a broken checkout
            raise ImportError(
                "opengda_b200 native extension is not built; run `python -m opengda_b200._build` "
                f"({e})"
            ) from e
        _native_mod = mod
    return _native_mod
