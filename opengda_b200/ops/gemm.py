"""tcgen05 GEMM: ``C = alpha * A @ B^T`` with A[M,K], B[N,K] bf16 (K-major both)."""
from __future__ import annotations

import torch

from .. import native


def gemm(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
         out_dtype: torch.dtype = torch.bfloat16, bn: int = 0) -> torch.Tensor:
    """Run the persistent warp-specialised tcgen05 GEMM (csrc/kernels/gemm.cu).

    A is [M, K], B is [N, K] (the nn.Linear weight layout); both bf16, row-major.
    Accumulation is f32 in TMEM; the output is bf16 or f32.  ``bn`` picks the tile:
    128 or 256 (one CTA, 128 x bn), 512 (CTA pairs, 256 x 256), 1024 (CTA pairs, 256 x 512)
    or 0 (the default for the shape).
    """
    if out_dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("out_dtype must be bfloat16 or float32")
    return native().gemm(A, B, out, float(alpha), out_dtype == torch.float32, int(bn))


def gemm_fp32(A: torch.Tensor, B: torch.Tensor, out: torch.Tensor | None = None, alpha: float = 1.0,
              bn: int = 0) -> torch.Tensor:
    """fp32 C = alpha * A @ B^T on the tcgen05 tensor cores (csrc/kernels/gemm.cu, gemm_fp32).

    A [M, K] and B [N, K] fp32 (K % 4 == 0, rows 16-byte aligned).  Each operand is split
    into its tf32 part and the remainder, and the three products hi.hi + hi.lo + lo.hi run
    as one kind::tf32 GEMM over 3K with f32 accumulation: the error stays within a few
    2^-21 of |A||B| per term (fp32 FMA: 2^-24), at tensor-core rather than CUDA-core speed.
    Uses (M + N) * 3K floats of workspace.  ``bn`` picks the tile as in ``gemm`` (256 one CTA,
    512 / 1024 CTA pairs with 256 x 256 / 256 x 512 tiles, 0 by shape)."""
    return native().gemm_fp32(A, B, out, float(alpha), int(bn))


def set_tuning(group_m: int = 16, l2_hint: int = 0, pair_group_m: int = 16, pair_l2_hint: int = 0,
               pair_prefetch: int = 0, pair_tma_store: int = 1) -> None:
    """Process-wide tuning of ``gemm`` (A/B experiments; the defaults are the measured
    configuration): m-blocks per raster group, L2 eviction hints on the operand loads
    (0 none, 1 keep A / stream B, 2 keep B / stream A), the CTA-pair kernel's raster
    group (256-row m-blocks), its L2 hints (same codes) and how many k-steps ahead its
    producer prefetches the operands into L2 (0 = no prefetch), and whether it stores bf16 C
    through shared memory and TMA (1) or from each thread's registers (0)."""
    native().set_gemm_tuning(int(group_m), int(l2_hint), int(pair_group_m), int(pair_l2_hint), int(pair_prefetch),
                             int(pair_tma_store))


def tuning() -> dict:
    return dict(native().gemm_tuning())


def check_errors(clear: bool = True) -> None:
    """Raise if a kernel of this library recorded a device-side error (timeout, bounds)."""
    rec = native().read_errors(clear)
    if rec["code"] != 0:
        raise RuntimeError(f"gicc device error: {rec}")
