"""Distributed GEMM workload (placeholder: single-GPU path; modes added next)."""
from __future__ import annotations

import torch


def smoke_step(device: torch.device) -> None:
    from ..ops.gemm import gemm, check_errors

    g = torch.Generator(device=device).manual_seed(2)
    A = torch.randn(256, 512, device=device, generator=g).to(torch.bfloat16)
    B = torch.randn(256, 512, device=device, generator=g).to(torch.bfloat16)
    C = gemm(A, B)
    torch.cuda.synchronize(device)
    check_errors()
    ref = A.float() @ B.float().t()
    err = (C.float() - ref).abs().max().item()
    if err > 1e-2 * ref.abs().max().item() + 1e-2:
        raise RuntimeError(f"smoke: GEMM mismatch {err}")
