"""Small single-GPU workloads for kernel profiling (ncu) -- one kernel family per case,
a few launches, a few GB on the device at most.

    python bench/profile_kernels.py gemm 8192          # k_gemm_bf16 (128 x 256 tiles), 4 launches
    python bench/profile_kernels.py gemm_pair 8192     # k_gemm_bf16_pair<1> (CTA pairs, 256 x 256), 4 launches
    python bench/profile_kernels.py gemm_pair_wide 8192  # k_gemm_bf16_pair<2> (CTA pairs, 256 x 512), 4 launches
    python bench/profile_kernels.py cublas 8192        # torch.matmul (cuBLAS) on the same operands, 4 launches
    python bench/profile_kernels.py gemm_fp32 8192     # k_tf32_split x 2 + k_gemm_tf32 (fp32 on the tensor cores), 4 calls
    python bench/profile_kernels.py sgemm 8192         # torch.matmul fp32 (cuBLAS SGEMM, tf32 off), 4 launches
    python bench/profile_kernels.py jacobi 8192 8192   # k_jacobi, 4 launches
    python bench/profile_kernels.py moe 1024           # MoE layer (n=1), 2 forwards
    python bench/profile_kernels.py copy 268435456     # k_copy (local HBM copy)

Example capture (after the same command has exited 0 without ncu):
    ncu --set full --clock-control none -k regex:k_gemm_bf16 -s 2 -c 1 \
        -o prof/gemm8k python bench/profile_kernels.py gemm 8192
"""
from __future__ import annotations

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402


def main():
    case = sys.argv[1]
    args = [int(a) for a in sys.argv[2:]]
    from opengda_b200 import native
    from opengda_b200.ops.gemm import check_errors, gemm
    torch.manual_seed(0)
    if case in ("gemm", "gemm_pair", "gemm_pair_wide", "cublas"):
        M = N = K = args[0] if args else 8192
        A = torch.randn(M, K, device="cuda").to(torch.bfloat16)
        B = torch.randn(N, K, device="cuda").to(torch.bfloat16)
        C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        bn = {"gemm": 256, "gemm_pair": 512, "gemm_pair_wide": 1024}.get(case)
        for _ in range(4):
            if bn is None:
                torch.matmul(A, B.t(), out=C)
            else:
                gemm(A, B, out=C, bn=bn)
    elif case in ("gemm_fp32", "sgemm"):
        from opengda_b200.ops.gemm import gemm_fp32
        torch.backends.cuda.matmul.allow_tf32 = False
        M = N = K = args[0] if args else 8192
        A = torch.randn(M, K, device="cuda")
        B = torch.randn(N, K, device="cuda")
        C = torch.empty(M, N, device="cuda")
        for _ in range(4):
            if case == "sgemm":
                torch.matmul(A, B.t(), out=C)
            else:
                gemm_fp32(A, B, out=C)
    elif case == "jacobi":
        from opengda_b200.models.jacobi import Jacobi
        nx = args[0] if args else 8192
        ny = args[1] if len(args) > 1 else nx
        Jacobi(nx, ny).run(4)
    elif case == "moe":
        from opengda_b200.models.moe import MoELayer, make_inputs
        T = args[0] if args else 1024
        layer = MoELayer(T, 7168, 32, 8, 2048, rt=None)
        x, logits = make_inputs(T, 7168, 32, 0)
        for _ in range(2):
            layer(x, logits)
    elif case == "copy":
        n = args[0] if args else 1 << 28
        a = torch.empty(n, dtype=torch.uint8, device="cuda")
        b = torch.empty(n, dtype=torch.uint8, device="cuda")
        for _ in range(4):
            native().k_copy(b.data_ptr(), a.data_ptr(), n)
    else:
        raise SystemExit(f"unknown case {case}")
    torch.cuda.synchronize()
    check_errors()
    print("ok")


if __name__ == "__main__":
    main()
