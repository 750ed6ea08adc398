"""Ring-stripe fp32 matmul benchmark (the reference's distributed-matmul example,
examples/gicc/mm.cu: N x N fp32, row stripes of A, column stripes of B moving around the
ring; default N = 4096 as there): this framework's ring (the step kernel pushes the stripe
over NVLink while its other CTAs split it into tf32 parts for a tcgen05 GEMM, or run the
fp32 SIMT SGEMM with --simt) against NCCL send/recv + cuBLAS fp32 SGEMM (tf32 off), both timed
on the device as the max over ranks, with an fp64 CPU check of sampled elements of C.

    python bench/ring_mm_bench.py [--size 4096] [--simt]
    torchrun --nproc-per-node N bench/ring_mm_bench.py
"""
from __future__ import annotations

import argparse
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", dest="n", type=int, default=4096, help="matrix edge N")
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--push-ctas", type=int, default=8)
    ap.add_argument("--samples", type=int, default=1000)
    ap.add_argument("--no-baseline", action="store_true")
    ap.add_argument("--simt", action="store_true", help="the fp32 SIMT SGEMM step instead of the tf32 tensor-core one")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    rt = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
        from opengda_b200.parallel import Runtime
        rt = Runtime()
    rank = rt.rank if rt else 0
    from opengda_b200.models.ring_mm import RingMatmul, make_stripes
    from opengda_b200.utils.timing import max_over_ranks

    N = args.n
    mm = RingMatmul(N, rt=rt, push_ctas=args.push_ctas, tensor_cores=False if args.simt else None)
    A_s, B_s, A, B = make_stripes(N, world, rank, seed=0)

    def timeit(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / args.steps)

    C = mm(A_s, B_s)
    torch.cuda.synchronize()
    if rt:
        rt.check_device_errors()
    # fp64 check of sampled elements of this rank's stripe
    g = torch.Generator().manual_seed(100 + rank)
    Ns = N // world
    ii = torch.randint(0, Ns, (args.samples,), generator=g)
    jj = torch.randint(0, N, (args.samples,), generator=g)
    Cc = C.cpu()
    prod = A[rank * Ns + ii].double() * B[:, jj].t().double()
    ref, scale = prod.sum(1), prod.abs().sum(1)
    # error relative to sum |a_k b_k| (the scale of fp32 accumulation error); a wrong or
    # missing column block gives O(1) here
    err = ((Cc[ii, jj].double() - ref).abs() / scale).max().item()
    bad = int(max_over_ranks(float(err > 2e-5)))
    ms = timeit(lambda: mm(A_s, B_s, C))
    if rt:
        rt.check_device_errors()
    res = {"metric": "ring_mm_ms", "impl": "ours", "n_gpus": world, "N": N, "dtype": "fp32",
           "ms": ms, "tflops_total": mm.flops() / (ms * 1e-3) / 1e12, "max_rel_err_sampled": err,
           "verified": bad == 0, "push_ctas": mm.push_ctas,
           "mode": "tensor cores (3 x tf32)" if mm.tensor_cores else "fp32 SIMT"}
    if not args.no_baseline and world > 1:
        from opengda_b200.baselines.ring_mm_nccl import NcclRingMatmul
        base = NcclRingMatmul(N)
        Cb = base(A_s, B_s)
        res["rel_diff_vs_baseline"] = float(((C - Cb).norm() / Cb.norm()).item())
        ms_b = timeit(lambda: base(A_s, B_s, Cb))
        res["nccl_cublas"] = {"ms": ms_b, "tflops_total": mm.flops() / (ms_b * 1e-3) / 1e12}
    if rank == 0:
        js = json.dumps(res)
        print(js)
        if args.out:
            with open(args.out, "w") as f:
                f.write(js + "\n")
    if world > 1:
        del mm
        torch.cuda.synchronize()
        rt.finalize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
