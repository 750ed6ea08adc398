"""Distributed GEMM (M = N = K = 16384, bf16) on N GPUs: the fused kernels' options side by side
with the NCCL + cuBLAS arm, in one process per GPU on one box.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/dist_gemm_variants.py \
        [--ag "nvls,units,pair[,transfer]:ctas/ctas;..."] [--rs-pair 2,0] [--rs-ctas 16,32] [--steps 40]

All-gather -> GEMM variants are given as `nvls,units,pair[,transfer]:C1/C2/...`:
  nvls      1 = the shard goes out through the NVLS multicast view, 0 = unicast peer stores;
  units     pieces each 128-row band is pushed in (arrival granularity);
  pair      0 = one CTA per 128 x 256 tile, 1 / 2 = CTA pairs with 256 x 256 / 256 x 512 tiles;
  transfer  sm (SMs push, default) or ce (copy engines);
  C1/C2     numbers of pushing CTAs, each timed on the same instance.
GEMM -> reduce-scatter variants: NVLS with each `--rs-pair` tile choice and each `--rs-ctas`
number of reducing CTAs, then the unicast kernel.  Every variant is timed over `--steps`
calls after 5 untimed ones (CUDA events, max over ranks, a one-element all-reduce lining the
ranks up first) and checked against fp32 on every 61st row (AG) or row of this rank's block
(RS).  A variant whose kernels record a device error is reported with ms = NaN and the error.
Rank 0 prints one JSON object; with --out it is also written there.
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=16384)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--ag", default="1,4,0:16;1,4,2:16", help="all-gather variants (see the module docstring)")
    ap.add_argument("--rs-pair", default="2,0", help="reduce-scatter tile choices (NVLS)")
    ap.add_argument("--rs-ctas", default="16,32", help="reduce-scatter: reducing CTAs (NVLS)")
    ap.add_argument("--rs-join", action="store_true",
                    help="also time the NVLS reduce-scatter on single-CTA tiles with the join option "
                         "(CTAs out of GEMM tiles join the reduction)")
    ap.add_argument("--no-rs", action="store_true")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    lr = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(lr)
    dev = torch.device("cuda", lr)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from opengda_b200 import native
    from opengda_b200.baselines.gemm_nccl import NcclDistGemm
    from opengda_b200.models.dist_gemm import DistGemm, make_operands
    from opengda_b200.parallel import Runtime
    from opengda_b200.utils.clocks import ClockSampler

    rt = Runtime()
    M = N = K = args.size
    flops = 2.0 * M * N * K
    out = {"n_gpus": world, "size": M, "steps": args.steps, "variants": {}}
    tiny = torch.zeros(1, device=dev)

    def mx(v):
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()

    def timeit(fn):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler([lr]) as cs:
            dist.all_reduce(tiny)
            s.record()
            for _ in range(args.steps):
                fn()
            e.record()
            torch.cuda.synchronize()
        ms = mx(s.elapsed_time(e) / args.steps)
        rec = native().read_errors(True)
        if mx(float(rec["code"] != 0)) > 0:
            return float("nan"), {"error": f"{rec['status']} at {rec['where']}" if rec["code"] else "on a peer"}
        return ms, cs.summary()

    def record(key, ms, clk, rel=None):
        v = {"ms": ms, "tflops": flops / ms / 1e9 if ms == ms else None}
        if isinstance(clk, dict) and "error" in clk:
            v.update(clk)
        elif isinstance(clk, dict):
            v.update({"sm_mhz": clk.get("sm_mhz"), "reasons": clk.get("reasons")})
        if rel is not None:
            v["rel_err"] = rel
        out["variants"][key] = v

    A, B, (Af, Bf) = make_operands(M, N, K, "ag", world, rank, seed=2, device=dev)
    rows = torch.arange(0, M, 61, device=dev)
    ref = Af[rows].float() @ B.float().t()
    del Af, Bf
    torch.cuda.empty_cache()
    for spec in [x for x in args.ag.split(";") if x]:
        head, ctas = spec.split(":")
        f = head.split(",")
        nv, q, pr = int(f[0]), int(f[1]), int(f[2])
        tr = f[3] if len(f) > 3 else "sm"
        m = DistGemm(M, N, K, "ag", rt=rt, device=dev, nvls=bool(nv), transfer=tr)
        m.pair, m.units_per_band = pr, q
        m.a_slot(0).copy_(A)
        m.a_slot(1).copy_(A)
        for c in (int(x) for x in ctas.split("/")):
            m.comm_ctas = c
            ms, clk = timeit(lambda: m(m.a_slot(), B))
            C = m(m.a_slot(), B)
            torch.cuda.synchronize()
            rel = mx(((C[rows].float() - ref).norm() / ref.norm()).item())
            record(f"ag nvls={nv} units={q} pair={pr} transfer={tr} ctas={c}", ms, clk, rel)
        del m
        torch.cuda.synchronize()
        dist.barrier()
        torch.cuda.empty_cache()
    nm = NcclDistGemm(M, N, K, "ag", device=dev)
    ms, clk = timeit(lambda: nm(A, B))
    record("ag nccl all_gather_into_tensor + cublas", ms, clk)
    del nm, A, B
    torch.cuda.empty_cache()
    if not args.no_rs:
        A, B, (Af, Bf) = make_operands(M, N, K, "rs", world, rank, seed=2, device=dev)
        Mr = M // world
        rrows = torch.arange(0, Mr, 61, device=dev)
        rref = Af[rank * Mr + rrows].float() @ Bf.float().t()
        del Af, Bf
        torch.cuda.empty_cache()
        variants = [(1, int(p), False) for p in args.rs_pair.split(",")] + [(0, 0, False)]
        if args.rs_join:
            variants.append((1, 0, True))
        for nv, pr, join in variants:
            m = DistGemm(M, N, K, "rs", rt=rt, device=dev, nvls=bool(nv))
            m.pair = pr
            m.rs_join = join
            for c in ([int(x) for x in args.rs_ctas.split(",")] if nv else [0]):
                m.rs_reduce_ctas = c
                ms, clk = timeit(lambda: m(A, B))
                C = m(A, B)
                torch.cuda.synchronize()
                rel = mx(((C[rrows].float() - rref).norm() / rref.norm()).item())
                record(f"rs nvls={nv} pair={pr} join={int(join)} reduce_ctas={c}", ms, clk, rel)
            del m
            torch.cuda.synchronize()
            dist.barrier()
            torch.cuda.empty_cache()
        nm = NcclDistGemm(M, N, K, "rs", device=dev)
        ms, clk = timeit(lambda: nm(A, B))
        record("rs cublas + nccl reduce_scatter_tensor", ms, clk)
        del nm
    if rank == 0:
        js = json.dumps(out)
        print(js)
        if args.out:
            with open(args.out, "w") as fh:
                fh.write(js + "\n")
    torch.cuda.synchronize()
    rt.finalize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
