"""Single-GPU sweep of the tcgen05 GEMM's tuning knobs against cuBLAS (torch.matmul) on
square bf16 problems: raster group (m-blocks per group) x L2 eviction hints, plus the
CTA-pair kernel.  Each configuration is timed with CUDA events over back-to-back launches
after warm-up (inputs larger than L2 at the default sizes), with the SM clock sampled during
the timed loop so power-capped runs can be compared by time x clock.

    python bench/gemm_sweep.py [--sizes 8192 16384] [--iters 20] [--out sweep.json]
"""
from __future__ import annotations

import argparse
import itertools
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--sizes", type=int, nargs="+", default=[8192, 16384])
    ap.add_argument("--groups", type=int, nargs="+", default=[4, 8, 16, 32])
    ap.add_argument("--hints", type=int, nargs="+", default=[0, 1, 2])
    ap.add_argument("--pair-groups", type=int, nargs="+", default=[4, 8, 16])
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    from opengda_b200 import native
    from opengda_b200.ops.gemm import check_errors, gemm, set_tuning
    from opengda_b200.utils.clocks import ClockSampler

    def timed(fn):
        for _ in range(args.warmup):
            fn()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler() as clk:
            s.record()
            for _ in range(args.iters):
                fn()
            e.record()
            torch.cuda.synchronize()
        return s.elapsed_time(e) / args.iters, clk.summary()

    rows = []
    for S in args.sizes:
        torch.manual_seed(0)
        A = torch.randn(S, S, device="cuda").to(torch.bfloat16)
        B = torch.randn(S, S, device="cuda").to(torch.bfloat16)
        C = torch.empty(S, S, device="cuda", dtype=torch.bfloat16)
        flop = 2.0 * S ** 3
        ref = torch.matmul(A, B.t())
        ms, clk = timed(lambda: torch.matmul(A, B.t(), out=C))
        rows.append({"size": S, "impl": "cublas", "ms": ms, "tflops": flop / ms / 1e9, "clocks": clk})
        for g, h in itertools.product(args.groups, args.hints):
            set_tuning(group_m=g, l2_hint=h)
            ms, clk = timed(lambda: gemm(A, B, out=C))
            err = float(((C.float() - ref.float()).norm() / ref.float().norm()).item())
            rows.append({"size": S, "impl": "tcgen05", "group_m": g, "l2_hint": h, "ms": ms,
                         "tflops": flop / ms / 1e9, "rel_err": err, "clocks": clk})
        for pg in args.pair_groups:
            set_tuning(pair_group_m=pg)
            ms, clk = timed(lambda: native().gemm(A, B, out=C, bn=512))
            rows.append({"size": S, "impl": "tcgen05_pair", "pair_group_m": pg, "ms": ms, "tflops": flop / ms / 1e9,
                         "clocks": clk})
        set_tuning()
        check_errors()
        del A, B, C, ref
        torch.cuda.empty_cache()
    for r in rows:
        print(json.dumps(r))
    if args.out:
        with open(args.out, "w") as f:
            for r in rows:
                f.write(json.dumps(r) + "\n")


if __name__ == "__main__":
    main()
