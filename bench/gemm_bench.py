"""Single-GPU GEMM benchmark: the tcgen05 GEMM's tile variants against cuBLAS
(torch.matmul) on a square bf16 problem, C = A . B^T, f32 accumulation.

    python bench/gemm_bench.py [--size 16384] [--rounds 3] [--iters 30] [--tiles 256,512,1024]
                               [--pair-opts h1p0,h0p4]

Under the 1 kW power cap the SM clock depends on what ran just before, so the variants
are timed round-robin (cuBLAS, then each tile, then again) and each keeps the median
over rounds.  Every timing is CUDA events around `--iters` back-to-back launches after 3
warm-up launches (inputs 512 MiB each at 16384, larger than L2), with the SM clock and
power sampled by nvidia-smi during it.  `tflops_per_ghz` divides by the median SM clock,
which separates how well a kernel keeps the tensor cores busy from how fast the power
cap lets it clock.  Tiles: 128 / 256 = one CTA per 128 x bn tile; 512 = CTA pairs,
256 x 256; 1024 = CTA pairs, 256 x 512.  `--pair-opts` adds 256 x 512 variants with the
pair kernel's options: `h<l2 hint>p<prefetch distance>[s<tma store>]` (`ops.gemm.set_tuning`'s
pair_l2_hint, pair_prefetch and pair_tma_store).  `--fp32` times the fp32 GEMM instead:
cuBLAS SGEMM (tf32 off) against `ops.gemm.gemm_fp32` (three tf32 products on the tensor
cores).  Prints one JSON object.
"""
from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import torch  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=16384)
    ap.add_argument("--rounds", type=int, default=3)
    ap.add_argument("--iters", type=int, default=30)
    ap.add_argument("--tiles", default="256,512,1024")
    ap.add_argument("--pair-group", type=int, default=0, help="raster group of the pair kernels (0 = default)")
    ap.add_argument("--pair-opts", default="", help="extra 256x512 variants: comma list of h<l2 hint>p<prefetch>")
    ap.add_argument("--fp32", action="store_true",
                    help="fp32 GEMM instead: cuBLAS SGEMM (tf32 off) against gemm_fp32 (three tf32 products)")
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    from opengda_b200 import native
    from opengda_b200.ops.gemm import check_errors, set_tuning, tuning
    from opengda_b200.utils.clocks import ClockSampler

    if args.pair_group:
        t = tuning()
        set_tuning(**dict(t, pair_group_m=args.pair_group))
    S = args.size
    g = torch.Generator(device="cuda").manual_seed(0)
    dt = torch.float32 if args.fp32 else torch.bfloat16
    A = torch.randn(S, S, device="cuda", generator=g).to(dt)
    B = torch.randn(S, S, device="cuda", generator=g).to(dt)
    C = torch.empty(S, S, device="cuda", dtype=dt)
    torch.backends.cuda.matmul.allow_tf32 = False  # the cuBLAS arm is a true fp32 SGEMM
    ref = torch.matmul(A, B.t()).float()
    flop = 2.0 * S ** 3
    base = tuning()
    variants = {"cublas": lambda: torch.matmul(A, B.t(), out=C)}
    setups = {}
    if args.fp32:
        from opengda_b200.ops.gemm import gemm_fp32
        variants["tc_fp32x3"] = lambda: gemm_fp32(A, B, out=C)
    for bn in ([] if args.fp32 else (int(x) for x in args.tiles.split(","))):
        variants[f"tile{bn}"] = (lambda bn=bn: native().gemm(A, B, out=C, bn=bn))
    for spec in (x for x in args.pair_opts.split(",") if x and not args.fp32):
        m = re.fullmatch(r"h(\d)p(\d+)(?:s(\d))?", spec)
        if not m:
            raise SystemExit(f"--pair-opts: {spec!r} is not h<hint>p<prefetch>[s<tma store>]")
        variants[f"tile1024_{spec}"] = lambda: native().gemm(A, B, out=C, bn=1024)
        setups[f"tile1024_{spec}"] = dict(base, pair_l2_hint=int(m[1]), pair_prefetch=int(m[2]),
                                          pair_tma_store=int(m[3] or base["pair_tma_store"]))

    def setup(name):
        set_tuning(**setups.get(name, base))

    out = {"size": S, "rounds": args.rounds, "iters": args.iters, "pair_group_m": tuning()["pair_group_m"],
           "variants": {}}
    for name, fn in variants.items():
        setup(name)
        fn()
        torch.cuda.synchronize()
        out["variants"][name] = {"rel_err_vs_cublas": float(((C.float() - ref).norm() / ref.norm()).item())}
    check_errors()
    samples = {k: [] for k in variants}
    for _ in range(args.rounds):
        for name, fn in variants.items():
            setup(name)
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with ClockSampler(period_ms=20) as cs:
                s.record()
                for _ in range(args.iters):
                    fn()
                e.record()
                torch.cuda.synchronize()
            ms = s.elapsed_time(e) / args.iters
            c = cs.summary()
            samples[name].append((flop / ms / 1e9, c.get("sm_mhz"), c.get("power_w"), c.get("reasons", [])))
    check_errors()
    set_tuning(**base)
    for name, v in samples.items():
        tf = statistics.median(x[0] for x in v)
        mhz = [x[1] for x in v if x[1]]
        w = [x[2] for x in v if x[2]]
        rec = out["variants"][name]
        rec.update({"tflops": round(tf, 1), "tflops_max": round(max(x[0] for x in v), 1),
                    "sm_mhz": statistics.median(mhz) if mhz else None,
                    "power_w": statistics.median(w) if w else None,
                    "reasons": sorted({r for x in v for r in x[3]})})
        if mhz:
            rec["tflops_per_ghz"] = round(tf / (statistics.median(mhz) / 1000.0), 1)
    print(json.dumps(out))
    if args.out:
        with open(args.out, "w") as f:
            f.write(json.dumps(out) + "\n")


if __name__ == "__main__":
    main()
