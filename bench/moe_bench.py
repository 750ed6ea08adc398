"""MoE expert-parallel layer benchmark: 4096 tokens per GPU, hidden
7168, 256 experts (E/n per GPU), top-8 softmax routing (router logits N(0,1), seed 4),
SwiGLU experts with intermediate 2048, weights N(0, 0.02).

    python bench/moe_bench.py [--tokens 4096 ...]
    torchrun --nproc-per-node N bench/moe_bench.py

Reports the layer time (device, max over ranks) of this framework's fused path and of the
NCCL all_to_all + cuBLAS per-expert arm, plus a numerics check of ours against the arm.
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
    ap.add_argument("--tokens", type=int, default=4096)
    ap.add_argument("--hidden", type=int, default=7168)
    ap.add_argument("--experts", type=int, default=256)
    ap.add_argument("--topk", type=int, default=8)
    ap.add_argument("--inter", type=int, default=2048)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--no-baseline", action="store_true")
    ap.add_argument("--out", default=None)
    ap.add_argument("--dispatch-ctas", type=int, default=None, help="CTAs that dispatch (0 = all; default: the layer's)")
    ap.add_argument("--comm-only", action="store_true",
                    help="time the dispatch + combine round trip alone (identity experts), vs NCCL all_to_all")
    ap.add_argument("--combine-ctas", type=int, default=None,
                    help="CTAs that push the combine (0 = all, from the epilogue; default: the layer's)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    rt = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
        from opengda_b200.parallel import Runtime
        rt = Runtime()
    rank = rt.rank if rt else 0
    from opengda_b200.models.moe import MoELayer, make_inputs
    from opengda_b200.utils.timing import max_over_ranks

    from opengda_b200.utils.clocks import BenchClocks

    clk = BenchClocks(local)
    layer = MoELayer(args.tokens, args.hidden, args.experts, args.topk, args.inter, rt=rt)
    if args.dispatch_ctas is not None:
        layer.dispatch_ctas = args.dispatch_ctas
    if args.combine_ctas is not None:
        layer.combine_ctas = args.combine_ctas
    x, logits = make_inputs(args.tokens, args.hidden, args.experts, rank, seed=4)

    def timeit(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(steps):
            fn()
        e.record()
        torch.cuda.synchronize()
        return max_over_ranks(s.elapsed_time(e) / steps)

    if args.comm_only:
        ms = timeit(lambda: layer.dispatch_combine(x, logits), args.steps, args.warmup)
        if rt:
            rt.check_device_errors()
        res = {"metric": "moe_dispatch_combine_us", "impl": "ours-fused", "n_gpus": world,
               "tokens_per_gpu": args.tokens, "hidden": args.hidden, "experts": args.experts, "topk": args.topk,
               "us": ms * 1e3}
        layer.dispatch_combine(x, logits, stage_times=True)
        res["stage_us_rank0"] = {k: round(v * 1e3, 1) for k, v in layer.last_stage_ms.items()}
        y = layer.dispatch_combine(x, logits).float()
        prob = torch.softmax(logits, dim=-1)
        wsum = torch.topk(prob, args.topk, dim=-1).values.sum(-1, keepdim=True)
        ref = x.float() * wsum
        res["rel_err_vs_identity_reference"] = float(((y - ref).norm() / ref.norm()).item())
        if not args.no_baseline:
            from opengda_b200.baselines.moe_nccl import NcclMoE
            base = NcclMoE(layer)
            ms_b = timeit(lambda: base.dispatch_combine(x, logits), max(2, args.steps // 2), 1)
            res["nccl_torch"] = {"us": ms_b * 1e3}
        res["clocks"] = clk.finish()
        if rank == 0:
            print(json.dumps(res))
            if args.out:
                with open(args.out, "w") as f:
                    f.write(json.dumps(res) + "\n")
        if world > 1:
            del layer
            torch.cuda.synchronize()
            rt.finalize()
            dist.barrier()
            dist.destroy_process_group()
        return
    ms = timeit(lambda: layer(x, logits), args.steps, args.warmup)
    if rt:
        rt.check_device_errors()
    tflops = layer.flops() * world / (ms * 1e-3) / 1e12
    res = {"metric": "moe_layer_us", "impl": "ours-fused", "n_gpus": world, "tokens_per_gpu": args.tokens,
           "hidden": args.hidden, "experts": args.experts, "topk": args.topk, "inter": args.inter,
           "layer_us": ms * 1e3, "tflops_total": tflops}
    # per-stage breakdown of one extra call (device events between the kernels)
    layer(x, logits, stage_times=True)
    res["stage_us_rank0"] = {k: round(v * 1e3, 1) for k, v in layer.last_stage_ms.items()}
    if not args.no_baseline:
        from opengda_b200.baselines.moe_nccl import NcclMoE
        base = NcclMoE(layer)
        ours = layer(x, logits).float().clone()
        ref = base(x, logits).float()
        res["rel_err_vs_baseline"] = float(((ours - ref).norm() / ref.norm()).item())
        ms_b = timeit(lambda: base(x, logits), max(2, args.steps // 2), 1)
        res["nccl_torch"] = {"layer_us": ms_b * 1e3, "tflops_total": layer.flops() * world / (ms_b * 1e-3) / 1e12}
    res["clocks"] = clk.finish()
    if rank == 0:
        js = json.dumps(res)
        print(js)
        if args.out:
            with open(args.out, "w") as f:
                f.write(js + "\n")
    if world > 1:
        del layer
        torch.cuda.synchronize()
        rt.finalize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
