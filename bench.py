"""Headline benchmark: distributed GEMM, all-gather -> GEMM,
bf16 in / f32 accumulate, M = N = K = 16384, A row-sharded, B column-sharded,
on 1..8 GPUs of one node (strong scaling: the problem is fixed, the GPUs grow).

    python bench.py --gpus N --steps K --warmup W            # this framework
    python bench.py --impl reference ...                      # the reference arm
    torchrun --nproc-per-node N ... bench.py --gpus N ...     # N > 1

Rank 0 prints one JSON line.  ``value`` is whole-job TFLOP/s = 2*M*N*K / step time,
where the step time is the max over ranks of device time measured with CUDA events.
``e2e`` is the same metric through the public API (``DistGemm.__call__``) including
the host->device copy of each step's A shard from pinned memory and a device->host read
of the step's result checksum.  ``nccl_arm`` is the NCCL + cuBLAS arm in the same process:
the same device-timed steps and the same end-to-end loop (``nccl_arm.e2e``).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "dist-GEMM TFLOPS (all-gather->GEMM, bf16 in / fp32 accumulate, M=N=K=16384)"
HEADLINE_METRIC_FAMILY = "put GB/s & latency vs size; barrier µs; dist-GEMM TFLOPS; MoE dispatch+combine µs @1/2/4/8"


def reference_unavailable(args) -> None:
    print(json.dumps({
        "impl": "reference",
        "unavailable": ("the reference (lwshanbd/OpenGDA, GICC) is a CMake C++/CUDA project with no setup.py or "
                        "pyproject.toml (pip install fails: 'not installable'), and it needs libibverbs/mlx5 DevX "
                        "with an InfiniBand HCA or HPE Slingshot libfabric + ROCm, plus MPI/PMI2 -- none exist on "
                        "this box; it publishes no numbers"),
        "metric": METRIC, "n_gpus": args.gpus,
    }))


def check_numerics(model, A, B, Afull, Bfull, mode, world, rank) -> float:
    """One call, then a 256-row block of this rank's output against fp32.  AG mode with
    several ranks checks rows of the NEXT rank's shard (data that crossed NVLink); RS mode
    checks this rank's rows (every rank's partial is in them).  Max over ranks."""
    import torch
    import torch.distributed as dist

    C = model(A, B)
    torch.cuda.synchronize()
    if mode == "ag":
        Ms, Ns = Afull.shape[0] // world, Bfull.shape[0] // world
        r0 = ((rank + 1) % world) * Ms + (Ms // 2 if world > 1 else 0)
        rows = slice(r0, r0 + 256)
        ref = Afull[rows].float() @ Bfull[rank * Ns:(rank + 1) * Ns].float().t()
        got = C[rows].float()
    else:
        Mr = Afull.shape[0] // world
        ref = Afull[rank * Mr:rank * Mr + 256].float() @ Bfull.float().t()
        got = C[0:256].float()
    rel = torch.tensor([((got - ref).norm() / ref.norm()).item()], device=A.device)
    if world > 1:
        dist.all_reduce(rel, op=dist.ReduceOp.MAX)
    return float(rel.item())


def timed_run(step, steps, warmup, world, local_rank):
    """W untimed steps, then K steps between a barrier + synchronize on both sides, timed
    with CUDA events on the launching stream (one event per step boundary, which adds no
    synchronisation); with several ranks a one-element all-reduce on the stream right
    before the first event lines the ranks' starts up on the device.  Returns (ms per step, max over ranks; per-step ms summary of the
    slowest rank; clock record during the timed steps, all ranks)."""
    import torch
    import torch.distributed as dist

    from opengda_b200.utils.clocks import ClockSampler
    from opengda_b200.utils.timing import max_over_ranks

    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    tiny = torch.zeros(1, device=torch.device("cuda", local_rank))
    with ClockSampler([local_rank]) as cs:
        if world > 1:
            # a device-side barrier (one-element all-reduce on this stream) right before the
            # first timed step: every rank's clock starts when all ranks are ready, so a rank
            # whose host left the barrier late does not stretch the others' first step
            dist.all_reduce(tiny)
        ev[0].record()
        for i in range(steps):
            step()
            ev[i + 1].record()
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    per = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(steps))
    total = ev[0].elapsed_time(ev[steps]) / steps
    ms = max_over_ranks(total)
    summ = {"min": round(per[0], 4), "p50": round(per[len(per) // 2], 4), "max": round(per[-1], 4)}
    clocks = cs.summary()
    if world > 1:
        allc = [None] * world
        dist.all_gather_object(allc, (clocks, total, summ))
        slowest = max(range(world), key=lambda q: allc[q][1])
        summ = dict(allc[slowest][2], rank=slowest)
        cl = [c[0] for c in allc]
        sm = [c["sm_mhz"] for c in cl if c.get("sm_mhz")]
        reasons = sorted({r for c in cl for r in c.get("reasons", [])})
        clocks = {"sm_mhz": min(sm) if sm else None, "sm_max_mhz": cl[0].get("sm_max_mhz"), "reasons": reasons,
                  "per_rank_sm_mhz": sm}
    return ms, summ, clocks


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "nccl"],
                    help="nccl: the NCCL + cuBLAS comparison arm (same shapes, library kernels only)")
    ap.add_argument("--mode", default="ag", choices=["ag", "rs"])
    ap.add_argument("--size", type=int, default=16384)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--unfused", action="store_true", help="decomposed path: copy kernels + GEMM (A/B only)")
    ap.add_argument("--no-nccl-arm", action="store_true", help="skip the same-run NCCL(+cuBLAS) comparison arm")
    ap.add_argument("--no-tune", action="store_true", help="AG, several GPUs: keep the default number of pushing CTAs")
    ap.add_argument("--transfer", default="sm", choices=["sm", "ce"],
                    help="fused AG: SM pushes (NVLS multicast or unicast) or copy engines (A/B option)")
    args = ap.parse_args()
    if args.impl == "reference":
        reference_unavailable(args)
        return 0
    if args.warmup < 3:
        args.warmup = 3

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    rt = None
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
        from opengda_b200.parallel import Runtime

        rt = Runtime()

    from opengda_b200.models.dist_gemm import DistGemm, make_operands

    M = N = K = args.size
    if args.impl == "nccl":
        from opengda_b200.baselines.gemm_nccl import NcclDistGemm

        model = NcclDistGemm(M, N, K, args.mode, device=dev)
    else:
        model = DistGemm(M, N, K, args.mode, rt=rt, device=dev, fused=not args.unfused,
                         transfer=args.transfer if args.mode == "ag" else "sm")
    A, B, (Afull, Bfull) = make_operands(M, N, K, args.mode, world, rank, seed=2, device=dev)
    rel = check_numerics(model, A, B, Afull, Bfull, args.mode, world, rank)
    del Afull, Bfull
    torch.cuda.empty_cache()
    zero_copy = world > 1 and args.mode == "ag" and args.impl == "ours"
    tuned = {}
    if zero_copy and not args.unfused and args.transfer == "sm" and not args.no_tune:
        # pick the number of pushing CTAs on this node (before warm-up, outside the timed steps)
        tuned = model.tune(A, B)
    if zero_copy:  # the shard lives in the symmetric landing buffers (both parities)
        model.a_slot(0).copy_(A)
        model.a_slot(1).copy_(A)

    def step():
        model(model.a_slot() if zero_copy else A, B)

    ms, step_ms, clocks = timed_run(step, args.steps, args.warmup, world, local_rank)
    if rt is not None:
        rt.check_device_errors()
    flops = 2.0 * M * N * K
    value = flops / (ms * 1e-3) / 1e12

    # ---- end to end through the public API: pinned H2D of A, forward, D2H of a checksum
    e2e_steps = args.e2e_steps or max(3, min(args.steps, 10))
    from opengda_b200.utils.feeder import HostFeeder

    A_host = A.cpu().pin_memory()
    h2d = A_host.numel() * A_host.element_size()

    from opengda_b200.utils.timing import max_over_ranks

    def e2e_ms_of(fn):
        # the fused AG model takes its input zero-copy: the host copy lands in its A slots
        slots = fn.input_slots() if hasattr(fn, "input_slots") else None
        feeder = HostFeeder(A.shape, A.dtype, dev, bufs=slots)

        def e2e_run(steps):
            # step i's pinned H2D copy is issued during step i-1 (double-buffered side
            # stream); every step ends with a 4-byte device->host read of its result checksum
            feeder.submit(A_host)
            for i in range(steps):
                if i + 1 < steps:
                    feeder.submit(A_host)
                a_dev = feeder.next()
                out = fn(a_dev, B)
                feeder.release()
                out.sum(dtype=torch.float32).item()  # 4-byte device->host read of a checksum

        e2e_run(2)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        es, ee = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        es.record()
        e2e_run(e2e_steps)
        ee.record()
        torch.cuda.synchronize()
        return max_over_ranks(es.elapsed_time(ee) / e2e_steps)

    e2e_ms = e2e_ms_of(model)

    # ---- the NCCL (+cuBLAS) arm, same process, same shapes, steps, warm-up and clock record
    arm = None
    if args.impl == "ours" and not args.no_nccl_arm:
        from opengda_b200.baselines.gemm_nccl import NcclDistGemm

        try:
            base = NcclDistGemm(M, N, K, args.mode, device=dev)
            base_rel = check_numerics(base, A, B,
                                      *make_operands(M, N, K, args.mode, world, rank, seed=2, device=dev)[2],
                                      args.mode, world, rank)
            torch.cuda.empty_cache()
            b_ms, b_step_ms, b_clocks = timed_run(lambda: base(A, B), args.steps, args.warmup, world, local_rank)
            arm = {"impl": "nccl+cublas", "what": ("all_gather_into_tensor + torch.matmul" if args.mode == "ag"
                                                   else "torch.matmul + reduce_scatter_tensor") if world > 1
                   else "torch.matmul (cuBLAS)",
                   "value": round(flops / (b_ms * 1e-3) / 1e12, 2), "ms_per_step": round(b_ms, 4),
                   "step_ms": b_step_ms, "clocks": b_clocks, "numerics_rel_err_vs_fp32": round(base_rel, 6)}
            # the same end-to-end loop (pinned H2D of A, D2H of a checksum) through the arm
            b_e2e_ms = e2e_ms_of(base)
            arm["e2e"] = {"value": round(flops / (b_e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                          "ms_per_step": round(b_e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                          "api": "opengda_b200.baselines.gemm_nccl.NcclDistGemm.__call__"}
            del base
        except (RuntimeError, torch.cuda.OutOfMemoryError) as exc:  # the comparison arm must not cost our line
            arm = {"impl": "nccl+cublas", "error": f"{type(exc).__name__}: {exc}"[:300]}
        torch.cuda.empty_cache()
    del A_host
    if rank == 0:
        out = {
            "metric": METRIC,
            "baseline_metric": HEADLINE_METRIC_FAMILY,
            "value": round(value, 2),
            "unit": "TFLOP/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms, 4),
            "higher_is_better": True,
            "scaling": "strong",
            # same-run NCCL(+cuBLAS) arm: its time / ours (> 1: this framework is faster)
            "vs_baseline": round(value / arm["value"], 4) if arm and "value" in arm else None,
            "vs_baseline_of": "same-run NCCL+cuBLAS arm (nccl_arm)" if arm and "value" in arm else None,
            "dtype": "bf16",
            "data": "synthetic: A, B ~ N(0, 1/sqrt(K)) from seed 2, random-init (no dataset)",
            "config": {
                "model": f"dist_gemm_{args.mode}", "M": M, "N": N, "K": K,
                "global_batch": M, "seq_len": K,
                "parallelism": (f"tp{world}-" + ("allgather-gemm" if args.mode == "ag" else "gemm-reducescatter")),
                "transfer": ("none" if world == 1 else "nccl" if args.impl == "nccl" else
                             "unfused-copy-kernels" if args.unfused else
                             model.transfer + ("-nvls" if model.nvls else "")),
                "l2": "inputs exceed L2 (A_full 512 MiB > 126 MB), no flush",
                "numerics_rel_err_vs_fp32": round(rel, 6),
                "numerics_rows": ("256 rows of the next rank's shard (gathered data), max over ranks"
                                  if args.mode == "ag" and world > 1 else "256 rows of each rank's output, max over ranks"),
                "step_ms": step_ms,
                "tiles": ("pair256x512" if getattr(model, "pair", 0) == 2 else "pair256x256"
                          if getattr(model, "pair", 0) == 1 else "cta128x256") if world > 1 else "by shape",
                "comm_ctas": getattr(model, "comm_ctas", None) if world > 1 else None,
                "comm_ctas_tuning_ms": {str(k): round(v, 4) for k, v in tuned.items()} or None,
            },
            "impl": args.impl,
            "clocks": clocks,
            "e2e": {"value": round(flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s", "ms_per_step": round(e2e_ms, 4),
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4,
                    "api": ("opengda_b200.baselines.gemm_nccl.NcclDistGemm.__call__" if args.impl == "nccl"
                            else "opengda_b200.models.dist_gemm.DistGemm.__call__")},
            "gpu_launches": model.launches_per_step * args.steps,
            "nccl_arm": arm,
        }
        print(json.dumps(out))
    if world > 1:
        del model
        torch.cuda.synchronize()
        rt.finalize()
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
