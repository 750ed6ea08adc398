"""Per-phase timing of a barrier / put / barrier / compute / verify / barrier loop on every
GPU (the reference's legacy/ofi/prototype/barrier_put_compute_verify.cpp:465-760, which
stamps each phase with clock64 and reports mean / std / min / max / p50 / p90 / p99 and
jitter per phase).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/phase_bench.py \
        [--floats 262144] [--iters 1000] [--nvls] [--csv out.csv] [--out out.json]

Each rank runs one block: barrier, put `--floats` fp32 values into its right neighbour,
barrier, SAXPY on its own data, verify what its left neighbour put, barrier -- all in one
kernel, with a %globaltimer stamp after every phase.  Stats per phase are taken on each
rank and the JSON reports, for every statistic, the maximum over ranks.  `bad_values`
counts verification failures (must be 0).  Runs on 1 GPU too (the neighbour is itself).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

PHASES = ["barrier1", "put_barrier2", "compute", "verify", "barrier3", "iteration"]


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--floats", type=int, default=1 << 18)
    ap.add_argument("--iters", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--nvls", action="store_true")
    ap.add_argument("--csv", default=None)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(lr)
    from opengda_b200 import native
    from opengda_b200.parallel import Barrier, Bootstrap, Runtime
    from opengda_b200.utils.timing import summarize

    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", lr))
        rt = Runtime()
    else:
        rt = Runtime(Bootstrap.create(0, 1, "127.0.0.1:0"))
    right, left = (rank + 1) % world, (rank - 1) % world
    n = args.floats
    recv = rt.alloc_tensor((n,), torch.float32)
    x = torch.zeros(n, dtype=torch.float32, device="cuda")
    y = torch.ones(n, dtype=torch.float32, device="cuda")
    bar = Barrier(rt, nvls=args.nvls)
    N = native()

    def run(iters):
        stamps = torch.zeros(iters * 6, dtype=torch.int64, device="cuda")
        bad = torch.zeros(1, dtype=torch.int64, device="cuda")
        bar._b.advance(3 * iters)  # the kernel advances the device epoch itself
        N.k_phase_loop(bar.device_ctx(), x.data_ptr(), y.data_ptr(), recv.ptr(), recv.ptr(right), n, iters, 2.0,
                       rank, left, stamps.data_ptr(), bad.data_ptr())
        torch.cuda.synchronize()
        rt.check_device_errors()
        return stamps.view(iters, 6).cpu(), int(bad.item())

    run(args.warmup)
    rt.barrier()
    st, bad = run(args.iters)
    d = (st[:, 1:] - st[:, :-1]).double() / 1e3  # us per phase
    per = {PHASES[k]: d[:, k].tolist() for k in range(5)}
    per["iteration"] = ((st[:, 5] - st[:, 0]).double() / 1e3).tolist()
    mine = {p: summarize(v) for p, v in per.items()}
    for p in mine:
        mine[p]["jitter_p99_minus_p50"] = mine[p]["p99"] - mine[p]["p50"]
    allr = rt.boot.allgather_obj({"stats": mine, "bad": bad})
    if args.csv:
        with open(f"{args.csv}.r{rank}" if world > 1 else args.csv, "w") as f:
            f.write("iter," + ",".join(PHASES) + "\n")
            for i in range(args.iters):
                f.write(f"{i}," + ",".join(f"{per[p][i]:.3f}" for p in PHASES) + "\n")
    if rank == 0:
        out = {"n_gpus": world, "floats": n, "bytes_per_put": 4 * n, "iters": args.iters, "nvls_barrier": bar.uses_nvls,
               "bad_values": sum(r["bad"] for r in allr), "unit": "us", "max_over_ranks": {}}
        for p in PHASES:
            out["max_over_ranks"][p] = {k: round(max(r["stats"][p][k] for r in allr), 3) for k in mine[p]}
        print(json.dumps(out))
        if args.out:
            with open(args.out, "w") as f:
                json.dump(out, f, indent=1)
    rt.barrier()
    rt.finalize()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
