"""Active-message ping-pong latency between ranks 0 and 1 (the reference's
examples/ofi/am_pingpong.cpp: request/reply with a 64-byte request and 8-byte reply, and
request/request with 64 bytes both ways; 10 round trips per kernel, 100 timed batches after
10 warm-up batches).

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 bench/am_pingpong.py [--batches 100]

Each batch is one kernel per rank running `--rtts` device-driven round trips; the
initiator's %globaltimer brackets the batch.  Prints one JSON object (rank 0).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batches", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--rtts", type=int, default=10)
    ap.add_argument("--out", default=None)
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    rank, world, lr = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    if world < 2:
        raise SystemExit("am_pingpong needs 2 ranks")
    torch.cuda.set_device(lr)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", lr))
    from opengda_b200.parallel import Runtime
    from opengda_b200.parallel.am import Am
    from opengda_b200.utils.timing import summarize

    rt = Runtime()
    am = Am(rt, nslots=128, max_payload=0)
    ns = torch.zeros(1, dtype=torch.int64, device="cuda")
    res = {"n_gpus": world, "rtts_per_batch": args.rtts, "batches": args.batches}
    for mode in ("reqrep", "reqreq"):
        samples = []
        for b in range(args.warmup + args.batches):
            rt.barrier()
            if rank < 2:
                am.pingpong(1 - rank, args.rtts, mode, rank == 0, ns.data_ptr())
            torch.cuda.synchronize()
            if b >= args.warmup and rank == 0:
                samples.append(ns.item() / 1e3 / args.rtts)  # us per round trip
        rt.check_device_errors()
        if rank == 0:
            s = summarize(samples)
            res[mode] = {"rtt_us": {k: round(v, 3) for k, v in s.items()},
                         "half_rtt_us_p50": round(s["p50"] / 2, 3)}
    if rank == 0:
        print(json.dumps(res))
        if args.out:
            with open(args.out, "w") as f:
                json.dump(res, f, indent=1)
    rt.barrier()
    del am
    torch.cuda.synchronize()
    rt.finalize()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
