"""Host-queued multi-stream put benchmark (the reference's examples/ofi/benchmark.cpp:
32 concurrent put_no_db "streams" per size, 1 B ... 16 MiB, 20 iterations of which the best
10 are averaged, with per-iteration pattern verification).

    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench/put_streams.py [--streams 32]
    python bench/put_streams.py                      # one GPU: puts into its own buffer

Per size and iteration, every rank queues `--streams` puts of that size into its right
neighbour (Runtime.put_no_db: host-side descriptors, no transfer yet), then one device
flush kernel executes all of them; the host waits for every token.  Device time of the
flush kernel is recorded with CUDA events (max over ranks); the receiver then checks the
seeded pattern of every stream's landing area.  Prints one JSON object.
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
    ap.add_argument("--streams", type=int, default=32)
    ap.add_argument("--max-log2", type=int, default=24)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--best", type=int, default=10)
    ap.add_argument("--out", default=None)
    ap.add_argument("--resume", default=None, help="JSON-lines store: sizes finished by an earlier run are skipped")
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    lr = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(lr)
    from opengda_b200 import native
    from opengda_b200.parallel import Bootstrap, Runtime
    from opengda_b200.utils.timing import max_over_ranks

    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", lr))
        rt = Runtime()
    else:
        rt = Runtime(Bootstrap.create(0, 1, "127.0.0.1:0"))
    N = native()
    S = args.streams
    maxb = 1 << args.max_log2
    src = rt.alloc_tensor((S * maxb,), torch.uint8)
    dst = rt.alloc_tensor((S * maxb,), torch.uint8)
    right, left = (rank + 1) % world, (rank - 1) % world
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    from opengda_b200.utils.results import ResultStore
    store = ResultStore(args.resume) if args.resume else None  # read by every rank before any write
    rows, total_bad = [], 0
    for lg in range(0, args.max_log2 + 1, 2):
        size = 1 << lg
        key = f"put_streams:n={world}:streams={S}:bytes={size}:iters={args.iters}"
        if store is not None and store.done(key):
            rows.append(store.get(key))
            continue
        times = []
        for it in range(args.iters):
            seed = 1000 * lg + it + 7 * rank
            N.k_fill_pattern(src.ptr(), S * maxb, seed)
            torch.cuda.synchronize()
            rt.barrier()
            rt.reset()
            toks = [rt.put_no_db(src.index, right, dst.index, size, src_off=s * maxb, dst_off=s * maxb)
                    for s in range(S)]
            ctx = rt.prepare_trigger(toks[-1])
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            N.k_flush(ctx, status.data_ptr())
            e1.record()
            for t in toks:
                rt.wait(t)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
            rt.barrier()
            # verify: stream s landed src bytes [s*maxb, s*maxb + size) of the left neighbour
            bad.zero_()
            for s in range(S):
                N.k_check_pattern_range(dst.ptr() + s * maxb, size, 1000 * lg + it + 7 * left, s * maxb,
                                        bad.data_ptr())
            torch.cuda.synchronize()
            total_bad += int(bad.item())
        best = sorted(times)[:args.best]
        ms = max_over_ranks(sum(best) / len(best))
        rows.append({"bytes": size, "streams": S, "us": round(ms * 1e3, 3),
                     "GBps": round(S * size / (ms * 1e-3) / 1e9, 3)})
        if store is not None and rank == 0:
            store.add(key, rows[-1])
    assert int(status.item()) == 0, "flush reported an error"
    if rank == 0:
        out = {"n_gpus": world, "iters": args.iters, "best_of": args.best, "bad_bytes": total_bad, "sizes": rows}
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
