"""GPU-triggered vs CPU-driven vs NCCL transfers, each behind a SAXPY on the data (the
reference's three-way comparisons legacy/ofi/prototype/gda-comp.cpp, ofi-comp.cpp and
mpi-comp.cpp, which run a SAXPY before the transfer).  Rank 0 sends to rank 1.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 bench/put_compare.py [--iters 50]

* gpu:  one kernel per iteration -- each CTA computes its chunk of y = a*x + y, stores it
        into rank 1's buffer over NVLink and bumps rank 1's arrival counter; rank 1's stream
        waits (bounded) for all CTAs.
* cpu:  SAXPY kernel, then a host-issued copy-engine copy into rank 1 (cudaMemcpyAsync on
        the peer mapping), the host waits for it and meets rank 1 at a host barrier.
* nccl: SAXPY kernel, then torch.distributed send / recv.

Times K iterations with CUDA events on each rank's stream (barrier + synchronize on both
sides), max over ranks; prints one JSON object with microseconds per iteration per size.
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
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--min-log2", type=int, default=12)
    ap.add_argument("--max-log2", type=int, default=26)
    ap.add_argument("--out", default=None)
    ap.add_argument("--resume", default=None, help="JSON-lines store: sizes finished by an earlier run are skipped")
    args = ap.parse_args()

    import torch
    import torch.distributed as dist

    rank, world, lr = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    if world < 2:
        raise SystemExit("put_compare needs 2 ranks")
    torch.cuda.set_device(lr)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", lr))
    from opengda_b200 import native
    from opengda_b200.parallel import Runtime
    from opengda_b200.utils.timing import max_over_ranks

    rt = Runtime()
    N = native()
    maxn = (1 << args.max_log2) // 4
    recv = rt.alloc_tensor((maxn,), torch.float32)
    x = torch.rand(maxn, device="cuda")
    y = torch.rand(maxn, device="cuda")
    cnt_off = rt.signal_alloc(1)
    epoch = 0
    blocks = 2 * torch.cuda.get_device_properties(lr).multi_processor_count
    nccl_buf = torch.empty(maxn, dtype=torch.float32, device="cuda")
    res = {"n_gpus": world, "iters": args.iters, "unit": "us per iteration", "sizes": []}

    def timed(step):
        for _ in range(3):
            step()
        torch.cuda.synchronize()
        rt.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(args.iters):
            step()
        e.record()
        torch.cuda.synchronize()
        rt.barrier()
        return max_over_ranks(s.elapsed_time(e) * 1e3 / args.iters)

    from opengda_b200.utils.results import ResultStore
    store = ResultStore(args.resume) if args.resume else None  # read by every rank before any write
    for lg in range(args.min_log2, args.max_log2 + 1, 2):
        n = (1 << lg) // 4
        key = f"put_compare:n={world}:bytes={4 * n}:iters={args.iters}"
        if store is not None and store.done(key):
            res["sizes"].append(store.get(key))
            continue
        row = {"bytes": 4 * n}

        def gpu_step():
            nonlocal epoch
            epoch += 1
            if rank == 0:
                N.k_saxpy_put(x.data_ptr(), y.data_ptr(), 2.0, n, recv.ptr(1), rt.signal_peer(1, cnt_off), blocks)
            elif rank == 1:
                N.k_wait_count(rt.signal_local(cnt_off), epoch * blocks, rt.timeout_ns, rank)

        def cpu_step():
            if rank == 0:
                N.k_saxpy(x.data_ptr(), y.data_ptr(), 2.0, n)
                rt.native.host_put(y.data_ptr(), 1, recv.index, 0, 4 * n)  # copy engine, current stream
                torch.cuda.current_stream().synchronize()
            rt.barrier()

        def nccl_step():
            if rank == 0:
                N.k_saxpy(x.data_ptr(), y.data_ptr(), 2.0, n)
                dist.send(y[:n], 1)
            elif rank == 1:
                dist.recv(nccl_buf[:n], 0)

        row["gpu_triggered"] = round(timed(gpu_step), 2)
        row["cpu_driven"] = round(timed(cpu_step), 2)
        row["nccl"] = round(timed(nccl_step), 2)
        res["sizes"].append(row)
        if store is not None and rank == 0:
            store.add(key, row)
    rt.check_device_errors()
    if rank == 0:
        print(json.dumps(res))
        if args.out:
            with open(args.out, "w") as f:
                json.dump(res, f, indent=1)
    rt.barrier()
    rt.finalize()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
