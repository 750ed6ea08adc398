"""Jacobi benchmark: 5-point fp32 stencil on a 32768 x 32768 grid,
1-D row decomposition over 1..8 GPUs, 1000 iterations, ours (halo puts fused into the
stencil kernel) vs an NCCL arm (same stencil kernel, halos exchanged with NCCL send/recv
between launches -- the host-driven pattern of the reference's MPI build).

    python bench/jacobi_bench.py [--nx 32768 --ny 32768 --iters 1000]
    torchrun --nproc-per-node N bench/jacobi_bench.py ...
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
    ap.add_argument("--nx", type=int, default=32768)
    ap.add_argument("--ny", type=int, default=32768)
    ap.add_argument("--iters", type=int, default=1000)
    ap.add_argument("--nccl-iters", type=int, default=None)
    ap.add_argument("--out", default=None)
    ap.add_argument("--persistent", action="store_true",
                    help="one cooperative launch for all iterations instead of one launch per iteration")
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
    from opengda_b200 import native
    from opengda_b200.models.jacobi import Jacobi
    from opengda_b200.utils.timing import max_over_ranks

    from opengda_b200.utils.clocks import BenchClocks

    clk = BenchClocks(local)
    jac = Jacobi(args.nx, args.ny, rt=rt, persistent=args.persistent)
    jac.run(5)  # warm-up
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    jac.run(args.iters)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e))
    if rt:
        rt.check_device_errors()
    interior = (args.nx - 2) * (args.ny - 2)
    res = {"metric": "jacobi_total_s", "impl": "ours-fused-halo-puts" + ("-persistent" if args.persistent else ""),
           "n_gpus": world, "nx": args.nx, "ny": args.ny,
           "iters": args.iters, "total_s": ms / 1e3, "ms_per_iter": ms / args.iters,
           "GLUPs": interior * args.iters / (ms * 1e-3) / 1e9,
           "hbm_GBps_per_gpu": 8.0 * interior / world * args.iters / (ms * 1e-3) / 1e9}

    # ---- NCCL arm: same kernel with no fused puts, halos by send/recv between launches
    if world > 1:
        it_n = args.nccl_iters or args.iters
        N = native()
        bufs = [torch.empty(jac.rows + 2, args.nx, dtype=torch.float32, device="cuda") for _ in range(2)]
        N.k_jacobi_init(bufs[0].data_ptr(), bufs[1].data_ptr(), args.nx, args.ny, jac.rows, jac.g0, 3)
        r, w = jac.rank, jac.world

        def nccl_iter(cur):
            a, b = bufs[cur], bufs[1 - cur]
            N.k_jacobi_step(a.data_ptr(), b.data_ptr(), args.nx, jac.rows, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, r)
            ops = []
            if r > 0:
                ops += [dist.P2POp(dist.isend, b[1], r - 1), dist.P2POp(dist.irecv, b[0], r - 1)]
            if r < w - 1:
                ops += [dist.P2POp(dist.isend, b[jac.rows], r + 1), dist.P2POp(dist.irecv, b[jac.rows + 1], r + 1)]
            for q in dist.batch_isend_irecv(ops):
                q.wait()
        for i in range(5):
            nccl_iter(i % 2)
        torch.cuda.synchronize()
        dist.barrier()
        s.record()
        for i in range(it_n):
            nccl_iter(i % 2)
        e.record()
        torch.cuda.synchronize()
        ms_n = max_over_ranks(s.elapsed_time(e))
        res["nccl"] = {"total_s_scaled_to_iters": ms_n / it_n * args.iters / 1e3, "ms_per_iter": ms_n / it_n}
        # numerics: fused and NCCL fields agree after the same number of iterations? (different
        # iteration counts here; equality is covered by the tests)
    res["clocks"] = clk.finish()
    if rank == 0:
        js = json.dumps(res)
        print(js)
        if args.out:
            with open(args.out, "w") as f:
                f.write(js + "\n")
    if world > 1:
        del jac
        torch.cuda.synchronize()
        rt.finalize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
