"""Timeline of the fused distributed GEMM kernels (M = N = K = 16384, bf16) on N GPUs.

    torchrun --nproc-per-node N bench/dist_gemm_trace.py [--mode ag|rs] [--size 16384]
             [--comm-ctas C] [--no-nvls] [--units 4] [--steps 40] [--out DIR]

--mode rs traces the NVLS reduce-scatter kernel (last tile stored, reduce start / end,
reduction lag behind each band, owner-side reduce rate); the rest below is for --mode ag.

Times the fused kernel (device time, max over ranks), then runs one more call with the
kernel's %globaltimer trace buffer switched on and summarises, per rank:

* ``comm_end_us`` / ``egress_GBps`` -- when the last unit of this rank's A shard was
  released to its consumers, and the bytes it sent per second (NVLS: one multicast copy of
  the shard; unicast: one copy per peer);
* ``tiles_per_ms_during_comm`` / ``after`` -- tensor-core tile throughput while the
  transfer is in flight and after it, which shows whether pushing slows the GEMM;
* ``producer_wait_us`` -- time the TMA producers spent waiting for remote A bands;
* ``span_us`` -- first CTA start to last CTA end.

With ``--out`` the raw trace of every rank is saved as ``ag_trace_r<rank>.npy``
(layout: see the comment above ``k_ag_gemm`` in csrc/kernels/gemm_dist.cu).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
from datetime import timedelta

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def summarize(t, n, M, nvls, Q, G):
    import numpy as np

    t = t.astype(np.int64)
    nb = M // n // 128
    num_n = (M // n) // 256
    T = n * nb * num_n
    U = (1 if nvls else n - 1) * nb * Q
    wait = t[:2 * T].reshape(T, 2)
    epi = t[2 * T:3 * T]
    units = t[3 * T:3 * T + 2 * U].reshape(U, 2)
    cta = t[3 * T + 2 * U:3 * T + 2 * U + 2 * G].reshape(G, 2)
    t0 = cta[:, 0].min()
    comm_end = (units[:, 1].max() - t0) / 1e3 if U else 0.0
    e = (epi - t0) / 1e3
    span = (cta[:, 1].max() - t0) / 1e3
    sent = (1 if nvls else n - 1) * (M // n) * M * 2
    during = (e <= comm_end).sum()
    return {
        "span_us": round(float(span), 1),
        "comm_end_us": round(float(comm_end), 1),
        "egress_GBps": round(float(sent / (comm_end * 1e-6) / 1e9), 1) if comm_end > 0 else None,
        "tiles_per_ms_during_comm": round(float(during / comm_end * 1e3), 1) if comm_end > 0 else None,
        "tiles_per_ms_after": round(float((len(e) - during) / max(e.max() - comm_end, 1e-3) * 1e3), 1),
        "producer_wait_us": round(float((wait[:, 1] - wait[:, 0]).sum() / 1e3), 1),
    }


def summarize_rs(t, n, M, Q, G):
    """NVLS reduce-scatter trace: [T] tile stored, [2U] reduce unit start/end, [2G] CTA."""
    import numpy as np

    t = t.astype(np.int64)
    nbo = M // n // 128
    num_n = M // 256
    T = n * nbo * num_n
    U = nbo * Q
    epi = t[:T]
    units = t[T:T + 2 * U].reshape(U, 2)
    cta = t[T + 2 * U:T + 2 * U + 2 * G].reshape(G, 2)
    t0 = cta[:, 0].min()
    us = lambda x: (x - t0) / 1e3  # noqa: E731
    span = float(us(cta[:, 1].max()))
    gemm_end = float(us(epi.max()))
    # per band b: when its last tile (any owner) was stored vs when its reduction ended
    mb = np.arange(T) // num_n                       # global m-block of tile t
    band_of = mb % nbo                               # band within the owner's block
    band_done = np.array([us(epi[band_of == b].max()) for b in range(nbo)])
    red_end = np.array([us(units[b * Q:(b + 1) * Q, 1].max()) for b in range(nbo)])
    red_start = np.array([us(units[b * Q:(b + 1) * Q, 0].min()) for b in range(nbo)])
    out_bytes = (M // n) * M * 2
    return {
        "span_us": round(span, 1),
        "last_tile_stored_us": round(gemm_end, 1),
        "reduce_after_gemm_us": round(span - gemm_end, 1),
        "reduce_first_start_us": round(float(red_start.min()), 1),
        "reduce_last_end_us": round(float(red_end.max()), 1),
        "reduce_lag_mean_us": round(float((red_end - band_done).mean()), 1),
        "owner_GBps_while_reducing": round(out_bytes / ((red_end.max() - red_start.min()) * 1e-6) / 1e9, 1),
        "tiles_per_ms": round(T / max(gemm_end, 1e-3) * 1e3, 1),
    }


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=16384)
    ap.add_argument("--comm-ctas", type=int, default=0, help="0 = the model's default")
    ap.add_argument("--no-nvls", action="store_true")
    ap.add_argument("--units", type=int, default=4)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--out", default=None)
    ap.add_argument("--mode", default="ag", choices=["ag", "rs"], help="rs: the NVLS reduce-scatter kernel")
    ap.add_argument("--transfer", default="sm", choices=["sm", "ce"], help="ag: SM pushes or copy engines")
    ap.add_argument("--join", action="store_true", help="rs: CTAs out of GEMM tiles join the reduction")
    ap.add_argument("--raster-group", type=int, default=0, help="rs: m-blocks per raster group (0 = 16)")
    args = ap.parse_args()

    import numpy as np
    import torch
    import torch.distributed as dist

    rank, world, lr = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(lr)
    dev = torch.device("cuda", lr)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from opengda_b200.models.dist_gemm import DistGemm, make_operands
    from opengda_b200.parallel import Runtime
    from opengda_b200.utils.timing import max_over_ranks

    rt = Runtime()
    M = N = K = args.size
    A, B, (Af, Bf) = make_operands(M, N, K, args.mode, world, rank, seed=2, device=dev)
    rows = torch.arange(0, M // world if args.mode == "rs" else M, 61, device=dev)
    if args.mode == "ag":
        ref = Af[rows].float() @ B.float().t()
    else:
        ref = Af[rank * (M // world) + rows].float() @ Bf.float().t()
    del Af, Bf
    m = DistGemm(M, N, K, args.mode, rt=rt, device=dev, nvls=False if args.no_nvls else None,
                 transfer=args.transfer if args.mode == "ag" else "sm")
    if args.mode == "rs" and not m.nvls:
        raise SystemExit("the trace covers the NVLS reduce-scatter kernel only")
    m.pair = 0  # the trace buffer belongs to the single-CTA kernels
    m.units_per_band = args.units
    m.rs_join = bool(args.join)
    m.rs_raster_group = args.raster_group
    if args.comm_ctas:
        if args.mode == "ag":
            m.comm_ctas = args.comm_ctas
        else:
            m.rs_reduce_ctas = args.comm_ctas
    if args.mode == "ag":
        m.a_slot(0).copy_(A)
        m.a_slot(1).copy_(A)
    step = (lambda: m(m.a_slot(), B)) if args.mode == "ag" else (lambda: m(A, B))
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        step()
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / args.steps)
    C = step()
    torch.cuda.synchronize()
    rel = ((C[rows].float() - ref).norm() / ref.norm()).item()
    m.trace = torch.zeros(m.trace_words(), dtype=torch.int64, device=dev)
    step()
    torch.cuda.synchronize()
    rt.check_device_errors()
    tr = m.trace.cpu().numpy()
    m.trace = None
    G = m.grid or torch.cuda.get_device_properties(dev).multi_processor_count
    if args.mode == "ag":
        summ = summarize(tr, world, M, m.nvls, m.units_per_band, G)
    else:
        summ = summarize_rs(tr, world, M, m.units_per_band, G)
    if args.out:
        os.makedirs(args.out, exist_ok=True)
        np.save(os.path.join(args.out, f"ag_trace_r{rank}.npy"), tr)
    allsum = [None] * world
    dist.all_gather_object(allsum, summ)
    if rank == 0:
        print(json.dumps({
            "kernel": "k_ag_gemm" if args.mode == "ag" else "k_gemm_rs_nvls", "n_gpus": world, "M": M, "N": N,
            "K": K, "nvls": m.nvls, "comm_ctas": m.comm_ctas if args.mode == "ag" else m.rs_reduce_ctas,
            "raster_group": args.raster_group,
            "units_per_band": m.units_per_band,
            "ms_per_call_max_over_ranks": round(ms, 4), "tflops": round(2.0 * M * N * K / ms / 1e9, 1),
            "relerr_vs_fp32": rel, "per_rank_trace": allsum}))
    del m
    torch.cuda.synchronize()
    rt.finalize()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
