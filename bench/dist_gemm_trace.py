"""Timeline of the fused all-gather -> GEMM kernel (BASELINE config 3a) on N GPUs.

    torchrun --nproc-per-node N bench/dist_gemm_trace.py [--size 16384] [--comm-ctas 16]
             [--no-nvls] [--units 4] [--steps 40] [--out DIR]

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


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--size", type=int, default=16384)
    ap.add_argument("--comm-ctas", type=int, default=0, help="0 = the model's default")
    ap.add_argument("--no-nvls", action="store_true")
    ap.add_argument("--units", type=int, default=4)
    ap.add_argument("--steps", type=int, default=40)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--out", default=None)
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
    A, B, (Af, Bf) = make_operands(M, N, K, "ag", world, rank, seed=2, device=dev)
    rows = torch.arange(0, M, 61, device=dev)
    ref = Af[rows].float() @ B.float().t()
    del Af, Bf
    m = DistGemm(M, N, K, "ag", rt=rt, device=dev, nvls=False if args.no_nvls else None)
    m.units_per_band = args.units
    if args.comm_ctas:
        m.comm_ctas = args.comm_ctas
    m.a_slot(0).copy_(A)
    m.a_slot(1).copy_(A)
    for _ in range(args.warmup):
        m(m.a_slot(), B)
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(args.steps):
        m(m.a_slot(), B)
    e.record()
    torch.cuda.synchronize()
    ms = max_over_ranks(s.elapsed_time(e) / args.steps)
    C = m(m.a_slot(), B)
    torch.cuda.synchronize()
    rel = ((C[rows].float() - ref).norm() / ref.norm()).item()
    m.trace = torch.zeros(m.trace_words(), dtype=torch.int64, device=dev)
    m(m.a_slot(), B)
    torch.cuda.synchronize()
    rt.check_device_errors()
    tr = m.trace.cpu().numpy()
    m.trace = None
    G = m.grid or torch.cuda.get_device_properties(dev).multi_processor_count
    summ = summarize(tr, world, M, m.nvls, m.units_per_band, G)
    if args.out:
        os.makedirs(args.out, exist_ok=True)
        np.save(os.path.join(args.out, f"ag_trace_r{rank}.npy"), tr)
    allsum = [None] * world
    dist.all_gather_object(allsum, summ)
    if rank == 0:
        print(json.dumps({
            "kernel": "k_ag_gemm", "n_gpus": world, "M": M, "N": N, "K": K, "nvls": m.nvls,
            "comm_ctas": m.comm_ctas, "units_per_band": m.units_per_band,
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
