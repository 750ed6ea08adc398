"""Communication microbenchmarks (put/get/ping-pong/barrier/allreduce configuration) on 2..8 GPUs of one node, ours vs NCCL.

    torchrun --nproc-per-node N bench/comm_bench.py [--quick] [--out results/comm_n{N}.json]

* put / get bandwidth, 8 B .. 256 MiB (powers of 2), byte buffers filled from seed 1:
  every rank puts to (or gets from) its right neighbour at the same time; per-GPU GB/s.
  NCCL arm: batched send/recv on the same ring.
* ping-pong (ranks 0 <-> 1): half round-trip latency per size; NCCL arm: send/recv.
* quiet latency: one 8-byte NVLink store + fence.acq_rel.sys.
* barrier: 10000 barriers in one kernel (continuous mode), dissemination and NVLS;
  NCCL arm: dist.barrier() and a 1-element all_reduce (both in a CUDA graph-free loop).
* with --rs-ag: reduce-scatter and all-gather (NVLS and direct) against NCCL's
  reduce_scatter_tensor / all_gather_into_tensor, bus bandwidth (n-1)/n * S / t;
* allreduce bf16 N(0,1), 1 KiB .. 1 GiB: bus bandwidth 2(n-1)/n * S / t for every
  algorithm (one-shot, two-shot, NVLS, auto) and NCCL.

All times are device times (CUDA events / %globaltimer), max over ranks.
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


def tmax(x: float) -> float:
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def timed(fn, iters: int, warmup: int = 3) -> float:
    """ms per call (device time, max over ranks)."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return tmax(s.elapsed_time(e) / iters)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--quick", action="store_true")
    ap.add_argument("--out", default=None)
    ap.add_argument("--max-put", type=int, default=28)  # 2^28 = 256 MiB
    ap.add_argument("--max-ar", type=int, default=30)   # 2^30 = 1 GiB
    ap.add_argument("--rs-ag", action="store_true", help="also time reduce-scatter and all-gather vs NCCL")
    args = ap.parse_args()
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from datetime import timedelta
    dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))
    n, r = dist.get_world_size(), dist.get_rank()
    from opengda_b200 import native
    from opengda_b200.ops.collectives import Allreduce
    from opengda_b200.parallel import Barrier, Runtime

    N = native()
    rt = Runtime()
    right, left = (r + 1) % n, (r - 1) % n
    results = {"n_gpus": n, "nvls": rt.multicast_supported, "gpu": torch.cuda.get_device_name()}
    from opengda_b200.utils.clocks import BenchClocks
    clk = BenchClocks(local)

    # ---------------- put / get bandwidth ----------------
    maxb = 1 << args.max_put
    buf = rt.alloc_tensor((maxb,), torch.uint8)
    src = torch.empty(maxb, dtype=torch.uint8, device="cuda")
    N.k_fill_pattern(src.data_ptr(), maxb, 1)
    recvb = torch.empty(maxb, dtype=torch.uint8, device="cuda")
    sizes = [1 << k for k in range(3, args.max_put + 1, 2 if args.quick else 1)]
    put, get, nccl_p2p = [], [], []
    for size in sizes:
        reps = max(1, min(1000, (64 << 20) // size))
        ms = timed(lambda: N.k_copy(buf.ptr(right), src.data_ptr(), size, reps, 0, 0, maxb), 5 if args.quick else 10)
        put.append({"bytes": size, "GBps": size * reps / (ms * 1e-3) / 1e9, "us_per_put": ms * 1e3 / reps})
        ms = timed(lambda: N.k_copy(recvb.data_ptr(), buf.ptr(left), size, reps, 0, 0, maxb), 5 if args.quick else 10)
        get.append({"bytes": size, "GBps": size * reps / (ms * 1e-3) / 1e9, "us_per_get": ms * 1e3 / reps})

        def nccl_ring():
            ops = [dist.P2POp(dist.isend, src[:size], right), dist.P2POp(dist.irecv, recvb[:size], left)]
            for w in dist.batch_isend_irecv(ops):
                w.wait()
        nreps = max(1, min(100, (64 << 20) // size))
        ms = timed(lambda: [nccl_ring() for _ in range(nreps)], 3 if args.quick else 5)
        nccl_p2p.append({"bytes": size, "GBps": size * nreps / (ms * 1e-3) / 1e9, "us_per_op": ms * 1e3 / nreps})
    # verify: one full-size put of the seeded pattern lands intact on the right neighbour
    torch.cuda.synchronize()
    dist.barrier()
    N.k_copy(buf.ptr(right), src.data_ptr(), maxb)
    torch.cuda.synchronize()
    dist.barrier()
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    N.k_check_pattern(buf.ptr(), maxb, 1, bad.data_ptr())
    torch.cuda.synchronize()
    results["put"] = put
    results["get"] = get
    results["nccl_sendrecv"] = nccl_p2p
    results["put_verify_bad_bytes"] = int(bad.item())

    # ---------------- ping-pong (ranks 0 and 1) ----------------
    flags_off = rt.signal_alloc(2)
    pp, nccl_pp = [], []
    base = 0
    for size in [8, 64, 512, 4096, 32768, 262144, 1 << 20]:
        iters = 1000 if size <= 4096 else 200
        out = torch.zeros(1, dtype=torch.int64, device="cuda")
        dist.barrier()
        if r in (0, 1):
            peer = 1 - r
            N.k_pingpong(buf.ptr(peer), src.data_ptr(), size, rt.signal_peer(peer, flags_off), rt.signal_local(flags_off),
                         iters, r == 0, base, out.data_ptr(), rt.timeout_ns, r)
        torch.cuda.synchronize()
        base += 2 * iters
        ns = tmax(float(out.item()) if r == 0 else 0.0)
        pp.append({"bytes": size, "half_rtt_us": ns / iters / 2 / 1e3})
        # NCCL ping-pong
        t = src[:size]
        rb = recvb[:size]

        def nccl_pp_fn():
            if r == 0:
                dist.send(t, 1)
                dist.recv(rb, 1)
            elif r == 1:
                dist.recv(rb, 0)
                dist.send(t, 0)
        k = 100
        ms = timed(lambda: [nccl_pp_fn() for _ in range(k)], 3)
        nccl_pp.append({"bytes": size, "half_rtt_us": ms * 1e3 / k / 2})
    results["pingpong"] = pp
    results["nccl_pingpong"] = nccl_pp

    # ---------------- quiet latency ----------------
    out = torch.zeros(1, dtype=torch.int64, device="cuda")
    N.k_quiet_latency(buf.ptr(right), 10000, out.data_ptr())
    torch.cuda.synchronize()
    results["quiet_us"] = tmax(out.item() / 10000 / 1e3)

    # ---------------- barrier ----------------
    nb = 10000
    b = Barrier(rt)
    ms = timed(lambda: b.run_continuous(nb), 2, 1)
    b.wait_continuous()
    results["barrier_us"] = ms * 1e3 / nb
    if rt.multicast_supported:
        bn = Barrier(rt, nvls=True)
        ms = timed(lambda: bn.run_continuous(nb), 2, 1)
        bn.wait_continuous()
        results["barrier_nvls_us"] = ms * 1e3 / nb
    ms = timed(lambda: [dist.barrier() for _ in range(100)], 2)
    results["nccl_barrier_us"] = ms * 1e3 / 100
    one = torch.ones(1, device="cuda")
    ms = timed(lambda: [dist.all_reduce(one) for _ in range(1000)], 2)
    results["nccl_allreduce1_us"] = ms * 1e3 / 1000
    # single barrier per kernel launch (reference test 1 style), host-timed per launch
    ms = timed(lambda: b.device_barrier(), 200, 5)
    results["barrier_single_launch_us"] = ms * 1e3

    # ---------------- allreduce ----------------
    max_count = (1 << args.max_ar) // 2
    del buf, src, recvb
    torch.cuda.empty_cache()
    ar = Allreduce(rt, max_count)
    g = torch.Generator(device="cuda").manual_seed(100 + r)
    ar.input().copy_(torch.randn(max_count, generator=g, device="cuda").to(torch.bfloat16))
    nccl_buf = torch.empty(max_count, dtype=torch.bfloat16, device="cuda")
    algos = ["oneshot", "twoshot"] + (["nvls"] if rt.multicast_supported else [])
    arr = []
    for k in range(10, args.max_ar + 1, 2 if args.quick else 1):
        nbytes = 1 << k
        count = nbytes // 2
        row = {"bytes": nbytes}
        reps = max(3, min(200, (256 << 20) // nbytes))
        for a in algos:
            if a == "oneshot" and nbytes > (64 << 20):
                continue
            ms = timed(lambda: ar(count, algo=a), reps)
            row[a] = {"us": ms * 1e3, "busbw_GBps": 2 * (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
        ms = timed(lambda: ar(count, algo="auto"), reps)
        row["auto"] = {"us": ms * 1e3, "busbw_GBps": 2 * (n - 1) / n * nbytes / (ms * 1e-3) / 1e9, "algo": ar.pick(count)}
        x = nccl_buf[:count]
        ms = timed(lambda: dist.all_reduce(x), reps)
        row["nccl"] = {"us": ms * 1e3, "busbw_GBps": 2 * (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
        arr.append(row)
    results["allreduce_bf16"] = arr
    rt.check_device_errors()

    # ---------------- reduce-scatter / all-gather (bus bandwidth (n-1)/n * S / t) ----------
    if args.rs_ag:
        from opengda_b200.ops.collectives import AllGather, ReduceScatter
        del ar
        torch.cuda.empty_cache()
        rs = ReduceScatter(rt, max_count)
        rs.input().copy_(torch.randn(max_count, generator=g, device="cuda").to(torch.bfloat16))
        ag = AllGather(rt, max_count * 2 // n)
        rows = []
        for k in range(16, args.max_ar + 1, 2):
            nbytes = 1 << k
            count = nbytes // 2
            if count % (8 * n):
                continue
            reps = max(3, min(100, (256 << 20) // nbytes))
            row = {"bytes": nbytes}
            for nv in ([True, False] if rs.nvls else [False]):
                tag = "nvls" if nv else "direct"
                ms = timed(lambda: rs(count, nvls=nv), reps)
                row[f"rs_{tag}"] = {"us": ms * 1e3, "busbw_GBps": (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
                ms = timed(lambda: ag(nbytes // n, nvls=nv), reps)
                row[f"ag_{tag}"] = {"us": ms * 1e3, "busbw_GBps": (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
            full = nccl_buf[:count]
            part = torch.empty(count // n, dtype=torch.bfloat16, device="cuda")
            ms = timed(lambda: dist.reduce_scatter_tensor(part, full), reps)
            row["rs_nccl"] = {"us": ms * 1e3, "busbw_GBps": (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
            ms = timed(lambda: dist.all_gather_into_tensor(full, part), reps)
            row["ag_nccl"] = {"us": ms * 1e3, "busbw_GBps": (n - 1) / n * nbytes / (ms * 1e-3) / 1e9}
            rows.append(row)
        results["reduce_scatter_all_gather"] = rows
        rt.check_device_errors()
        ar = None
    results["clocks"] = clk.finish()
    if r == 0:
        js = json.dumps(results)
        print(js)
        if args.out:
            with open(args.out, "w") as f:
                f.write(js + "\n")
    del ar
    torch.cuda.synchronize()
    rt.finalize()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
