"""Rank program for the multi-GPU tests (one process per GPU, launched by
opengda_b200.parallel.launch).  Writes a JSON result per rank."""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from opengda_b200 import native  # noqa: E402
from opengda_b200.parallel import Barrier, Bootstrap, Runtime  # noqa: E402


def main():
    out = sys.argv[1]
    boot = Bootstrap.from_env()
    rt = Runtime(boot)
    r, n = rt.rank, rt.size
    N = native()
    res = {"rank": r, "gpu": rt.gpu_id, "nvls": rt.multicast_supported}
    right, left = (r + 1) % n, (r - 1) % n

    # 1. puts into the right neighbour with a per-rank pattern, verified by the receiver
    buf = rt.alloc_tensor((1 << 22,), torch.uint8)
    src = torch.empty(1 << 22, dtype=torch.uint8, device="cuda")
    N.k_fill_pattern(src.data_ptr(), 1 << 22, 100 + r)
    bar = Barrier(rt)
    torch.cuda.synchronize()
    bar.device_barrier()
    N.k_copy(buf.ptr(right), src.data_ptr(), 1 << 22)
    bar.device_barrier()
    bad = torch.zeros(1, dtype=torch.int64, device="cuda")
    N.k_check_pattern(buf.ptr(), 1 << 22, 100 + left, bad.data_ptr())
    torch.cuda.synchronize()
    res["put_bad_bytes"] = int(bad.item())

    # 2. get: read the left neighbour's buffer (it holds left-left's pattern)
    dst = torch.zeros(1 << 22, dtype=torch.uint8, device="cuda")
    N.k_copy(dst.data_ptr(), buf.ptr(left), 1 << 22)
    bad.zero_()
    N.k_check_pattern(dst.data_ptr(), 1 << 22, 100 + (left - 1) % n, bad.data_ptr())
    bar.device_barrier()
    torch.cuda.synchronize()
    res["get_bad_bytes"] = int(bad.item())

    # 3. host-queued put_no_db to the right neighbour, flushed on the device
    qsrc = rt.alloc_tensor((1 << 16,), torch.uint8)
    qdst = rt.alloc_tensor((1 << 16,), torch.uint8)
    N.k_fill_pattern(qsrc.ptr(), 1 << 16, 7 + r)
    torch.cuda.synchronize()
    rt.reset()
    tok = rt.put_no_db(qsrc.index, right, qdst.index, 1 << 16)
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    N.k_flush(rt.prepare_trigger(tok), st.data_ptr())
    rt.wait(tok)
    bar.device_barrier()
    bad.zero_()
    N.k_check_pattern(qdst.ptr(), 1 << 16, 7 + left, bad.data_ptr())
    torch.cuda.synchronize()
    res["queued_bad_bytes"] = int(bad.item()) + int(st.item())

    # 4. barriers: single (reference-style setup/wait) and continuous 10000
    flag = torch.zeros(1, dtype=torch.int64, device="cuda")
    bar.run_single(flag.data_ptr())
    bar.wait_completion()
    torch.cuda.synchronize()
    res["single_flag"] = int(flag.item())
    cnt = torch.zeros(1, dtype=torch.int64, device="cuda")
    nb = 10000
    torch.cuda.synchronize()
    boot.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    bar.run_continuous(nb, cnt.data_ptr())
    e.record()
    bar.wait_continuous()
    torch.cuda.synchronize()
    res["continuous_count"] = int(cnt.item())
    res["barrier_us"] = s.elapsed_time(e) * 1e3 / nb
    if rt.multicast_supported:
        bn = Barrier(rt, nvls=True)
        boot.barrier()
        s.record()
        bn.run_continuous(nb, cnt.data_ptr())
        e.record()
        bn.wait_continuous()
        torch.cuda.synchronize()
        res["nvls_barrier_us"] = s.elapsed_time(e) * 1e3 / nb
        res["nvls_continuous_count"] = int(cnt.item())

    # 5. allreduce, every algorithm, against a torch fp32 reference
    from opengda_b200.ops.collectives import Allreduce
    ar = Allreduce(rt, 1 << 20)
    errs = {}
    for algo in (["oneshot", "twoshot"] + (["nvls"] if rt.multicast_supported else [])):
        for count in (1024, 65536, 1 << 20):
            g = torch.Generator(device="cuda").manual_seed(1000 + count)
            allx = [torch.randn(count, generator=g, device="cuda").to(torch.bfloat16) for _ in range(n)]
            ar.input(count).copy_(allx[r])
            y = ar(count, algo=algo, scale=0.5)
            torch.cuda.synchronize()
            ref = 0.5 * torch.stack([x.float() for x in allx]).sum(0)
            errs[f"{algo}_{count}"] = float((y.float() - ref).abs().max().item())
            boot.barrier()
    res["allreduce_maxerr"] = errs

    # 6. distributed GEMM, both modes, small shape vs fp32
    from opengda_b200.models.dist_gemm import DistGemm, make_operands
    for fused in (False, True):
        for mode in ("ag", "rs"):
            M = Nn = K = 2048
            model = DistGemm(M, Nn, K, mode, rt=rt, fused=fused)
            worst = 0.0
            for call in range(4):  # several calls: epochs, both buffer parities, done counters
                A, B, (Af, Bf) = make_operands(M, Nn, K, mode, n, r, seed=2 + call)
                C = model(A, B)
                torch.cuda.synchronize()
                full = Af.float() @ Bf.float().t()
                ref = full[:, r * Nn // n:(r + 1) * Nn // n] if mode == "ag" else full[r * M // n:(r + 1) * M // n]
                worst = max(worst, float(((C.float() - ref).norm() / ref.norm()).item()))
            res[f"gemm_{mode}{'_fused' if fused else ''}_relerr"] = worst
    # 7. Jacobi with fused halo puts vs the CPU oracle (gathered field, bit-exact)
    import numpy as np
    from opengda_b200.models.jacobi import Jacobi, jacobi_np
    jnx, jny, jit = 1024, 4 * n + 70, 25
    jac = Jacobi(jnx, jny, rt=rt)
    jac.run(jit)
    torch.cuda.synchronize()
    parts = boot.allgather_obj(jac.owned().cpu().numpy())
    field = np.concatenate(parts, axis=0)
    ref = jacobi_np(jnx, jny, jit)[1:-1]
    res["jacobi_mismatch"] = int((field != ref).sum())
    # 8. MoE expert-parallel layer vs an fp32 reference (all experts' weights gathered)
    from opengda_b200.models.moe import MoELayer, make_inputs, reference_moe
    T, H, E, k, I = 256, 512, 8 * n, 4, 256
    layer = MoELayer(T, H, E, k, I, rt=rt, weight_std=0.05)
    cat = lambda t: torch.cat([q.cuda() for q in boot.allgather_obj(t.cpu())])  # noqa: E731
    wg, wu, w2 = cat(layer.w_gate), cat(layer.w_up), cat(layer.w2)
    worst = 0.0
    for call in range(3):
        x, logits = make_inputs(T, H, E, r, seed=20 + call)
        y = layer(x, logits)
        torch.cuda.synchronize()
        rows = torch.arange(0, T, 16, device="cuda")
        ref = reference_moe(x, logits, k, wg, wu, w2, rows)
        worst = max(worst, float(((y[rows].float() - ref).norm() / ref.norm()).item()))
    res["moe_relerr"] = worst

    # 9. active messages: host sends + device poll, device request/reply ping-pong
    from opengda_b200.parallel.am import Am, CHECKSUM, COUNTER_ADD
    am = Am(rt, nslots=8, max_payload=1024)
    for i in range(20):  # more than the ring: exercises credits (receiver drains in between)
        while not am.check_can_send(right):
            am.poll_once()
        am.send_handle(right, COUNTER_ADD, [r + 1])
        am.poll_once()
    payload = bytes((i * 7 + r) % 256 for i in range(1000))
    am.send_payload(right, CHECKSUM, [0], payload)
    import time as _t
    t0 = _t.time()
    while (am.counter() < 20 * (left + 1) or am.checksum() == 0) and _t.time() - t0 < 10:
        am.poll_once()
    res["am_counter_ok"] = am.counter() == 20 * (left + 1)
    res["am_checksum_ok"] = am.checksum() == sum((i * 7 + left) % 256 for i in range(1000))
    boot.barrier()
    rtt = torch.zeros(1, dtype=torch.int64, device="cuda")
    if r < 2:  # device-driven sends on directions that also carried host sends above
        am.pingpong(1 - r, 1000, "reqrep", r == 0, rtt.data_ptr())
    torch.cuda.synchronize()
    res["am_reqrep_rtt_us"] = rtt.item() / 1000 / 1e3 if r == 0 else None
    rt.check_device_errors()
    torch.cuda.synchronize()

    # 10. litmus tests across GPUs 0 and 1 (NVLink peer words, random delays)
    from opengda_b200.utils import litmus
    mp = litmus.run(litmus.MP, iters=20000, k=64, max_delay=512, rt=rt)
    sb = litmus.run(litmus.SB, iters=20000, use_fence=True, max_delay=512, rt=rt)
    if r == 0:
        res["litmus_mp"] = mp
        res["litmus_sb"] = sb
    torch.cuda.synchronize()

    # 11. failure injection: in a dissemination barrier rank 1 leaves its signal out; the rank
    # waiting for it ends the barrier with ETIMEDOUT (300 ms bound), and every context still
    # runs kernels afterwards.  Nobody leaves the job and no multicast memory is involved.
    boot.barrier()
    fb = Barrier(rt)  # dissemination (no NVLS)
    fb.device_barrier(3)
    torch.cuda.synchronize()
    N.read_errors(True)
    fb.inject_fault(Barrier.SKIP_SIGNAL if r == 1 else 0, after=0, timeout_ms=300)
    fb.device_barrier(1)
    torch.cuda.synchronize()
    e = N.read_errors(True)
    res["inject_error"] = {"status": e["status"], "where": e["where"]}
    probe = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    N.k_fill_pattern(probe.data_ptr(), 1 << 20, 7)
    badp = torch.zeros(1, dtype=torch.int64, device="cuda")
    N.k_check_pattern(probe.data_ptr(), 1 << 20, 7, badp.data_ptr())
    torch.cuda.synchronize()
    res["context_ok_after_inject"] = int(badp.item()) == 0
    boot.barrier()
    with open(f"{out}.{r}", "w") as f:
        json.dump(res, f)
    keep = os.environ.get("GICC_RESULTS_DIR")  # optional copy of every rank's results
    if keep and os.path.isdir(keep):
        with open(os.path.join(keep, f"multigpu_rank{r}.json"), "w") as f:
            json.dump(res, f)
    del ar
    rt.finalize()


if __name__ == "__main__":
    main()
