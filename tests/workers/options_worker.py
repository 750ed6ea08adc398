"""Rank program for the multi-GPU checks of the options and secondary kernels
(launched by opengda_b200.parallel.launch; one JSON result per rank):

* the ring-stripe fp32 matmul (RingMatmul) against an fp64 product of the full matrices;
* the fused all-gather GEMM with the copy-engine transfer (transfer="ce"), and fed
  zero-copy from pinned host memory through its input slots;
* the reduce-scatter GEMM with the join option (rs_join);
* the MoE layer with confined dispatch and the staged combine (dispatch_ctas, combine_ctas);
* the persistent Jacobi kernel (one cooperative launch for many iterations);
* allreduce with a device-side call counter, captured in a CUDA graph and replayed.
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

from opengda_b200.parallel import Bootstrap, Runtime  # noqa: E402


def main():
    out = sys.argv[1]
    boot = Bootstrap.from_env()
    rt = Runtime(boot)
    r, n = rt.rank, rt.size
    res = {"rank": r}

    # 1. ring-stripe fp32 matmul, three calls (monotonic counters across calls), in the
    #    tensor-core mode (default) and the SIMT mode
    try:
        from opengda_b200.models.ring_mm import RingMatmul, make_stripes
        N = 1024
        for key, tc in (("ring_mm_err", True), ("ring_mm_simt_err", False)):
            mm = RingMatmul(N, rt=rt, push_ctas=4, tensor_cores=tc)
            worst = 0.0
            for call in range(3):
                A_s, B_s, A, B = make_stripes(N, n, r, seed=call)
                C = mm(A_s, B_s).cpu().double()
                Ns = N // n
                ref = A[r * Ns:(r + 1) * Ns].double() @ B.double()
                scale = A[r * Ns:(r + 1) * Ns].double().abs() @ B.double().abs()
                worst = max(worst, float(((C - ref).abs() / scale).max()))
            rt.check_device_errors()
            res[key] = worst
    except Exception as e:  # record it and go on: the other steps still report
        res["step1_error"] = f"{type(e).__name__}: {e}"

    # 2. distributed GEMM options vs fp32
    try:
        from opengda_b200.models.dist_gemm import DistGemm, make_operands
        for name, mode, kw, attr in (("ag_ce", "ag", {"transfer": "ce"}, {}), ("rs_join", "rs", {}, {"rs_join": True}),
                                     ("rs_group2", "rs", {}, {"rs_raster_group": 2}),
                                     ("ag_unicast", "ag", {"nvls": False}, {}), ("rs_unicast", "rs", {"nvls": False}, {}),
                                     ("ag_pair1", "ag", {}, {"pair": 1}), ("ag_pair2", "ag", {}, {"pair": 2}),
                                     ("ag_pair2_unicast", "ag", {"nvls": False}, {"pair": 2}),
                                     ("rs_pair1", "rs", {}, {"pair": 1}), ("rs_pair2", "rs", {}, {"pair": 2})):
            # CTA-pair tiles need 256-row bands per shard and 512-column blocks per rank
            M = Nn = 4096 if "pair" in attr else 2048
            K = 2048
            model = DistGemm(M, Nn, K, mode, rt=rt, fused=True, **kw)
            for k, v in attr.items():
                setattr(model, k, v)
            worst = 0.0
            for call in range(4):
                A, B, (Af, Bf) = make_operands(M, Nn, K, mode, n, r, seed=2 + call)
                C = model(A, B)
                torch.cuda.synchronize()
                full = Af.float() @ Bf.float().t()
                ref = full[:, r * Nn // n:(r + 1) * Nn // n] if mode == "ag" else full[r * M // n:(r + 1) * M // n]
                worst = max(worst, float(((C.float() - ref).norm() / ref.norm()).item()))
            rt.check_device_errors()
            res[f"gemm_{name}_relerr"] = worst
    except Exception as e:  # record it and go on: the other steps still report
        res["step2_error"] = f"{type(e).__name__}: {e}"

    # 2b. the fused AG GEMM fed zero-copy: pinned host copies land in the model's input slots
    #     (HostFeeder over DistGemm.input_slots()), a different A every call
    try:
        from opengda_b200.models.dist_gemm import DistGemm, make_operands
        from opengda_b200.utils.feeder import HostFeeder
        M = Nn = 2048
        K = 1024
        model = DistGemm(M, Nn, K, "ag", rt=rt, fused=True)
        model(*make_operands(M, Nn, K, "ag", n, r, seed=1)[:2])  # one plain call first: the slots rotate
        ops = [make_operands(M, Nn, K, "ag", n, r, seed=30 + i) for i in range(5)]
        hosts = [o[0].cpu().pin_memory() for o in ops]
        feeder = HostFeeder(ops[0][0].shape, ops[0][0].dtype, torch.device("cuda"), bufs=model.input_slots())
        worst = 0.0
        feeder.submit(hosts[0])
        for i in range(5):
            if i + 1 < 5:
                feeder.submit(hosts[i + 1])
            a = feeder.next()
            C = model(a, ops[i][1])
            feeder.release()
            Af, Bf = ops[i][2]
            ref = (Af.float() @ Bf.float().t())[:, r * Nn // n:(r + 1) * Nn // n]
            worst = max(worst, float(((C.float() - ref).norm() / ref.norm()).item()))
        torch.cuda.synchronize()
        rt.check_device_errors()
        res["gemm_ag_feeder_relerr"] = worst
    except Exception as e:  # record it and go on: the other steps still report
        res["step2b_error"] = f"{type(e).__name__}: {e}"

    # 3. MoE with few dispatching CTAs and the staged combine
    try:
        from opengda_b200.models.moe import MoELayer, make_inputs, reference_moe
        T, H, E, k, I = 256, 512, 8 * n, 4, 256
        layer = MoELayer(T, H, E, k, I, rt=rt, weight_std=0.05)
        layer.dispatch_ctas = 8
        layer.combine_ctas = 8
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
        rt.check_device_errors()
        res["moe_confined_relerr"] = worst
    except Exception as e:  # record it and go on: the other steps still report
        res["step3_error"] = f"{type(e).__name__}: {e}"

    # 4. persistent Jacobi (one cooperative launch per run), mixed with per-iteration steps,
    #    against the CPU oracle (bit-exact)
    try:
        import numpy as np
        from opengda_b200.models.jacobi import Jacobi, jacobi_np
        jnx, jny = 1024, 4 * n + 70
        jac = Jacobi(jnx, jny, rt=rt, persistent=True)
        jac.run(9)
        jac.step()
        jac.run(15)
        torch.cuda.synchronize()
        rt.check_device_errors()
        field = np.concatenate(boot.allgather_obj(jac.owned().cpu().numpy()), axis=0)
        res["jacobi_persistent_mismatch"] = int((field != jacobi_np(jnx, jny, 25)[1:-1]).sum())
    except Exception as e:  # record it and go on: the other steps still report
        res["step4_error"] = f"{type(e).__name__}: {e}"

    # 5. allreduce captured in a CUDA graph (device-side call counter), every algorithm,
    #    three replays with new inputs each
    try:
        from opengda_b200.ops.collectives import Allreduce
        count = 1 << 18
        errs = {}
        for algo in (["oneshot", "twoshot"] + (["nvls"] if rt.multicast_supported else [])):
            ar = Allreduce(rt, count, graph_safe=True)
            src = torch.zeros(count, dtype=torch.bfloat16, device="cuda")
            ar.input(count).copy_(src)
            ar(count, algo=algo)
            torch.cuda.synchronize()
            boot.barrier()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                ar.input(count).copy_(src)
                ar(count, algo=algo, scale=0.5)
            worst = 0.0
            for k in range(3):
                gen = torch.Generator(device="cuda").manual_seed(500 + k)
                allx = [torch.randn(count, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(n)]
                src.copy_(allx[r])
                boot.barrier()
                graph.replay()
                torch.cuda.synchronize()
                ref = 0.5 * torch.stack([x.float() for x in allx]).sum(0)
                worst = max(worst, float((ar.output(count).float() - ref).abs().max().item()))
                boot.barrier()
            errs[algo] = worst
            del graph, ar
        rt.check_device_errors()
        res["allreduce_graph_maxerr"] = errs
    except Exception as e:  # record it and go on: the other steps still report
        res["step5_error"] = f"{type(e).__name__}: {e}"

    # 6. standalone reduce-scatter (NVLS when available, and direct) and all-gather
    try:
        from opengda_b200.ops.collectives import AllGather, ReduceScatter
        count = 8 * n * 4096
        rs = ReduceScatter(rt, count, out_dtype=torch.float32)
        gen = torch.Generator(device="cuda").manual_seed(900)
        allx = [torch.randn(count, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(n)]
        ref = torch.stack([x.float() for x in allx]).sum(0)[r * count // n:(r + 1) * count // n]
        errs = {}
        for nv in ([True, False] if rs.nvls else [False]):
            rs.input(count).copy_(allx[r])
            boot.barrier()
            y = rs(count, scale=1.0, nvls=nv)
            torch.cuda.synchronize()
            errs["nvls" if nv else "direct"] = float((y - ref).abs().max().item())
            boot.barrier()
        res["reduce_scatter_maxerr"] = errs
        ag = AllGather(rt, 1 << 16)
        bad = 0
        for nv in ([True, False] if ag.nvls else [False]):
            ag.shard(1 << 16).copy_(torch.full((1 << 16,), 10 + r, dtype=torch.uint8, device="cuda"))
            boot.barrier()
            out_ag = ag(1 << 16, nvls=nv)
            torch.cuda.synchronize()
            want = torch.arange(n, device="cuda", dtype=torch.uint8).view(n, 1) + 10
            bad += int((out_ag != want).sum().item())
            boot.barrier()
        rt.check_device_errors()
        res["all_gather_bad"] = bad
    except Exception as e:  # record it and go on: the other steps still report
        res["step6_error"] = f"{type(e).__name__}: {e}"

    # 7. MoE all-to-all round trip alone (identity experts)
    try:
        layer2 = MoELayer(T, H, E, k, I, rt=rt, weight_std=0.05)
        worst = 0.0
        for call in range(3):
            x, logits = make_inputs(T, H, E, r, seed=60 + call)
            y = layer2.dispatch_combine(x, logits).float()
            torch.cuda.synchronize()
            wsum = torch.topk(torch.softmax(logits, -1), k, dim=-1).values.sum(-1, keepdim=True)
            ref = x.float() * wsum
            worst = max(worst, float(((y - ref).norm() / ref.norm()).item()))
        rt.check_device_errors()
        res["moe_dispatch_combine_relerr"] = worst
    except Exception as e:  # record it and go on: the other steps still report
        res["step7_error"] = f"{type(e).__name__}: {e}"

    # 8. torch.distributed-style calls on ordinary tensors
    try:
        from opengda_b200.parallel.functional import Collectives
        col = Collectives(rt)
        gen = torch.Generator(device="cuda").manual_seed(1234)
        xs = [torch.randn(1000, 37, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(n)]
        t = xs[r].clone()
        col.all_reduce(t)
        ref = torch.stack([x.float() for x in xs]).sum(0)
        errs = {"all_reduce": float((t.float() - ref).abs().max().item())}
        big = [torch.randn(8 * n * 300, generator=gen, device="cuda").to(torch.bfloat16) for _ in range(n)]
        o = torch.empty(8 * 300, dtype=torch.float32, device="cuda")
        col.reduce_scatter_tensor(o, big[r])
        ref = torch.stack([x.float() for x in big]).sum(0)[r * 2400:(r + 1) * 2400]
        errs["reduce_scatter"] = float((o - ref).abs().max().item())
        shard = torch.full((4, 8), float(r), dtype=torch.float32, device="cuda")
        g_out = torch.empty(4 * n, 8, dtype=torch.float32, device="cuda")
        col.all_gather_into_tensor(g_out, shard)
        want = torch.arange(n, device="cuda", dtype=torch.float32).repeat_interleave(4).view(-1, 1).expand(-1, 8)
        errs["all_gather"] = float((g_out - want).abs().max().item())
        torch.cuda.synchronize()
        rt.check_device_errors()
        res["functional_maxerr"] = errs
    except Exception as e:  # record it and go on: the other steps still report
        res["step8_error"] = f"{type(e).__name__}: {e}"

    boot.barrier()
    with open(f"{out}.{r}", "w") as f:
        json.dump(res, f)
    torch.cuda.synchronize()
    rt.finalize()


if __name__ == "__main__":
    main()
