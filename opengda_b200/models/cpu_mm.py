"""Distributed dense matmul on CPU ranks (the plumbing configuration, no GPU).

C = A . B in fp32 with M = N = K = 1024; A and B i.i.d. uniform[-1, 1) from seed 0.
A is row-block partitioned across the ranks, B is broadcast from rank 0, each rank
multiplies its row block, and C is gathered to rank 0 and checked against a single-rank
matmul to rtol 1e-5.  Runs over ``torch.distributed`` with the gloo backend (the
reference's analogue is the host MPI ring of examples/mpi_mm.cpp:32-84; with B broadcast
instead of ring-passed, as the config specifies).

    python -m opengda_b200.models.cpu_mm            # spawns 2 gloo ranks on 127.0.0.1
"""
from __future__ import annotations

import os
import time

import torch
import torch.distributed as dist


def make_inputs(M: int = 1024, N: int = 1024, K: int = 1024, seed: int = 0):
    g = torch.Generator().manual_seed(seed)
    A = torch.rand(M, K, generator=g, dtype=torch.float32) * 2 - 1
    B = torch.rand(K, N, generator=g, dtype=torch.float32) * 2 - 1
    return A, B


def distributed_matmul(M: int = 1024, N: int = 1024, K: int = 1024, seed: int = 0):
    """Collective over the default (gloo) group.  Returns (C on rank 0 else None, seconds)."""
    rank, world = dist.get_rank(), dist.get_world_size()
    if M % world:
        raise ValueError("M must divide evenly over the ranks")
    rows = M // world
    if rank == 0:
        A, B = make_inputs(M, N, K, seed)
        blocks = list(A.split(rows, dim=0))
    else:
        B = torch.empty(K, N, dtype=torch.float32)
        blocks = None
    dist.barrier()
    t0 = time.perf_counter()
    a_blk = torch.empty(rows, K, dtype=torch.float32)
    dist.scatter(a_blk, blocks if rank == 0 else None, src=0)
    dist.broadcast(B, src=0)
    c_blk = a_blk @ B
    gathered = [torch.empty(rows, N, dtype=torch.float32) for _ in range(world)] if rank == 0 else None
    dist.gather(c_blk, gathered, dst=0)
    dt = time.perf_counter() - t0
    return (torch.cat(gathered, dim=0) if rank == 0 else None), dt


def _worker(rank: int, world: int, port: int, out: dict):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    C, dt = distributed_matmul()
    if rank == 0:
        A, B = make_inputs()
        ref = A @ B
        out["ok"] = bool(torch.allclose(C, ref, rtol=1e-5, atol=1e-5))
        out["max_rel"] = float(((C - ref).abs() / ref.abs().clamp_min(1e-6)).max())
        out["seconds"] = dt
    dist.destroy_process_group()


def run(world: int = 2) -> dict:
    import multiprocessing as mp

    from ..parallel.launch import free_port

    ctx = mp.get_context("spawn")
    mgr = ctx.Manager()
    out = mgr.dict()
    port = free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    return dict(out)


if __name__ == "__main__":
    print(run(2))
