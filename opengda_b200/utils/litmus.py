"""Memory-model litmus tests (message passing, store buffering) of the flag protocols,
on one GPU (the two roles as two CTAs of one launch) or across two GPUs (rank 0 and rank
1, words reached through the NVLink peer mapping).  The protocol code is
``csrc/include/gicc/proto/litmus.hpp``; the CPU-rank version of the same code runs in the
CPU test-suite.

``run(test, ...)`` returns, on every rank that took part, a dict with ``status`` (0 = ok,
1 = a wait timed out), and for MP ``violations`` (the reader saw the new flag with old
data: forbidden), for SB ``outcomes`` -- the counts of the four (side 0, side 1) load
results; (0, 0) is forbidden with the fence and allowed without it.
"""
from __future__ import annotations

from typing import Optional

import torch

MP, SB = 0, 1


def region_words(k: int, iters: int) -> int:
    return 2 + k + 2 * iters + 2  # ready, flag, data[k], W[iters], out[iters], result[2]


def _offsets(k: int, iters: int) -> dict:
    return {"ready": 0, "flag": 1, "data": 2, "W": 2 + k, "out": 2 + k + iters, "result": 2 + k + 2 * iters}


def _role_ptrs(test: int, r: int, mine: int, other: int, k: int, iters: int) -> list:
    o = _offsets(k, iters)
    w = lambda base, name: base + 8 * o[name]  # noqa: E731
    if test == MP:
        tgt = other if r == 0 else mine  # the writer stores into the reader's words
        return [w(tgt, "data"), w(tgt, "flag"), 0, 0, 0, 0, 0, w(mine, "result")]
    return [0, 0, w(other, "ready"), w(mine, "ready"), w(other, "W"), w(mine, "W"), w(mine, "out"), w(mine, "result")]


def _summary(test: int, res: torch.Tensor, outs) -> dict:
    d = {"status": int(res[0].item())}
    if test == MP:
        d["violations"] = int(res[1].item())
    else:
        a, b = outs
        d["outcomes"] = {f"{x}{y}": int(((a == x) & (b == y)).sum().item()) for x in (0, 1) for y in (0, 1)}
    return d


def run(test: int, iters: int = 20000, k: int = 64, use_fence: bool = True, seed: int = 1, max_delay: int = 256,
        rt=None, timeout_ns: Optional[int] = None) -> Optional[dict]:
    from .. import native

    n = native()
    timeout_ns = timeout_ns or n.default_timeout_ns()
    words = region_words(k, iters)
    o = _offsets(k, iters)
    if rt is None or rt.size == 1:
        buf = torch.zeros(2, words, dtype=torch.int64, device="cuda")
        base = [buf[0].data_ptr(), buf[1].data_ptr()]
        roles = [_role_ptrs(test, r, base[r], base[1 - r], k, iters) for r in range(2)]
        n.k_litmus(test, iters, k, int(use_fence), seed, max_delay, timeout_ns, 0, 2, roles)
        torch.cuda.synchronize()
        res = buf[1, o["result"]:o["result"] + 2] if test == MP else buf[0, o["result"]:o["result"] + 2]
        st = int(max(buf[0, o["result"]].item(), buf[1, o["result"]].item()))
        outs = (buf[0, o["out"]:o["out"] + iters], buf[1, o["out"]:o["out"] + iters])
        d = _summary(test, res, outs)
        d["status"] = st
        return d
    # two GPUs: ranks 0 and 1 play the roles; every rank allocates (collective).  Results
    # are gathered through the bootstrap (host bytes), not by reading peer memory.
    sym = rt.alloc_tensor((words,), torch.int64)
    me = rt.rank
    rt.barrier()
    mine = None
    if me < 2:
        other = 1 - me
        roles = [[0] * 8, [0] * 8]
        roles[me] = _role_ptrs(test, me, sym.ptr(), sym.ptr(other), k, iters)
        n.k_litmus(test, iters, k, int(use_fence), seed, max_delay, timeout_ns, me, 1, roles)
        torch.cuda.synchronize()
        mine = sym.local.cpu()
    rt.barrier()
    allv = rt.boot.allgather_obj(mine.numpy().tobytes() if mine is not None else b"")
    out = None
    if me == 0:
        r0 = torch.frombuffer(bytearray(allv[0]), dtype=torch.int64)
        r1 = torch.frombuffer(bytearray(allv[1]), dtype=torch.int64)
        st = int(max(r0[o["result"]].item(), r1[o["result"]].item()))
        res = r1[o["result"]:o["result"] + 2] if test == MP else r0[o["result"]:o["result"] + 2]
        outs = (r0[o["out"]:o["out"] + iters], r1[o["out"]:o["out"] + iters])
        out = _summary(test, res, outs)
        out["status"] = st
    return out
