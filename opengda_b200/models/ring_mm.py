"""Ring-stripe fp32 matrix multiply: the reference's distributed-matmul example
(examples/gicc/mm.cu:116-225) as an API-level workload of this runtime.

Every rank r holds a row stripe A_r [Ns, N] of A, a column stripe B_r [N, Ns] of B, and
computes its row stripe C_r = A_r . B [Ns, N] in n steps.  In step s it holds the B stripe of
rank (r - s) mod n, writes that column block of C_r, and forwards the stripe to its right
neighbour's landing buffer for step s + 1.  One kernel per step does both (``k_ring_mm_step``:
a few CTAs push the stripe with 16-byte NVLink stores while the others run an fp32 SIMT
SGEMM); the landing buffers alternate, and a neighbour overwrites one only after the rank
that reads it reported the step that last read it.  Counters are monotonic across calls, so
nothing is reset between calls.

With ``tensor_cores=True`` (the default when N % 32 == 0) the step kernel's other CTAs write
the held stripe transposed as its tf32 parts (hi, lo, hi) instead, and the column block is
one kind::tf32 tcgen05 GEMM over 3N with A_s's parts (hi, hi, lo) (``ops.gemm.gemm_fp32``'s
method: fp32 data, error about 2^-21 of |A||B| per term); ``tensor_cores=False`` keeps the
fp32 SIMT SGEMM.  The bf16 tensor-core version of this workload at scale is ``DistGemm``
(all-gather fused into the GEMM); this one keeps the reference's fp32 data and ring structure
and is checked against a CPU oracle.  ``opengda_b200.baselines.ring_mm_nccl`` runs the same ring with NCCL
send/recv and cuBLAS.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import native
from ..utils.graphs import refuse_capture


class RingMatmul:
    def __init__(self, N: int, rt=None, push_ctas: int = 8, device: Optional[torch.device] = None,
                 tensor_cores: Optional[bool] = None):
        self.rt = rt
        self.n = rt.size if rt is not None else 1
        self.r = rt.rank if rt is not None else 0
        if N % self.n:
            raise ValueError("N must be divisible by the number of ranks")
        self.N, self.Ns = N, N // self.n
        if self.Ns % 64 or N % 16:
            raise ValueError("need N / ranks % 64 == 0 and N % 16 == 0")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.push_ctas = push_ctas if self.n > 1 else 0
        self.tensor_cores = (N % 32 == 0) if tensor_cores is None else bool(tensor_cores)
        if self.tensor_cores:
            if N % 32:
                raise ValueError("tensor_cores needs N % 32 == 0")
            # A_s's tf32 parts (hi, hi, lo) and two buffers for the held stripe's (hi, lo, hi)
            self.a_split = torch.empty(self.Ns, 3 * N, dtype=torch.float32, device=self.device)
            self.b_split = [torch.empty(self.Ns, 3 * N, dtype=torch.float32, device=self.device) for _ in range(2)]
            self.grid = native().ring_mm_grid_tc(self.push_ctas)
        else:
            self.grid = native().ring_mm_grid(self.Ns, self.push_ctas)
        self.steps_done = 0  # this rank's steps over all calls
        self.calls = 0
        if self.n > 1:
            self.land = [rt.alloc_tensor((N, self.Ns), torch.float32, exchange=False) for _ in range(2)]
            rt.exchange()
            w = rt.signal_alloc(2)  # [0] stripes arrived here (x push_ctas), [1] steps the right rank finished
            self.w_arrivals, self.w_consumed = w, w + 1
            self.ticket = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.launches_per_call = self.n * (2 if self.tensor_cores else 1) + (1 if self.tensor_cores else 0)

    def forward(self, A_s: torch.Tensor, B_s: torch.Tensor, C_s: Optional[torch.Tensor] = None) -> torch.Tensor:
        """A_s [Ns, N] and B_s [N, Ns] fp32 (this rank's stripes) -> C_s [Ns, N] = A_s . B."""
        N, Ns, n, r = self.N, self.Ns, self.n, self.r
        if n > 1:
            refuse_capture("RingMatmul")
        assert A_s.shape == (Ns, N) and A_s.dtype == torch.float32 and A_s.is_contiguous()
        assert B_s.shape == (N, Ns) and B_s.dtype == torch.float32 and B_s.is_contiguous()
        if C_s is None:
            C_s = torch.empty(Ns, N, dtype=torch.float32, device=self.device)
        self.calls += 1
        left, right = (r - 1) % n, (r + 1) % n
        if self.tensor_cores:
            native().tf32_split(A_s.data_ptr(), N, Ns, N, self.a_split.data_ptr(), 0)
        for s in range(n):
            p = ring_step_plan(n, r, self.calls, s, self.push_ctas, self.steps_done, self.grid)
            d = {"N": N, "Ns": Ns, "A": A_s.data_ptr(), "C": C_s.data_ptr(), "col_block": p["col_block"],
                 "push_ctas": self.push_ctas, "rank": r, "left": left, "right": right}
            if self.tensor_cores:
                d["Asplit"] = self.a_split.data_ptr()
                d["Bsplit"] = self.b_split[s & 1].data_ptr()
            if n == 1:
                d["Bcur"] = B_s.data_ptr()
            else:
                rt = self.rt
                d["timeout_ns"] = rt.timeout_ns
                d["Bcur"] = B_s.data_ptr() if p["read"] is None else self.land[p["read"]].ptr(r)
                if p["arrivals_target"] is not None:
                    d["arrivals"] = rt.signal_local(self.w_arrivals)
                    d["arrivals_target"] = p["arrivals_target"]
                if p["push"] is not None:
                    d["Bnext_remote"] = self.land[p["push"]].ptr(right)
                    d["arrivals_remote"] = rt.signal_peer(right, self.w_arrivals)
                    d["consumed"] = rt.signal_local(self.w_consumed)
                    d["consumed_target"] = p["consumed_target"]
                d["consumed_left"] = rt.signal_peer(left, self.w_consumed)
                d["ticket"] = self.ticket.data_ptr()
                d["ticket_target"] = p["ticket_target"]
            native().k_ring_mm_step(d)
            self.steps_done += 1
        return C_s

    __call__ = forward

    def flops(self) -> float:
        """Whole-job FLOPs of one call (2 N^3)."""
        return 2.0 * self.N ** 3


def ring_step_plan(n: int, r: int, call: int, s: int, push_ctas: int, steps_done: int, grid: int) -> dict:
    """What rank r does in step s of its call-th call (1-based) of an n-rank ring:

    * ``col_block``: the stripe it holds, (r - s) mod n;
    * ``read``: the landing buffer it reads (None: its own stripe, step 0);
    * ``arrivals_target``: the value its arrival word must reach first (None: no wait) --
      the left rank adds push_ctas per forwarded stripe, n - 1 of them per call;
    * ``push``: the right rank's landing buffer it forwards into (None: last step);
    * ``consumed_target``: the steps the right rank must have finished before that push
      (all of its steps before its own step s, so the buffer's last reader is done);
    * ``ticket_target``: (steps_done + 1) * grid, reached by the last CTA of the step.
    """
    return {
        "col_block": (r - s) % n,
        "read": None if s == 0 else s & 1,
        "arrivals_target": None if s == 0 else ((call - 1) * (n - 1) + s) * push_ctas,
        "push": None if s == n - 1 else (s + 1) & 1,
        "consumed_target": None if s == n - 1 else (call - 1) * n + s,
        "ticket_target": (steps_done + 1) * grid,
    }


def make_stripes(N: int, n: int, r: int, seed: int = 0, device="cuda"):
    """Rank r's stripes of A, B ~ uniform[-1, 1) from `seed` (the full matrices are the same
    on every rank): A_r = A[r*Ns:(r+1)*Ns, :], B_r = B[:, r*Ns:(r+1)*Ns]."""
    g = torch.Generator().manual_seed(seed)
    A = torch.rand(N, N, generator=g) * 2 - 1
    B = torch.rand(N, N, generator=g) * 2 - 1
    Ns = N // n
    A_r = A[r * Ns:(r + 1) * Ns].contiguous()
    B_r = B[:, r * Ns:(r + 1) * Ns].contiguous()
    return A_r.to(device), B_r.to(device), A, B
