"""NCCL + cuBLAS ring-stripe fp32 matmul: the comparison arm of
``opengda_b200.models.ring_mm.RingMatmul`` and the host-driven ring of the reference's
examples/mm_hip_mpi.cpp:150-184 (send the held B stripe right, receive the next one from the
left, multiply, repeat), restated over NCCL point-to-point because MPI is absent.

Each step posts the send/receive pair (``batch_isend_irecv``) and then multiplies the held
stripe with ``torch.matmul`` (fp32, TF32 off), so the transfer overlaps the multiply as in the
reference's non-blocking send; the step ends when both are done.  Same stripes, layouts and
result as ``RingMatmul``; no code of this framework on its path.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


class NcclRingMatmul:
    def __init__(self, N: int, device: Optional[torch.device] = None):
        self.n = dist.get_world_size() if dist.is_initialized() else 1
        self.r = dist.get_rank() if dist.is_initialized() else 0
        if N % self.n:
            raise ValueError("N must be divisible by the number of ranks")
        self.N, self.Ns = N, N // self.n
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        self.buf = [torch.empty(N, self.Ns, dtype=torch.float32, device=self.device) for _ in range(2)]
        self.launches_per_call = 0  # library kernels only

    def forward(self, A_s: torch.Tensor, B_s: torch.Tensor, C_s: Optional[torch.Tensor] = None) -> torch.Tensor:
        N, Ns, n, r = self.N, self.Ns, self.n, self.r
        if C_s is None:
            C_s = torch.empty(Ns, N, dtype=torch.float32, device=self.device)
        prev_tf32 = torch.backends.cuda.matmul.allow_tf32
        torch.backends.cuda.matmul.allow_tf32 = False
        try:
            cur = B_s
            for s in range(n):
                reqs = []
                if s < n - 1:
                    nxt = self.buf[(s + 1) & 1]
                    reqs = dist.batch_isend_irecv([dist.P2POp(dist.isend, cur, (r + 1) % n),
                                                   dist.P2POp(dist.irecv, nxt, (r - 1) % n)])
                b = (r - s) % n
                C_s[:, b * Ns:(b + 1) * Ns] = torch.matmul(A_s, cur)
                for q in reqs:
                    q.wait()
                if s < n - 1:
                    cur = nxt
        finally:
            torch.backends.cuda.matmul.allow_tf32 = prev_tf32
        return C_s

    __call__ = forward
