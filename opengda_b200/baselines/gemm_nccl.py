"""NCCL + cuBLAS distributed GEMM: the comparison arm for the 16384^3 distributed GEMM.

* ``ag``: ``all_gather_into_tensor`` of the A row shards, then ``torch.matmul`` (cuBLAS)
  with the local column shard of B -- the unfused all-gather -> GEMM.
* ``rs``: ``torch.matmul`` of the local K shards (full M x N partial), then
  ``reduce_scatter_tensor`` by rows -- the unfused GEMM -> reduce-scatter.

Same shapes, layouts (B stored as B^T rows) and call signature as
``opengda_b200.models.dist_gemm.DistGemm``; no code of this framework on its path.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.distributed as dist


class NcclDistGemm:
    def __init__(self, M: int, N: int, K: int, mode: str = "ag", device: Optional[torch.device] = None):
        self.M, self.N, self.K, self.mode = M, N, K, mode
        self.world = dist.get_world_size() if dist.is_initialized() else 1
        self.rank = dist.get_rank() if dist.is_initialized() else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        w = self.world
        self.launches_per_step = 0  # library kernels only
        if mode == "ag":
            self.A_full = torch.empty(M, K, dtype=torch.bfloat16, device=self.device)
            self.C = torch.empty(M, N // w, dtype=torch.bfloat16, device=self.device)
        else:
            self.P = torch.empty(M, N, dtype=torch.bfloat16, device=self.device)
            self.C = torch.empty(M // w, N, dtype=torch.bfloat16, device=self.device)

    def a_slot(self, parity=None):
        return None

    def forward(self, A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        C = out if out is not None else self.C
        if self.world == 1:
            return torch.matmul(A, B.t(), out=C)
        if self.mode == "ag":
            dist.all_gather_into_tensor(self.A_full, A)
            return torch.matmul(self.A_full, B.t(), out=C)
        torch.matmul(A, B.t(), out=self.P)
        dist.reduce_scatter_tensor(C, self.P)
        return C

    __call__ = forward
