"""NCCL + PyTorch MoE layer: the comparison arm for the MoE layer.

Routing with torch softmax/top-k, dispatch with ``all_to_all_single`` (variable splits),
one cuBLAS matmul pair per local expert, combine with ``all_to_all_single`` and a
gate-weighted sum on the source rank.  Same math and weights as
``opengda_b200.models.moe.MoELayer``; no code of this framework on its path.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


class NcclMoE:
    def __init__(self, layer):
        """Share the weights of a MoELayer (w_gate, w_up [El, I, H]; w2 [El, H, I])."""
        self.T, self.H, self.E, self.topk, self.I = layer.T, layer.H, layer.E, layer.topk, layer.I
        self.n = dist.get_world_size() if dist.is_initialized() else 1
        self.El = self.E // self.n
        self.w_gate, self.w_up, self.w2 = layer.w_gate, layer.w_up, layer.w2

    def forward(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        T, k, El, n = self.T, self.topk, self.El, self.n
        prob = torch.softmax(logits, dim=-1)
        w, idx = torch.topk(prob, k, dim=-1)
        flat = idx.flatten()
        order = torch.argsort(flat, stable=True)  # by global expert => by destination rank
        tok = order // k
        send = x[tok]
        counts = torch.bincount(flat, minlength=self.E)
        send_split = counts.view(n, El).sum(1)
        if n > 1:
            recv_counts = torch.empty_like(counts)
            dist.all_to_all_single(recv_counts, counts)
            recv_split = recv_counts.view(n, El).sum(1)
            rs, ss = recv_split.tolist(), send_split.tolist()
            recv = torch.empty(sum(rs), self.H, dtype=x.dtype, device=x.device)
            dist.all_to_all_single(recv, send, rs, ss)
            per_src = recv_counts.view(n, El)
        else:
            recv, per_src, rs, ss = send, counts.view(1, El), [send.shape[0]], [send.shape[0]]
        # rows arrive grouped by source, then by local expert: regroup per expert
        pcl = per_src.tolist()
        chunks = [[] for _ in range(El)]
        pos = 0
        for s in range(n):
            for e in range(El):
                c = pcl[s][e]
                chunks[e].append((pos, c))
                pos += c
        out_rows = torch.empty_like(recv)
        for e in range(El):
            idxs = [torch.arange(p, p + c, device=x.device) for p, c in chunks[e] if c]
            if not idxs:
                continue
            ii = torch.cat(idxs)
            xe = recv[ii]
            act = F.silu(xe @ self.w_gate[e].t()) * (xe @ self.w_up[e].t())
            out_rows[ii] = act @ self.w2[e].t()
        if n > 1:
            back = torch.empty_like(send)
            dist.all_to_all_single(back, out_rows, ss, rs)
        else:
            back = out_rows
        y = torch.zeros(T * k, self.H, dtype=torch.float32, device=x.device)
        y[order] = back.float()
        y = (y.view(T, k, self.H) * w.unsqueeze(-1)).sum(1)
        return y.to(x.dtype)

    def dispatch_combine(self, x: torch.Tensor, logits: torch.Tensor) -> torch.Tensor:
        """The all-to-all round trip alone (identity experts): route, all_to_all_single of the
        rows to their owners and back, gate-weighted sum on the source."""
        T, k, El, n = self.T, self.topk, self.El, self.n
        prob = torch.softmax(logits, dim=-1)
        w, idx = torch.topk(prob, k, dim=-1)
        flat = idx.flatten()
        order = torch.argsort(flat, stable=True)
        send = x[order // k]
        counts = torch.bincount(flat, minlength=self.E)
        if n > 1:
            recv_counts = torch.empty_like(counts)
            dist.all_to_all_single(recv_counts, counts)
            ss, rs = counts.view(n, El).sum(1).tolist(), recv_counts.view(n, El).sum(1).tolist()
            recv = torch.empty(sum(rs), self.H, dtype=x.dtype, device=x.device)
            dist.all_to_all_single(recv, send, rs, ss)
            back = torch.empty_like(send)
            dist.all_to_all_single(back, recv, ss, rs)
        else:
            back = send
        y = torch.zeros(T * k, self.H, dtype=torch.float32, device=x.device)
        y[order] = back.float()
        return (y.view(T, k, self.H) * w.unsqueeze(-1)).sum(1).to(x.dtype)

    __call__ = forward
