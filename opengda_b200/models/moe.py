"""Expert-parallel MoE layer (4096 tokens per GPU, hidden 7168, 256 experts, top-8) over the NVLink runtime.

tokens T per GPU, hidden H, E experts split evenly over the ranks (E/n local experts),
top-k routing with softmax gates (the softmax probability of each selected expert, not
renormalised), SwiGLU experts with intermediate size I:

    y[t] = sum_j  w[t,j] * W2_e (silu(W_gate,e x_t) * (W_up,e x_t)),   e = topk[t, j]

The forward pass is six kernels (csrc/kernels/moe.cu): routing, a one-CTA plan that
exchanges per-expert counts over NVLink, a send-list sort, grouped GEMM 1 whose
communication warps perform the dispatch all-to-all while the tensor cores work
(SwiGLU in the epilogue), grouped GEMM 2 whose epilogue pushes gate-weighted rows back
to their source GPU (the combine all-to-all), and the per-token top-k sum.

W1 of an expert is stored as [2I, H] with gate and up rows interleaved in blocks of 128
(rows [256 b, 256 b + 128) = gate rows [128 b, 128 b + 128), the next 128 = up rows), so
one 256-wide output tile holds matching gate and up columns.
"""
from __future__ import annotations

from typing import Optional

import torch

from .. import native
from ..utils.graphs import refuse_capture


def interleave_w1(w_gate: torch.Tensor, w_up: torch.Tensor) -> torch.Tensor:
    """[E, I, H] gate and up -> [E, 2I, H] with 128-row blocks interleaved."""
    E, I, H = w_gate.shape
    g = w_gate.view(E, I // 128, 128, H)
    u = w_up.view(E, I // 128, 128, H)
    return torch.stack([g, u], dim=2).reshape(E, 2 * I, H)


class MoELayer:
    def __init__(self, T: int, H: int, E: int, topk: int, I: int, rt=None, seed: int = 4,
                 device: Optional[torch.device] = None, weight_std: float = 0.02):
        self.T, self.H, self.E, self.topk, self.I = T, H, E, topk, I
        self.rt = rt
        self.n = rt.size if rt is not None else 1
        self.r = rt.rank if rt is not None else 0
        if E % self.n:
            raise ValueError("experts must split evenly over the ranks")
        self.El = E // self.n
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        n, El = self.n, self.El
        # expert weights of this rank (global experts r*El ... r*El+El-1), N(0, std) from seed
        g = torch.Generator(device=dev).manual_seed(seed * 1000 + self.r)
        w_gate = (torch.randn(El, I, H, generator=g, device=dev) * weight_std).to(torch.bfloat16)
        w_up = (torch.randn(El, I, H, generator=g, device=dev) * weight_std).to(torch.bfloat16)
        self.w2 = (torch.randn(El, H, I, generator=g, device=dev) * weight_std).to(torch.bfloat16)
        self.w1 = interleave_w1(w_gate, w_up).contiguous()
        self.w_gate, self.w_up = w_gate, w_up  # kept for the reference check
        # receive capacity: every source may send each token to <= min(topk, El) local experts
        self.cap = n * T * min(topk, El) + El * 128
        pairs = T * topk
        if rt is not None:
            self.count_tab = [rt.alloc_tensor((n, E), torch.int32, exchange=False) for _ in range(2)]
            self.recv = [rt.alloc_tensor((self.cap, H), torch.bfloat16, exchange=False) for _ in range(2)]
            self.meta = [rt.alloc_tensor((self.cap, 4), torch.int32, exchange=False) for _ in range(2)]
            self.comb = rt.alloc_tensor((pairs, H), torch.bfloat16, exchange=False)
            rt.exchange()
            off = rt.signal_alloc(n + n * El + 1)
            self.plan_flags = [rt.signal_peer(p, off) for p in range(n)]
            self.arrivals = [rt.signal_peer(p, off + n) for p in range(n)]
            self.comb_arrivals = [rt.signal_peer(p, off + n + n * El) for p in range(n)]
            ptr = lambda sym, q: sym.ptr(q)  # noqa: E731
        else:
            mk = lambda shape, dt: torch.zeros(shape, dtype=dt, device=dev)  # noqa: E731
            self.count_tab = [mk((1, E), torch.int32) for _ in range(2)]
            self.recv = [mk((self.cap, H), torch.bfloat16) for _ in range(2)]
            self.meta = [mk((self.cap, 4), torch.int32) for _ in range(2)]
            self.comb = mk((pairs, H), torch.bfloat16)
            self._words = torch.zeros(1 + El + 1, dtype=torch.int64, device=dev)
            base = self._words.data_ptr()
            self.plan_flags = [base]
            self.arrivals = [base + 8]
            self.comb_arrivals = [base + 8 * (1 + El)]
            ptr = lambda t, q: t.data_ptr()  # noqa: E731
        self._ptr = ptr
        i32 = lambda k: torch.zeros(k, dtype=torch.int32, device=dev)  # noqa: E731
        self.ws_t = {
            "dest_row_base": i32(E), "key_base": i32(El * n + 1), "key_cursor": i32(El * n),
            "expert_base": i32(El), "expert_rows": i32(El), "mblk_prefix": i32(El + 1),
            "cum_rows": torch.zeros(n * El, dtype=torch.int64, device=dev),
            "cum_pairs": torch.zeros(1, dtype=torch.int64, device=dev),
            "send_pair": i32(pairs), "send_row": i32(pairs),
            "g1_tile_ctr": torch.zeros(2, dtype=torch.int64, device=dev),
            "g2_ctr": torch.zeros(6, dtype=torch.int64, device=dev),
            "g2_queue": torch.zeros(self.cap // 128 * (H // 256), dtype=torch.int64, device=dev),
        }
        # CTAs whose communication warps run the dispatch all-to-all (0 = every CTA).  With
        # fewer, the first grouped GEMM takes its tiles dynamically so those CTAs do less math.
        self.dispatch_ctas = 0
        # CTAs that push the second GEMM's rows back to the sources (0 = every CTA pushes its
        # own tiles from the epilogue).  With fewer, the rows are staged in local HBM
        # (self.y_stage, [cap, H] bf16, allocated on first use) and queued for those CTAs.
        # Default: staged with 64 pushing CTAs at 8 or more ranks, where 7/8 of the rows leave
        # the GPU (8 GPUs: 5.00 ms per layer against 5.49 ms with epilogue pushes).
        self.combine_ctas = 64 if n >= 8 else 0
        self.y_stage = None
        self.topk_idx = i32(pairs)
        self.topk_w = torch.zeros(pairs, dtype=torch.float32, device=dev)
        self.counts = i32(E)
        self.h = torch.empty(self.cap, I, dtype=torch.bfloat16, device=dev)
        self.out = torch.empty(T, H, dtype=torch.bfloat16, device=dev)
        self.epoch = 0
        self.launches_per_step = 7  # memset + route + plan + sort + gemm1 + gemm2 + combine

    STAGES = ("route", "plan", "sort", "gemm1+dispatch", "gemm2+combine_push", "combine")
    COMM_STAGES = ("route", "plan", "sort", "dispatch", "return", "combine")

    def dispatch_combine(self, x: torch.Tensor, logits: torch.Tensor, stage_times: bool = False) -> torch.Tensor:
        """The all-to-all round trip alone, with identity experts: routing, dispatch of every
        (token, expert) row to its owner, return of the row scaled by its gate, combine.
        Returns y[t] = sum_j w_j * x[t]; the counters advance exactly as in ``forward``."""
        return self.forward(x, logits, stage_times=stage_times, comm_only=True)

    def forward(self, x: torch.Tensor, logits: torch.Tensor, stage_times: bool = False,
                comm_only: bool = False) -> torch.Tensor:
        """x [T, H] bf16, logits [T, E] fp32 -> y [T, H] bf16 (this rank's tokens).
        stage_times=True also records per-kernel device times into ``self.last_stage_ms``
        (synchronises; profiling only)."""
        refuse_capture("MoELayer")
        assert x.shape == (self.T, self.H) and x.dtype == torch.bfloat16 and x.is_contiguous()
        assert logits.shape == (self.T, self.E) and logits.dtype == torch.float32 and logits.is_contiguous()
        self.epoch += 1
        p = self.epoch % 2
        n = self.n
        P = self._ptr
        if self.combine_ctas > 0 and self.y_stage is None:
            self.y_stage = torch.empty(self.cap, self.H, dtype=torch.bfloat16, device=self.h.device)
        d = {
            "n": n, "r": self.r, "T": self.T, "H": self.H, "I": self.I, "E": self.E, "topk": self.topk,
            "logits": logits.data_ptr(), "x": x.data_ptr(), "w1": self.w1.data_ptr(), "w2": self.w2.data_ptr(),
            "topk_idx": self.topk_idx.data_ptr(), "topk_w": self.topk_w.data_ptr(), "counts": self.counts.data_ptr(),
            "count_tab": [P(self.count_tab[p], q) for q in range(n)],
            "plan_flags": self.plan_flags,
            "recv": [P(self.recv[p], q) for q in range(n)],
            "meta": [P(self.meta[p], q) for q in range(n)],
            "arrivals": self.arrivals,
            "h": self.h.data_ptr(),
            "comb": [P(self.comb, q) for q in range(n)],
            "comb_arrivals": self.comb_arrivals,
            "out": self.out.data_ptr(), "cap_rows": self.cap, "epoch": self.epoch,
            "timeout_ns": self.rt.timeout_ns if self.rt is not None else 0,
            "ws": {k: v.data_ptr() for k, v in self.ws_t.items()},
            "stage_times": stage_times,
            "dispatch_ctas": self.dispatch_ctas,
            "combine_ctas": self.combine_ctas,
            "comm_only": int(comm_only),
            "y_stage": self.y_stage.data_ptr() if self.y_stage is not None else 0,
        }
        st = native().k_moe_forward(d)
        if stage_times:
            self.last_stage_ms = dict(zip(self.COMM_STAGES if comm_only else self.STAGES, st))
        return self.out

    __call__ = forward

    def flops(self) -> float:
        """Useful FLOPs of this rank's share: 2*pairs*(H*2I + I*H)."""
        return 2.0 * self.T * self.topk * (self.H * 2 * self.I + self.I * self.H)


def make_inputs(T: int, H: int, E: int, rank: int, seed: int = 4, device=None):
    """Router logits N(0,1) and tokens N(0,1) (bf16) for this rank, from `seed`."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=device).manual_seed(seed * 7919 + rank)
    logits = torch.randn(T, E, generator=g, device=device, dtype=torch.float32)
    x = torch.randn(T, H, generator=g, device=device).to(torch.bfloat16)
    return x, logits


def reference_moe(x, logits, topk, w_gate_all, w_up_all, w2_all, rows=None):
    """fp32 reference on (a subset of) one rank's tokens; weights of ALL experts [E, ...]."""
    xs = x.float() if rows is None else x[rows].float()
    ls = logits if rows is None else logits[rows]
    prob = torch.softmax(ls, dim=-1)
    w, idx = torch.topk(prob, topk, dim=-1)
    out = torch.zeros_like(xs)
    for t in range(xs.shape[0]):
        acc = torch.zeros(xs.shape[1], device=xs.device)
        for j in range(topk):
            e = int(idx[t, j])
            gate = w_gate_all[e].float() @ xs[t]
            up = w_up_all[e].float() @ xs[t]
            act = torch.nn.functional.silu(gate) * up
            acc += w[t, j] * (w2_all[e].float() @ act)
        out[t] = acc
    return out
