"""Collectives over the NVLink runtime: grid copy (put/get), multi-source reduction and
allreduce (one-shot / two-shot / NVLS) fused with scale + cast (csrc/kernels/collectives.cu).
"""
from __future__ import annotations

from typing import List, Optional, Sequence

import torch

from .. import native

ONESHOT, TWOSHOT, NVLS = 0, 1, 2
ALGOS = {"oneshot": ONESHOT, "twoshot": TWOSHOT, "nvls": NVLS}


def copy(dst_ptr: int, src_ptr: int, nbytes: int, iters: int = 1, blocks: int = 0, threads: int = 0) -> None:
    """Grid-wide copy (either side may be a peer's memory); ends with fence.acq_rel.sys."""
    native().k_copy(int(dst_ptr), int(src_ptr), int(nbytes), iters, blocks, threads)


def reduce_sum(out: torch.Tensor, src_ptrs: Sequence[int], count: int, scale: float = 1.0) -> torch.Tensor:
    """out[:count] = scale * sum of bf16 vectors at src_ptrs (local or peer memory)."""
    native().k_reduce_bf16([int(p) for p in src_ptrs], out.data_ptr(), int(count), float(scale),
                           out.dtype == torch.float32)
    return out


class Allreduce:
    """Allreduce of bf16 vectors of up to ``max_count`` elements across all ranks.

    ``inp`` is a symmetric bf16 buffer (write the data into ``allreduce.input(count)``),
    the result goes to a symmetric output buffer (bf16 or f32).  ``algo``: "oneshot",
    "twoshot", "nvls" or "auto" (one-shot <= 256 KiB, NVLS when available, else two-shot).

    ``graph_safe=True`` keeps the call counter on the device (each kernel reads it and its
    last CTA advances it), so calls can be captured in a CUDA graph (``torch.cuda.graph``)
    and replayed; every rank must replay the same calls in the same order.  Without it the
    host passes the counter, and capturing a call is refused (a replay would reuse it).
    """

    MAX_BLOCKS = 1024

    def __init__(self, rt, max_count: int, out_dtype: torch.dtype = torch.bfloat16, graph_safe: bool = False):
        self.rt = rt
        self.n, self.me = rt.size, rt.rank
        self.max_count = (max_count + 7) // 8 * 8
        mc = rt.multicast_supported
        self.inp = rt.alloc_tensor((self.max_count,), torch.bfloat16, multicast=mc)
        self.out = rt.alloc_tensor((self.max_count,), out_dtype, multicast=mc)
        self.out_dtype = out_dtype
        off = rt.signal_alloc(2 * self.MAX_BLOCKS * self.n)
        self.flags = [rt.signal_peer(p, off) for p in range(self.n)]
        self.epoch = 0
        self.in_ptrs = [self.inp.ptr(p) for p in range(self.n)]
        self.out_ptrs = [self.out.ptr(p) for p in range(self.n)]
        self.graph_safe = graph_safe
        if graph_safe:  # [0] epoch (u64), [1] low half: the CTA ticket (u32)
            self._dev_words = torch.zeros(2, dtype=torch.int64, device=self.inp.local.device)

    def input(self, count: Optional[int] = None) -> torch.Tensor:
        return self.inp.local[: (count or self.max_count)]

    def output(self, count: Optional[int] = None) -> torch.Tensor:
        return self.out.local[: (count or self.max_count)]

    def pick(self, count: int) -> int:
        nbytes = count * 2
        if nbytes <= 256 * 1024 or self.n == 1:
            return ONESHOT
        # NVLS moves 1/n of the data per GPU; with two ranks it saves nothing over two-shot
        return NVLS if (self.rt.multicast_supported and self.n > 2) else TWOSHOT

    def __call__(self, count: int, algo: str = "auto", scale: float = 1.0, blocks: int = 0) -> torch.Tensor:
        if count % 8 or count > self.max_count:
            raise ValueError("count must be a multiple of 8 and <= max_count")
        a = self.pick(count) if algo == "auto" else ALGOS[algo]
        if a == NVLS and not self.rt.multicast_supported:
            raise RuntimeError("NVLS allreduce needs multicast support")
        dev = tick = 0
        if self.graph_safe:
            dev = self._dev_words.data_ptr()
            tick = dev + 8
        elif torch.cuda.is_current_stream_capturing():
            raise RuntimeError("Allreduce: capturing a call in a CUDA graph needs Allreduce(..., graph_safe=True)")
        self.epoch += 1
        native().k_allreduce_bf16(a, self.in_ptrs, self.out_ptrs, self.inp.mc_ptr if a == NVLS else 0,
                                  self.out.mc_ptr if a == NVLS else 0, self.n, self.me, count, float(scale),
                                  self.out_dtype == torch.float32, self.flags, self.MAX_BLOCKS, self.epoch,
                                  self.rt.timeout_ns, blocks, dev, tick)
        return self.output(count)
