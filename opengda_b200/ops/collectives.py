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
    "twoshot", "nvls" or "auto" (one-shot <= 256 KiB, NVLS when available on more than two
    ranks below 512 MiB, else two-shot).

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
        # NVLS moves 1/n of the data per GPU; with two ranks it saves nothing over two-shot.
        # Measured at 8 GPUs: NVLS leads up to 256 MiB (724 GB/s bus bandwidth there) and falls
        # behind two-shot at 1 GiB (588 against 646 GB/s).
        if self.rt.multicast_supported and self.n > 2 and nbytes < (512 << 20):
            return NVLS
        return TWOSHOT

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


class _Collective:
    """Shared state of the symmetric-buffer collectives: flag area, call counter (host or,
    with graph_safe, device-resident) and the capture guard."""

    MAX_BLOCKS = 1024

    def __init__(self, rt, graph_safe: bool):
        self.rt = rt
        self.n, self.me = rt.size, rt.rank
        off = rt.signal_alloc(2 * self.MAX_BLOCKS * self.n)
        self.flags = [rt.signal_peer(p, off) for p in range(self.n)]
        self.epoch = 0
        self.graph_safe = graph_safe
        self._dev_words = torch.zeros(2, dtype=torch.int64, device="cuda") if graph_safe else None

    def _next(self, name: str):
        if self.graph_safe:
            dev = self._dev_words.data_ptr()
            return dev, dev + 8
        if torch.cuda.is_current_stream_capturing():
            raise RuntimeError(f"{name}: capturing a call in a CUDA graph needs graph_safe=True")
        self.epoch += 1
        return 0, 0


class ReduceScatter(_Collective):
    """Reduce-scatter of bf16 vectors: write up to ``max_count`` elements into
    ``input(count)`` (symmetric), call; rank r gets chunk r of the sum (count / n elements,
    scaled, bf16 or f32) in ``output(count)``.  NVLS (sum inside the switch) when the node
    has it, else every rank's input is read over NVLink.  ``graph_safe`` as for Allreduce."""

    def __init__(self, rt, max_count: int, out_dtype: torch.dtype = torch.bfloat16, graph_safe: bool = False):
        super().__init__(rt, graph_safe)
        q = 8 * self.n
        self.max_count = (max_count + q - 1) // q * q
        self.nvls = bool(rt.multicast_supported and self.n > 1)
        self.inp = rt.alloc_tensor((self.max_count,), torch.bfloat16, multicast=self.nvls)
        self.out = torch.empty(self.max_count // self.n, dtype=out_dtype, device=self.inp.local.device)
        self.out_dtype = out_dtype
        self.in_ptrs = [self.inp.ptr(p) for p in range(self.n)]

    def input(self, count: Optional[int] = None) -> torch.Tensor:
        return self.inp.local[: (count or self.max_count)]

    def output(self, count: Optional[int] = None) -> torch.Tensor:
        return self.out[: (count or self.max_count) // self.n]

    def __call__(self, count: int, scale: float = 1.0, blocks: int = 0, nvls: Optional[bool] = None) -> torch.Tensor:
        if count % (8 * self.n) or count > self.max_count:
            raise ValueError("count must be a multiple of 8 * ranks and <= max_count")
        use_nvls = self.nvls if nvls is None else bool(nvls)
        if use_nvls and not self.nvls:
            raise RuntimeError("NVLS reduce-scatter needs multicast support")
        dev, tick = self._next("ReduceScatter")
        native().k_reduce_scatter_bf16(use_nvls, self.in_ptrs, self.inp.mc_ptr if use_nvls else 0,
                                       self.out.data_ptr(), self.n, self.me, count, float(scale),
                                       self.out_dtype == torch.float32, self.flags, self.MAX_BLOCKS, self.epoch,
                                       self.rt.timeout_ns, blocks, dev, tick)
        return self.output(count)


class AllGather(_Collective):
    """All-gather: write this rank's shard (up to ``max_shard_bytes``, a multiple of 16)
    into ``shard(nbytes)``, call; every rank's ``output(nbytes)`` then holds all shards in
    rank order (n * nbytes bytes, symmetric).  NVLS multicast stores when the node has them,
    else one store per rank.  ``graph_safe`` as for Allreduce."""

    def __init__(self, rt, max_shard_bytes: int, graph_safe: bool = False):
        super().__init__(rt, graph_safe)
        self.max_shard_bytes = (max_shard_bytes + 15) // 16 * 16
        self.nvls = bool(rt.multicast_supported and self.n > 1)
        self.out = rt.alloc_tensor((self.n * self.max_shard_bytes,), torch.uint8, multicast=self.nvls)
        self._shard = torch.empty(self.max_shard_bytes, dtype=torch.uint8, device=self.out.local.device)
        self.out_ptrs = [self.out.ptr(p) for p in range(self.n)]

    def shard(self, nbytes: Optional[int] = None) -> torch.Tensor:
        return self._shard[: (nbytes or self.max_shard_bytes)]

    def output(self, nbytes: Optional[int] = None) -> torch.Tensor:
        """[n, nbytes]: row r is rank r's shard (the gathered bytes are contiguous)."""
        b = nbytes or self.max_shard_bytes
        return self.out.local[: self.n * b].view(self.n, b)

    def __call__(self, nbytes: int, blocks: int = 0, nvls: Optional[bool] = None) -> torch.Tensor:
        if nbytes % 16 or nbytes > self.max_shard_bytes:
            raise ValueError("nbytes must be a multiple of 16 and <= max_shard_bytes")
        use_nvls = self.nvls if nvls is None else bool(nvls)
        if use_nvls and not self.nvls:
            raise RuntimeError("NVLS all-gather needs multicast support")
        dev, tick = self._next("AllGather")
        native().k_all_gather(use_nvls, self._shard.data_ptr(), self.out_ptrs, self.out.mc_ptr if use_nvls else 0,
                              self.n, self.me, nbytes, self.flags, self.MAX_BLOCKS, self.epoch, self.rt.timeout_ns,
                              blocks, dev, tick)
        return self.output(nbytes)
