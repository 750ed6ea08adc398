"""torch.distributed-style collective calls on ordinary tensors, backed by this package's
NVLink kernels (ops.collectives): ``all_reduce``, ``reduce_scatter_tensor`` and
``all_gather_into_tensor`` with the same argument order as torch.distributed, so a training
loop can switch a call over without restructuring.

The kernels work on symmetric buffers, so each call copies its input into a cached
symmetric buffer of the right size class (a power of two, allocated collectively on first
use) and the result back out.  Every rank must make the same calls in the same order, as
with any collective.  bf16 is the reduction dtype (f32 accumulation inside the kernels);
all-gather moves bytes, so it takes any dtype.
"""
from __future__ import annotations

from typing import Dict, Tuple

import torch

from ..ops.collectives import AllGather, Allreduce, ReduceScatter


def _size_class(n: int, quantum: int) -> int:
    c = quantum
    while c < n:
        c *= 2
    return c


class Collectives:
    """One per process (per Runtime); caches the symmetric buffers per size class."""

    def __init__(self, rt, graph_safe: bool = False):
        self.rt = rt
        self.n = rt.size
        self.graph_safe = graph_safe
        self._ar: Dict[Tuple[int, torch.dtype], Allreduce] = {}
        self._rs: Dict[Tuple[int, torch.dtype], ReduceScatter] = {}
        self._ag: Dict[int, AllGather] = {}

    @staticmethod
    def _check_bf16(t: torch.Tensor, what: str) -> None:
        if t.dtype != torch.bfloat16 or not t.is_cuda:
            raise TypeError(f"{what}: a CUDA bf16 tensor is needed (the reduction kernels sum bf16 in f32)")

    def all_reduce(self, tensor: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        """In place: tensor <- scale * sum over ranks (bf16)."""
        self._check_bf16(tensor, "all_reduce")
        count = tensor.numel()
        padded = _size_class(count, 8)
        key = (padded, tensor.dtype)
        if key not in self._ar:
            self._ar[key] = Allreduce(self.rt, padded, graph_safe=self.graph_safe)
        ar = self._ar[key]
        c8 = (count + 7) // 8 * 8
        inp = ar.input(c8)
        inp[:count].copy_(tensor.reshape(-1))
        if c8 != count:
            inp[count:].zero_()
        out = ar(c8, scale=scale)
        tensor.view(-1).copy_(out[:count])
        return tensor

    def reduce_scatter_tensor(self, output: torch.Tensor, input: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
        """output (numel = input.numel() / n) <- this rank's chunk of scale * sum(input)."""
        self._check_bf16(input, "reduce_scatter_tensor")
        count = input.numel()
        if count % self.n or output.numel() != count // self.n:
            raise ValueError("reduce_scatter_tensor: output must hold input.numel() / world_size elements")
        if count % (8 * self.n):
            raise ValueError("reduce_scatter_tensor: input.numel() must be a multiple of 8 * world_size")
        padded = _size_class(count, 8 * self.n)
        key = (padded, output.dtype)
        if key not in self._rs:
            self._rs[key] = ReduceScatter(self.rt, padded, out_dtype=output.dtype, graph_safe=self.graph_safe)
        rs = self._rs[key]
        rs.input(count).copy_(input.reshape(-1))
        res = rs(count, scale=scale)
        output.view(-1).copy_(res)
        return output

    def all_gather_into_tensor(self, output: torch.Tensor, input: torch.Tensor) -> torch.Tensor:
        """output (n * input.numel() elements, same dtype) <- every rank's input in rank order."""
        if output.dtype != input.dtype or output.numel() != self.n * input.numel():
            raise ValueError("all_gather_into_tensor: output must hold world_size * input.numel() of input's dtype")
        nbytes = input.numel() * input.element_size()
        if nbytes % 16:
            raise ValueError("all_gather_into_tensor: the shard must be a multiple of 16 bytes")
        padded = _size_class(nbytes, 16)
        if padded not in self._ag:
            self._ag[padded] = AllGather(self.rt, padded, graph_safe=self.graph_safe)
        ag = self._ag[padded]
        ag.shard(nbytes).copy_(input.reshape(-1).view(torch.uint8))
        res = ag(nbytes)
        output.reshape(-1).view(torch.uint8).copy_(res.reshape(-1))
        return output
