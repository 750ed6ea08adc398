"""2-D 5-point Jacobi (32768 x 32768 fp32, 1000 iterations) with halo puts fused into the stencil kernel.

Grid nx x ny fp32, Dirichlet boundary (top edge 1.0, other edges 0), interior
U[0,1) from a counter-based hash of (seed, global index) -- so every decomposition starts
from the same field.  Interior rows are split over the ranks in contiguous, possibly
uneven chunks (reference: examples/gicc/jacobi.cu:317-339); each rank holds its rows plus
one halo row above and below.  Per iteration one kernel (csrc/kernels/jacobi.cu) updates
all owned rows, pushes the first/last row into the neighbours' halo rows over NVLink and
bumps their arrival counters; the next iteration waits on those counters on the device.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .. import native
from ..utils.graphs import refuse_capture


def split_rows(ny: int, world: int, rank: int):
    interior = ny - 2
    base, extra = divmod(interior, world)
    rows = base + (1 if rank < extra else 0)
    g0 = 1 + rank * base + min(rank, extra)  # global index of the first owned row
    return rows, g0


class Jacobi:
    """``persistent=True`` runs ``run(iters)`` as one cooperative launch (``k_jacobi_persistent``:
    each CTA owns a block of rows and waits on device for its neighbouring blocks and, at the
    ends, for the neighbour ranks' halo rows) instead of one launch per iteration; both use
    the same buffers and counters, so ``step()`` and ``run()`` can be mixed."""

    def __init__(self, nx: int, ny: int, rt=None, seed: int = 3, device: Optional[torch.device] = None,
                 persistent: bool = False):
        if nx % 4:
            raise ValueError("nx must be a multiple of 4")
        self.nx, self.ny, self.seed = nx, ny, seed
        self.rt = rt
        self.world = rt.size if rt is not None else 1
        self.rank = rt.rank if rt is not None else 0
        self.rows, self.g0 = split_rows(ny, self.world, self.rank)
        if self.rows < 1:
            raise ValueError("too many ranks for this grid")
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        shape = (self.rows + 2, nx)
        if self.world > 1:
            self.sym = [rt.alloc_tensor(shape, torch.float32, exchange=False) for _ in range(2)]
            rt.exchange()
            self.bufs = [s.local for s in self.sym]
            self.flag_off = rt.signal_alloc(2)  # [0] top-halo arrivals, [1] bottom-halo arrivals
            # neighbours' row counts (for the address of their bottom halo row)
            self.nrows = [split_rows(ny, self.world, q)[0] for q in range(self.world)]
            self.ctas = native().jacobi_ctas_per_row(nx)
        else:
            self.bufs = [torch.empty(shape, dtype=torch.float32, device=self.device) for _ in range(2)]
        self.cur = 0
        self.done = 0  # iterations completed (same count on every rank)
        native().k_jacobi_init(self.bufs[0].data_ptr(), self.bufs[1].data_ptr(), nx, ny, self.rows, self.g0, seed)
        if self.world > 1:
            # The init writes both buffers' halo rows, which the neighbours overwrite with their
            # pushed rows from the first iteration on: no rank may push before every rank's init
            # has completed, or the init would clobber the pushed row.
            torch.cuda.synchronize(self.device)
            rt.barrier()
        self.norm_buf = torch.zeros(1, dtype=torch.float64, device=self.device)
        self.persistent = persistent
        if persistent:
            grid = native().jacobi_persistent_grid(self.rows)
            self.done_ctr = torch.zeros(grid, dtype=torch.int64, device=self.device)

    def step(self, norm: bool = False) -> None:
        if self.world > 1:
            refuse_capture("Jacobi.step on several ranks")
        a, b = self.bufs[self.cur], self.bufs[1 - self.cur]
        top_dst = bot_dst = top_sig = bot_sig = top_flag = bot_flag = 0
        wait = 0
        if self.world > 1:
            r, nx, rt = self.rank, self.nx, self.rt
            wb = self.sym[1 - self.cur]
            if r > 0:  # my first row -> upper neighbour's bottom halo (row rows[r-1]+1)
                top_dst = wb.ptr(r - 1) + (self.nrows[r - 1] + 1) * nx * 4
                top_sig = rt.signal_peer(r - 1, self.flag_off + 1)
                top_flag = rt.signal_local(self.flag_off)
            if r < self.world - 1:  # my last row -> lower neighbour's top halo (row 0)
                bot_dst = wb.ptr(r + 1)
                bot_sig = rt.signal_peer(r + 1, self.flag_off)
                bot_flag = rt.signal_local(self.flag_off + 1)
            wait = self.done * self.ctas
        native().k_jacobi_step(a.data_ptr(), b.data_ptr(), self.nx, self.rows, top_dst, bot_dst, top_sig, bot_sig,
                               top_flag, bot_flag, wait, wait, self.norm_buf.data_ptr() if norm else 0,
                               self.rt.timeout_ns if self.rt is not None else 0, self.rank)
        self.cur ^= 1
        self.done += 1

    def _run_persistent(self, iters: int, norm: bool) -> None:
        d = {"buf": [b.data_ptr() for b in self.bufs], "nx": self.nx, "rows": self.rows, "iter0": self.done,
             "iters": iters, "done": self.done_ctr.data_ptr(), "norm": self.norm_buf.data_ptr() if norm else 0,
             "rank": self.rank, "timeout_ns": self.rt.timeout_ns if self.rt is not None else 0}
        if self.world > 1:
            r, nx, rt = self.rank, self.nx, self.rt
            if r > 0:  # my first row -> upper neighbour's bottom halo, in its buffer of either parity
                d["top_dst"] = [self.sym[q].ptr(r - 1) + (self.nrows[r - 1] + 1) * nx * 4 for q in range(2)]
                d["top_sig_remote"] = rt.signal_peer(r - 1, self.flag_off + 1)
                d["top_flag"] = rt.signal_local(self.flag_off)
            if r < self.world - 1:  # my last row -> lower neighbour's top halo (row 0)
                d["bot_dst"] = [self.sym[q].ptr(r + 1) for q in range(2)]
                d["bot_sig_remote"] = rt.signal_peer(r + 1, self.flag_off)
                d["bot_flag"] = rt.signal_local(self.flag_off + 1)
        native().k_jacobi_run(d)
        self.done += iters
        self.cur = self.done & 1

    def run(self, iters: int, norm_last: bool = False) -> Optional[float]:
        """Run `iters` iterations; optionally return the global L2 norm of the last update."""
        if self.persistent and iters > 0:
            refuse_capture("Jacobi.run (persistent)")
            if norm_last:
                self.norm_buf.zero_()
            self._run_persistent(iters, norm_last)
        for i in range(0 if self.persistent else iters):
            want = norm_last and i == iters - 1
            if want:
                self.norm_buf.zero_()
            self.step(norm=want)
        if not norm_last:
            return None
        torch.cuda.synchronize()
        local = float(self.norm_buf.item())
        if self.rt is not None and self.world > 1:
            from ..parallel.bootstrap import allreduce_sum

            local = allreduce_sum(self.rt.boot, local)
        return local ** 0.5

    def owned(self) -> torch.Tensor:
        """This rank's owned rows of the current field."""
        return self.bufs[self.cur][1:self.rows + 1]


# ---- CPU oracle -------------------------------------------------------------------------------
def hash_uniform_np(seed: int, idx: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = np.uint64(seed) * np.uint64(0x9E3779B97F4A7C15) + idx.astype(np.uint64) + np.uint64(1)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        z ^= z >> np.uint64(31)
    return (z >> np.uint64(40)).astype(np.float32) * np.float32(1.0 / 16777216.0)


def init_field_np(nx: int, ny: int, seed: int = 3) -> np.ndarray:
    g = np.arange(ny, dtype=np.uint64)[:, None]
    j = np.arange(nx, dtype=np.uint64)[None, :]
    a = hash_uniform_np(seed, g * np.uint64(nx) + j)
    a[0, :] = 1.0
    a[-1, :] = 0.0
    a[1:-1, 0] = 0.0
    a[1:-1, -1] = 0.0
    return a.astype(np.float32)


def jacobi_np(nx: int, ny: int, iters: int, seed: int = 3) -> np.ndarray:
    """Single-rank CPU restatement with the kernel's operation order (bit-identical)."""
    a = init_field_np(nx, ny, seed)
    b = a.copy()
    q = np.float32(0.25)
    for _ in range(iters):
        b[1:-1, 1:-1] = ((a[1:-1, 2:] + a[1:-1, :-2]) + (a[:-2, 1:-1] + a[2:, 1:-1])) * q
        a, b = b, a
    return a
