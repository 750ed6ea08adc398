"""Distributed GEMM (M = N = K = 16384, bf16): bf16 in / f32 accumulate, C = A . B.

Two modes, both over the NVLink symmetric-memory runtime (no NCCL on this path):

* ``ag`` -- all-gather -> GEMM.  A [M, K] is row-sharded (rank r owns rows
  r*M/w ... (r+1)*M/w), B is column-sharded (rank r owns output columns r*N/w ...),
  stored as B^T rows [N/w, K] (the weight layout of nn.Linear).  Each rank computes
  C[:, cols_r] = A_full @ B_r^T.
* ``rs`` -- GEMM -> reduce-scatter.  K is sharded: rank r owns A[:, k_r] and B[:, k_r];
  partial products are summed across ranks and rank r keeps rows r*M/w ... of C.

With one GPU both reduce to the single tcgen05 GEMM.  The reference's version of this
workload is the striped fp32 ring matmul of examples/gicc/mm.cu:116-225 (B stripes
rotated around the ring while a SIMT kernel accumulates with atomicAdd).
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from ..ops.gemm import gemm
from ..utils.graphs import refuse_capture


# The fused kernels on CTA pairs are the default where their tiles fill the GPU evenly
# (measured on two B200s: all-gather GEMM 2.93 ms on 256 x 512 pair tiles against 3.46 ms on
# 128 x 256 tiles, NCCL + cuBLAS 3.34 ms).
PAIR_BY_DEFAULT = True


class DistGemm:
    def __init__(self, M: int, N: int, K: int, mode: str = "ag", rt=None, device: Optional[torch.device] = None,
                 fused: bool = True, nvls: Optional[bool] = None, transfer: str = "sm"):
        self.M, self.N, self.K, self.mode = M, N, K, mode
        self.fused = fused
        self.rt = rt
        self.world = rt.size if rt is not None else 1
        self.rank = rt.rank if rt is not None else 0
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        w = self.world
        if mode not in ("ag", "rs"):
            raise ValueError("mode must be 'ag' or 'rs'")
        if M % w or N % w or K % w:
            raise ValueError("M, N and K must be divisible by the number of ranks")
        self.launches_per_step = 1
        self.epoch = 0
        # Fused AG: the shard goes out through the NVLS multicast view when the node has
        # NVLS (one write reaches every GPU), else by unicast pushes to each peer.  Only
        # `comm_ctas` CTAs push (SMs that push stall their own tensor-core work, so few do,
        # and the dynamic tile order gives them fewer tiles).  Tuning and diagnostics:
        # units each 128-row band is pushed in, CTAs (0 = one per SM), a uint64 trace
        # tensor (None = off) and the diag bits.
        # transfer="ce" (AG only): the copy engines move the shard (ops ag_transfer_ce on a side
        # stream, arrival counters written by stream memory operations) and no SM pushes.
        if transfer not in ("sm", "ce") or (transfer == "ce" and mode != "ag"):
            raise ValueError("transfer must be 'sm', or 'ce' for the ag mode")
        self.transfer = transfer
        self.ce_chunks = 4
        self._side = None
        if transfer == "ce":
            nvls = False
        self.nvls = bool(nvls if nvls is not None else (rt is not None and w > 1 and rt.multicast_supported))
        # Pieces each 128-row band of the shard is pushed in.  With NVLS, 16 pieces let the
        # pushing CTAs finish the lowest bands first (8 GPUs: 1.015 ms against 1.114 ms with 4)
        self.units_per_band = 16 if (self.nvls and mode == "ag") else 4
        self.grid = 0
        # NVLS at 8 GPUs is bound by each GPU's NVLink ingress (7 shards arrive at once), so
        # more CTAs push there; at 2-4 GPUs 8 keep well ahead of the tensor cores.
        self.comm_ctas = (16 if w >= 8 else 8) if self.nvls else 32
        # RS over NVLS: CTAs whose reduce warps run multimem.ld_reduce (32 measured faster than 16
        # at two GPUs: 3.36 vs 3.55 ms with pair tiles)
        self.rs_reduce_ctas = 32
        self.rs_join = False      # RS over NVLS: CTAs out of GEMM tiles join the reduction (A/B option)
        # RS over NVLS: m-blocks per raster group (0 = 16).  A band can be reduced once all its
        # column tiles are done, so smaller groups feed the reduction sooner; when B fits in L2
        # (small K shards) they cost no extra DRAM traffic.  A/B option.
        self.rs_raster_group = 0
        self.trace: Optional[torch.Tensor] = None
        self.diag = 0
        # Tensor-core tiles of the fused kernels (AG, and RS over NVLS): 0 = one CTA per
        # 128 x 256 tile; 1 / 2 = CTA pairs (cta_group::2) with 256 x 256 / 256 x 512 tiles.
        # Fixed by the first call (the counters depend on it).  Default: the 256 x 512 pair
        # tile where it fills the CTA pairs about as evenly as 128 x 256 tiles fill the SMs.
        # GICC_DIST_GEMM_PAIR=0|1|2 overrides the default (A/B experiments).
        self.pair = self._default_pair() if (w > 1 and fused and (mode == "ag" or self.nvls) and PAIR_BY_DEFAULT) else 0
        env_pair = os.environ.get("GICC_DIST_GEMM_PAIR")
        if env_pair not in (None, "") and w > 1 and fused and (mode == "ag" or self.nvls):
            if env_pair not in ("0", "1", "2"):
                raise ValueError("GICC_DIST_GEMM_PAIR must be 0, 1 or 2")
            self.pair = int(env_pair)
        if w > 1 and fused:
            # fused kernels: double-buffered landing areas + epoch counters in the signal heap
            if mode == "ag":
                self.A_bufs = [rt.alloc_tensor((M, K), torch.bfloat16, multicast=self.nvls, exchange=False)
                               for _ in range(2)]
                nbands = (M // w) // 128
            elif self.nvls:
                # NVLS reduce-scatter: each rank's whole [M, N] bf16 partial, reduced in the switch
                self.slot_bufs = [rt.alloc_tensor((M, N), torch.bfloat16, multicast=True, exchange=False)
                                  for _ in range(2)]
                nbands = (M // w) // 128
            else:
                self.slot_bufs = [rt.alloc_tensor((w, M // w, N), torch.bfloat16, exchange=False) for _ in range(2)]
                nbands = (M // w) // 128
            rt.exchange()
            off = rt.signal_alloc(w * nbands + w + 1)
            self.arrivals = [rt.signal_peer(p, off) for p in range(w)]
            self.done = [rt.signal_peer(p, off + w * nbands) for p in range(w)]
            self.tile_counter = rt.signal_local(off + w * nbands + w)  # AG dynamic tile order
            self.arrivals_mc = rt.signal_multicast(off) if self.nvls and mode == "ag" else 0
            if self.nvls and mode == "ag" and (not self.arrivals_mc or not self.A_bufs[0].mc_ptr):
                raise RuntimeError("DistGemm: NVLS requested but the runtime has no multicast mapping")
            if self.nvls and mode == "rs":
                if not self.slot_bufs[0].mc_ptr:
                    raise RuntimeError("DistGemm: NVLS requested but the runtime has no multicast mapping")
                self.band_tiles = rt.signal_local(rt.signal_alloc(w * nbands))
                self.unit_counter = rt.signal_local(rt.signal_alloc(1))
            self.C = torch.empty(*self.out_shape(), dtype=torch.bfloat16, device=self.device)
            self.launches_per_step = 1
        elif w > 1:
            from ..ops import collectives
            from ..parallel import Barrier

            self._coll = collectives
            self.barrier = Barrier(rt)
            if mode == "ag":
                self.A_full = rt.alloc_tensor((M, K), torch.bfloat16)
                self.C = torch.empty(M, N // w, dtype=torch.bfloat16, device=self.device)
                self.launches_per_step = 2 + (w - 1) + 1
            else:
                self.P = rt.alloc_tensor((M, N), torch.bfloat16)  # bf16 partials, f32 reduction
                self.C = torch.empty(M // w, N, dtype=torch.bfloat16, device=self.device)
                self.launches_per_step = 1 + 2 + 1

    def _default_pair(self) -> int:
        w = self.world
        rows, cols = (self.M, self.N // w) if self.mode == "ag" else (self.M, self.N)
        if (self.M // w) % 256 or cols % 256 or self.transfer != "sm":
            return 0
        cols512_ok = cols % 512 == 0
        # B200: 148 SMs (used where no GPU is visible, e.g. host-side tests)
        sms = torch.cuda.get_device_properties(self.device).multi_processor_count if torch.cuda.is_available() else 148

        def fill(tiles: int, slots: int) -> float:
            return tiles / (-(-tiles // slots) * slots)

        t2 = (rows // 256) * (cols // 512)
        t1 = (rows // 256) * (cols // 256)
        t0 = (rows // 128) * (cols // 256)
        if cols512_ok and t2 >= sms // 2 and fill(t2, sms // 2) >= fill(t0, sms) - 0.05:
            return 2
        # 256 x 256 pair tiles where the 256 x 512 ones fill the pairs unevenly (the all-gather
        # GEMM at 8 GPUs: 0.965 ms against 1.010 ms with 128 x 256 tiles, same run)
        return 1 if t1 >= sms // 2 and fill(t1, sms // 2) >= fill(t0, sms) - 0.05 else 0

    def tune(self, A: torch.Tensor, B: torch.Tensor, comm_ctas=None, calls: int = 3) -> dict:
        """Fused all-gather GEMM on several ranks: time candidate numbers of pushing CTAs on
        this node and keep the fastest.  How fast a few SMs fill the NVLink ingress differs
        from node to node (NVLS multicast or unicast, switch load), so the count is measured
        rather than fixed.  Each candidate gets one untimed call and `calls` timed calls
        (device time of the calls, max over ranks); A (this rank's shard) goes into both
        landing buffers first, so the calls read it in place.  Collective: every rank calls
        it with the same arguments.  Returns {comm_ctas: ms per call}; other modes return {}."""
        if not (self.fused and self.mode == "ag" and self.world > 1 and self.transfer == "sm"):
            return {}
        from ..parallel.bootstrap import allreduce_max

        cands = list(comm_ctas) if comm_ctas else ([8, 16, 24, 32] if self.nvls else [16, 32, 48])
        self.a_slot(0).copy_(A)
        self.a_slot(1).copy_(A)
        boot = self.rt.boot
        res = {}
        for c in cands:
            self.comm_ctas = c
            self(self.a_slot(), B)
            torch.cuda.synchronize(self.device)
            boot.barrier()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(calls):
                self(self.a_slot(), B)
            e.record()
            torch.cuda.synchronize(self.device)
            res[c] = allreduce_max(boot, s.elapsed_time(e) / calls)
        self.comm_ctas = min(res, key=res.get)
        self.rt.check_device_errors()
        return res

    # shapes of this rank's operands
    def a_shape(self):
        w = self.world
        return (self.M // w, self.K) if self.mode == "ag" else (self.M, self.K // w)

    def b_shape(self):
        w = self.world
        return (self.N // w, self.K) if self.mode == "ag" else (self.N, self.K // w)

    def out_shape(self):
        w = self.world
        return (self.M, self.N // w) if self.mode == "ag" else (self.M // w, self.N)

    def _check_frozen_settings(self) -> None:
        """The counters of a fused instance advance by amounts that depend on the grid, the
        units per band and the diag bits (tile counter: tiles + grid per call; arrival
        counters: units per band per call, none with diag bit 0; RS reduce-unit counter: only
        with rs_join).  They are fixed by the first call; changing them later would
        desynchronise the counters, so it is refused.
        comm_ctas, rs_reduce_ctas and trace may change freely."""
        now = (self.grid, self.units_per_band, self.diag, self.rs_join, self.pair)
        first = getattr(self, "_frozen", None)
        if first is None:
            self._frozen = now
        elif first != now:
            raise ValueError(f"DistGemm: grid / units_per_band / diag were {first} at the first call and are {now} "
                             "now; create a new DistGemm to change them")

    def trace_words(self) -> int:
        """Size (uint64 words) of the fused kernel's trace buffer for the current settings
        (AG: unicast or NVLS; RS: NVLS only)."""
        w = self.world
        nb = (self.M // w) // 128
        grid = self.grid or torch.cuda.get_device_properties(self.device).multi_processor_count
        if self.mode == "rs":
            tiles = w * nb * (self.N // 256)
            return tiles + 2 * nb * self.units_per_band + 2 * grid
        tiles = w * nb * ((self.N // w) // 256)
        units = 0 if self.diag & 1 else (1 if self.nvls else w - 1) * nb * self.units_per_band
        return 3 * tiles + 2 * units + 2 * grid

    def a_slot(self, parity: Optional[int] = None) -> torch.Tensor:
        """Where this rank's A shard must live for the AG mode (zero-copy input).  Fused
        mode alternates two landing buffers; by default the slot of the *next* call."""
        Ms = self.M // self.world
        if self.fused:
            p = (self.epoch + 1) % 2 if parity is None else parity
            return self.A_bufs[p].local[self.rank * Ms:(self.rank + 1) * Ms]
        return self.A_full.local[self.rank * Ms:(self.rank + 1) * Ms]

    def input_slots(self) -> Optional[list]:
        """The A slots of this rank's next two calls, in call order, when the fused AG mode
        double-buffers them (so a producer can fill call i+1's slot while call i runs);
        None otherwise.  Valid while every call takes its A from these slots in turn."""
        if not (self.fused and self.mode == "ag" and self.world > 1):
            return None
        return [self.a_slot((self.epoch + 1) % 2), self.a_slot((self.epoch + 2) % 2)]

    def _peer_ptrs(self, buf, parity: int):
        """Every rank's address of a symmetric buffer (fixed for the object's life; cached so
        a call does not rebuild the list)."""
        cache = self.__dict__.setdefault("_ptr_cache", {})
        key = (id(buf), parity)
        if key not in cache:
            cache[key] = [buf.ptr(q) for q in range(self.world)]
        return cache[key]

    def forward(self, A: torch.Tensor, B: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        w, r = self.world, self.rank
        if w == 1:
            return gemm(A, B, out=out)
        refuse_capture("DistGemm")
        if self.fused:
            from .. import native

            self._check_frozen_settings()
            if self.pair and self.trace is not None:
                raise ValueError("DistGemm: the trace buffer is supported by the single-CTA kernel only (pair=0)")
            self.epoch += 1
            p = self.epoch % 2
            C = out if out is not None else self.C
            n = native()
            if self.mode == "ag":
                slot = self.a_slot(p)
                if A.data_ptr() != slot.data_ptr():
                    slot.copy_(A)
                buf = self.A_bufs[p]
                ptrs = self._peer_ptrs(buf, p)
                diag = self.diag
                done_ev = None
                if self.transfer == "ce":
                    diag |= 2  # the kernel waits for arrivals but does not push
                    cur = torch.cuda.current_stream()
                    if self._side is None:
                        self._side = torch.cuda.Stream(device=self.device)
                    ready = torch.cuda.Event()
                    ready.record(cur)  # the shard is in the slot
                    self._side.wait_event(ready)
                    grid = self.grid or torch.cuda.get_device_properties(self.device).multi_processor_count
                    with torch.cuda.stream(self._side):
                        n.ag_transfer_ce(w, r, self.M, self.K, ptrs, self.arrivals, self.done[r], self.epoch, grid,
                                         self.units_per_band, self.ce_chunks, self.rt.timeout_ns)
                    done_ev = torch.cuda.Event()
                    done_ev.record(self._side)
                n.k_ag_gemm(w, r, self.M, self.N // w, self.K, ptrs, B.data_ptr(),
                            B.stride(0), C.data_ptr(), C.stride(0), self.arrivals, self.done, self.epoch,
                            self.units_per_band, self.grid, self.rt.timeout_ns,
                            self.trace.data_ptr() if self.trace is not None else 0, diag, self.comm_ctas,
                            self.tile_counter, buf.mc_ptr if self.nvls else 0, self.arrivals_mc,
                            self.pair)
                if done_ev is not None:
                    # later work on this stream (e.g. rewriting the shard slot) waits for the outgoing copies
                    torch.cuda.current_stream().wait_event(done_ev)
            else:
                buf = self.slot_bufs[p]
                if self.nvls:
                    n.k_gemm_rs(w, r, self.M, self.N, self.K // w, A.data_ptr(), A.stride(0), B.data_ptr(),
                                B.stride(0), self._peer_ptrs(buf, p), self.arrivals, self.done, C.data_ptr(),
                                C.stride(0), self.epoch, self.grid, self.rt.timeout_ns, buf.mc_ptr, self.band_tiles,
                                self.tile_counter, self.rs_reduce_ctas, self.units_per_band,
                                self.trace.data_ptr() if self.trace is not None else 0, int(self.rs_join),
                                self.unit_counter, self.rs_raster_group, self.pair)
                else:
                    n.k_gemm_rs(w, r, self.M, self.N, self.K // w, A.data_ptr(), A.stride(0), B.data_ptr(),
                                B.stride(0), self._peer_ptrs(buf, p), self.arrivals, self.done, C.data_ptr(),
                                C.stride(0), self.epoch, self.grid, self.rt.timeout_ns)
            return C
        if self.mode == "ag":
            Ms = self.M // w
            slot = self.a_slot()
            if A.data_ptr() != slot.data_ptr():
                slot.copy_(A)
            self.barrier.device_barrier()  # every shard is in place
            row_bytes = self.K * 2
            for k in range(1, w):
                p = (r + k) % w
                off = p * Ms * row_bytes
                self._coll.copy(self.A_full.ptr() + off, self.A_full.ptr(p) + off, Ms * row_bytes)
            C = gemm(self.A_full.local, B, out=out if out is not None else self.C)
            self.barrier.device_barrier()  # peers finished reading our shard
            return C
        # rs: partial product, then each rank reduces its row block from all peers
        gemm(A, B, out=self.P.local)
        self.barrier.device_barrier()
        Mr = self.M // w
        C = out if out is not None else self.C
        srcs = [self.P.ptr(p) + r * Mr * self.N * 2 for p in range(w)]
        self._coll.reduce_sum(C, srcs, Mr * self.N)
        self.barrier.device_barrier()
        return C

    __call__ = forward


def make_operands(M: int, N: int, K: int, mode: str, world: int, rank: int, seed: int = 2,
                  device: Optional[torch.device] = None):
    """Synthetic A, B ~ N(0, sigma^2) with sigma^2 = 1/sqrt(K) (so C has unit variance),
    generated identically on every rank from `seed`; returns this rank's shards."""
    device = device or torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=device).manual_seed(seed)
    std = K ** -0.25
    A = (torch.randn(M, K, generator=g, device=device) * std).to(torch.bfloat16)
    B = (torch.randn(N, K, generator=g, device=device) * std).to(torch.bfloat16)  # B^T layout
    if mode == "ag":
        Ms, Ns = M // world, N // world
        return A[rank * Ms:(rank + 1) * Ms].contiguous(), B[rank * Ns:(rank + 1) * Ns].contiguous(), (A, B)
    Ks = K // world
    return A[:, rank * Ks:(rank + 1) * Ks].contiguous(), B[:, rank * Ks:(rank + 1) * Ks].contiguous(), (A, B)


def smoke_step(device: torch.device) -> None:
    """One tiny forward through the flagship path on one GPU, checked against fp32."""
    from ..ops.gemm import check_errors

    torch.cuda.set_device(device)
    model = DistGemm(256, 512, 384, "ag", rt=None, device=device)
    A, B, (Af, Bf) = make_operands(256, 512, 384, "ag", 1, 0, device=device)
    C = model(A, B)
    torch.cuda.synchronize(device)
    check_errors()
    ref = Af.float() @ Bf.float().t()
    err = (C.float() - ref).abs().max().item()
    if not err <= 2e-2 * ref.abs().max().item() + 1e-2:
        raise RuntimeError(f"smoke: distributed GEMM mismatch (max abs err {err})")
