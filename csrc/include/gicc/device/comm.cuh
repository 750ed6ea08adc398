// comm.cuh -- the device API: put / put_no_db / flush / quiet / barrier (+ group-scope
// puts, gets, put_signal and bounded signal waits).
//
// Reference device API (platform/mlx5/mlx5_device.cuh:29-92, gicc_context.cuh:102-147,
// platform/ofi/ofi_device.cuh:52-75) builds NIC work-queue entries and rings doorbells.
// On NVLink a put is the copy itself: 16-byte vector stores from SMs into the peer's HBM
// (the peer buffer is mapped into this process by Runtime::exchange).  Completion:
//   quiet  = fence.acq_rel.sys  (this thread's stores are performed system-wide)
//   signal = release store / release add on a peer flag word, acquire polls on the
//            other side, every poll bounded by %globaltimer.
// `flush` keeps its OFI meaning: it executes the puts that the host queued with
// Runtime::put_no_db and marks their completion slots.
#pragma once
#include <cstdint>

#include "gicc/device/ptx.cuh"
#include "gicc/proto/barrier.hpp"
#include "gicc/proto/mem.hpp"
#include "gicc/types.hpp"

namespace gicc {

enum class Scope { Thread, Warp, Block };

template <Scope S>
__device__ __forceinline__ int scope_rank() {
  if (S == Scope::Thread) return 0;
  if (S == Scope::Warp) return threadIdx.x & 31;
  return threadIdx.x + blockDim.x * (threadIdx.y + blockDim.y * threadIdx.z);
}
template <Scope S>
__device__ __forceinline__ int scope_size() {
  if (S == Scope::Thread) return 1;
  if (S == Scope::Warp) return 32;
  return blockDim.x * blockDim.y * blockDim.z;
}
template <Scope S>
__device__ __forceinline__ void scope_sync() {
  if (S == Scope::Warp) __syncwarp();
  if (S == Scope::Block) __syncthreads();
}

// Cooperative copy of n bytes (any alignment).  16-byte vectors when src and dst share
// their alignment modulo 16, with 4 independent vectors in flight per thread.
template <Scope S>
__device__ __forceinline__ void copy_bytes(void* dst, const void* src, size_t n) {
  const int r = scope_rank<S>(), w = scope_size<S>();
  char* d = static_cast<char*>(dst);
  const char* s = static_cast<const char*>(src);
  if ((((uintptr_t)d ^ (uintptr_t)s) & 15) == 0) {
    size_t head = (16 - ((uintptr_t)d & 15)) & 15;
    if (head > n) head = n;
    for (size_t i = r; i < head; i += w) d[i] = s[i];
    const size_t nv = (n - head) >> 4;
    const uint4* sv = reinterpret_cast<const uint4*>(s + head);
    uint4* dv = reinterpret_cast<uint4*>(d + head);
    size_t i = r;
    for (; i + 3 * (size_t)w < nv; i += 4 * (size_t)w) {
      const uint4 a = sv[i], b = sv[i + w], c = sv[i + 2 * w], e = sv[i + 3 * w];
      dv[i] = a;
      dv[i + w] = b;
      dv[i + 2 * w] = c;
      dv[i + 3 * w] = e;
    }
    for (; i < nv; i += w) dv[i] = sv[i];
    for (size_t j = head + (nv << 4) + r; j < n; j += w) d[j] = s[j];
  } else if ((((uintptr_t)d ^ (uintptr_t)s) & 3) == 0) {
    size_t head = (4 - ((uintptr_t)d & 3)) & 3;
    if (head > n) head = n;
    for (size_t i = r; i < head; i += w) d[i] = s[i];
    const size_t nw = (n - head) >> 2;
    const uint32_t* sw = reinterpret_cast<const uint32_t*>(s + head);
    uint32_t* dw = reinterpret_cast<uint32_t*>(d + head);
    for (size_t i = r; i < nw; i += w) dw[i] = sw[i];
    for (size_t j = head + (nw << 2) + r; j < n; j += w) d[j] = s[j];
  } else {
    for (size_t i = r; i < n; i += w) d[i] = s[i];
  }
}

// ---------------------------------------------------------------------------------------
// pointer-based primitives
// ---------------------------------------------------------------------------------------
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put(void* dst_remote, const void* src, size_t n) {
  copy_bytes<S>(dst_remote, src, n);
}
template <Scope S = Scope::Thread>
__device__ __forceinline__ void get(void* dst, const void* src_remote, size_t n) {
  copy_bytes<S>(dst, src_remote, n);
}
__device__ __forceinline__ void quiet() { ptx::fence_acq_rel_sys(); }

// Bulk put of a tile staged in this CTA's shared memory: one thread issues a cp.async.bulk
// shared -> global store (no multicast) straight into the peer's memory, so the copy needs
// no registers and no further instructions of the CTA.  Addresses 16-byte aligned, bytes a
// multiple of 16.  Before it: the threads that wrote the tile run fence_tile_for_put() and
// the CTA synchronises.  put_tile_wait_read(): the tile's shared memory may be rewritten;
// put_tile_wait(): the stores are complete, after which quiet() + a release signal publish
// them like any other put.
__device__ __forceinline__ void fence_tile_for_put() { ptx::fence_proxy_async_smem(); }
__device__ __forceinline__ void put_tile(void* dst_remote, const void* src_smem, uint32_t bytes) {
  ptx::bulk_store(dst_remote, src_smem, bytes);
  ptx::bulk_commit();
}
__device__ __forceinline__ void put_tile_wait_read() { ptx::bulk_wait_read_all(); }
__device__ __forceinline__ void put_tile_wait() {
  ptx::bulk_wait_all();
  ptx::fence_proxy_async_global();  // the async-proxy writes are ordered with what follows
}

enum SignalOp : int { SIGNAL_SET = 0, SIGNAL_ADD = 1 };

// Put n bytes, then publish `value` on the peer's signal word once the data is visible.
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put_signal(void* dst_remote, const void* src, size_t n, uint64_t* sig_remote,
                                           uint64_t value, int op = SIGNAL_SET) {
  copy_bytes<S>(dst_remote, src, n);
  ptx::fence_acq_rel_sys();
  scope_sync<S>();
  if (scope_rank<S>() == 0) {
    if (op == SIGNAL_ADD)
      ptx::red_release_sys_add(sig_remote, value);
    else
      ptx::st_release_sys(sig_remote, value);
  }
}

__device__ __forceinline__ void signal_set(uint64_t* sig, uint64_t v) { ptx::st_release_sys(sig, v); }
__device__ __forceinline__ void signal_add(uint64_t* sig, uint64_t v) { ptx::red_release_sys_add(sig, v); }

// Bounded wait until cmp(*sig, value).  Returns GICC_OK or GICC_ETIMEDOUT (recorded in err).
__device__ __forceinline__ int signal_wait_until(const uint64_t* sig, int cmp, uint64_t value, uint64_t timeout_ns,
                                                 ErrorRecord* err = nullptr, int rank = -1, int peer = -1,
                                                 int where = W_SIGNAL_WAIT) {
  uint64_t seen = 0;
  if (proto::wait_until<proto::DevMem>(sig, cmp, value, timeout_ns, &seen)) return GICC_OK;
  report_error(err, GICC_ETIMEDOUT, where, rank, peer, seen, value);
  return GICC_ETIMEDOUT;
}

// ---------------------------------------------------------------------------------------
// DeviceCtx API (reference signatures; lkey/rkey are buffer indices)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ bool range_ok(const DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr,
                                         uint32_t rkey, uint64_t size) {
  // Bounds checks: on when the context was prepared with GICC_CHECKS=1 in the environment
  // (or the library was built with -DGICC_CHECKS).  A violation records GICC_ERANGE and the
  // access is skipped -- never a trap.
#if !defined(GICC_CHECKS)
  if (!ctx->checks) return true;
#endif
  const bool lok = lkey < (uint32_t)ctx->n_bufs && laddr >= ctx->local_base[lkey] &&
                   laddr + size <= ctx->local_base[lkey] + ctx->local_size[lkey];
  const bool rok = rkey < (uint32_t)ctx->n_bufs && raddr >= ctx->remote_base[rkey] &&
                   raddr + size <= ctx->remote_base[rkey] + ctx->remote_size[rkey];
  if (!(lok && rok)) {
    report_error(ctx->err, GICC_ERANGE, W_BOUNDS, ctx->my_rank, ctx->peer, raddr, size);
    return false;
  }
  return true;
}

template <Scope S = Scope::Thread>
__device__ __forceinline__ void put(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey,
                                    uint32_t size, bool signaled = false) {
  (void)signaled;  // every NVLink put completes at quiet(); no completion entry needed
  if (!range_ok(ctx, laddr, lkey, raddr, rkey, size)) return;
  copy_bytes<S>(reinterpret_cast<void*>(raddr), reinterpret_cast<const void*>(laddr), size);
}
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint32_t size,
                                    bool signaled = false) {
  put<S>(ctx, laddr, lkey, ctx->remote_addr, ctx->remote_rkey, size, signaled);
}
// No doorbell exists on NVLink: the data moves at once; kept for source compatibility.
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put_no_db(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr,
                                          uint32_t rkey, uint32_t size, bool signaled = false) {
  put<S>(ctx, laddr, lkey, raddr, rkey, size, signaled);
}

// Run the puts the host queued with Runtime::put_no_db (OFI semantics: ofi_device.cuh:52-58).
// Call from one thread, or from a whole block with S = Block for bandwidth.
template <Scope S = Scope::Thread>
__device__ __forceinline__ void flush(DeviceCtx* ctx) {
  OpTable* t = ctx->ops;
  if (t == nullptr) {
    ptx::fence_acq_rel_sys();
    return;
  }
  const uint32_t n = *reinterpret_cast<volatile uint32_t*>(&t->n_ops);
  const uint32_t first = *reinterpret_cast<volatile uint32_t*>(&t->n_done);
  const uint64_t epoch = *reinterpret_cast<volatile uint64_t*>(&t->epoch);
  for (uint32_t i = first; i < n; ++i) {
    const QueuedOp op = t->ops[i];
    copy_bytes<S>(reinterpret_cast<void*>(op.dst), reinterpret_cast<const void*>(op.src), op.size);
  }
  ptx::fence_acq_rel_sys();
  scope_sync<S>();
  if (scope_rank<S>() == 0) {
    for (uint32_t i = first; i < n; ++i) ptx::st_release_sys(&t->completion[t->ops[i].slot], epoch);
    t->n_done = n;
  }
  scope_sync<S>();
}

// Wait until every queued op of the current batch completed, then make this thread's
// stores visible system-wide.  Bounded; returns a status (0 = ok).
__device__ __forceinline__ int quiet(DeviceCtx* ctx) {
  int st = GICC_OK;
  OpTable* t = ctx->ops;
  if (t != nullptr) {
    const uint32_t n = *reinterpret_cast<volatile uint32_t*>(&t->n_ops);
    const uint64_t epoch = *reinterpret_cast<volatile uint64_t*>(&t->epoch);
    for (uint32_t i = 0; i < n && st == GICC_OK; ++i)
      st = signal_wait_until(&t->completion[i], proto::CMP_GE, epoch, ctx->timeout_ns, ctx->err, ctx->my_rank,
                             t->ops[i].peer, W_QUIET);
  }
  ptx::fence_acq_rel_sys();
  return st;
}

// ---------------------------------------------------------------------------------------
// GiccContext API (NVSHMEM-style: dst is gicc::remote_ptr(local, peer))
// ---------------------------------------------------------------------------------------
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put(GiccContext* ctx, void* dst, const void* src, uint32_t size, int peer,
                                    bool signaled = true) {
  (void)signaled;
#if !defined(GICC_CHECKS)
  if (ctx->checks)
#endif
  {
    bool ok = false;
    const uint64_t d = (uint64_t)(uintptr_t)dst;
    if (peer >= 0 && peer < ctx->n_ranks)
      for (int b = 0; b < ctx->n_bufs; ++b)
        ok |= d >= ctx->peer_base[peer][b] && d + size <= ctx->peer_base[peer][b] + ctx->size[b];
    if (!ok) {
      report_error(ctx->err, GICC_ERANGE, W_BOUNDS, ctx->my_rank, peer, d, size);
      return;
    }
  }
  copy_bytes<S>(dst, src, size);
}
template <Scope S = Scope::Thread>
__device__ __forceinline__ void put_no_db(GiccContext* ctx, void* dst, const void* src, uint32_t size, int peer,
                                          bool signaled = true) {
  put<S>(ctx, dst, src, size, peer, signaled);
}
__device__ __forceinline__ void flush(GiccContext* ctx, int peer) {
  (void)ctx;
  (void)peer;
  ptx::fence_acq_rel_sys();
}
__device__ __forceinline__ void quiet(GiccContext* ctx, int peer) {
  (void)ctx;
  (void)peer;
  ptx::fence_acq_rel_sys();
}
__device__ __forceinline__ void* remote_ptr(GiccContext* ctx, const void* local, int peer) {
  const uint64_t a = (uint64_t)(uintptr_t)local;
  for (int b = 0; b < ctx->n_bufs; ++b)
    if (a >= ctx->local_base[b] && a < ctx->local_base[b] + ctx->size[b])
      return reinterpret_cast<void*>(ctx->peer_base[peer][b] + (a - ctx->local_base[b]));
  return nullptr;
}

// ---------------------------------------------------------------------------------------
// Barrier (reference: platform/ofi/ofi_barrier_device.cuh:61-86).  One thread.
// Uses ctx->expected_signal as the epoch; the caller (host setup() or a continuous
// kernel) advances it.  Returns a status instead of spinning forever.
// ---------------------------------------------------------------------------------------
// report=false skips the progress store into mapped host memory (continuous kernels report
// once at the end: a pending PCIe write would otherwise stall the next barrier's fence).
__device__ __forceinline__ int barrier(BarrierCtx* ctx, bool report = true) {
  const uint64_t epoch = *reinterpret_cast<volatile uint64_t*>(&ctx->expected_signal);
  const int inject = (ctx->inject_mode && epoch == ctx->inject_epoch) ? ctx->inject_mode : proto::INJECT_NONE;
  uint64_t seen = 0;
  int st;
  if (ctx->mc_counter != nullptr) {
    uint64_t* mc = ctx->mc_counter;
    st = proto::counter_barrier<proto::DevMem>([mc] { ptx::multimem_red_release_add_u64(mc, 1); }, ctx->mc_local,
                                               ctx->size, epoch, ctx->timeout_ns, &seen, inject);
  } else {
    int round = -1;
    st = proto::dissemination_barrier<proto::DevMem>(ctx->n_rounds, ctx->trigger_addrs, ctx->signals, epoch,
                                                     ctx->timeout_ns, &round, &seen, inject);
  }
  if (st != GICC_OK) {
    report_error(ctx->err, st, W_BARRIER, ctx->rank, -1, seen, epoch);
    return st;
  }
  // progress report for the host (plain posted store into mapped host memory)
  if (report) *reinterpret_cast<volatile uint64_t*>(ctx->done_counter) = epoch;
  return GICC_OK;
}

// Whole-block form: every thread calls it; thread 0 runs the protocol.
__device__ __forceinline__ int barrier_block(BarrierCtx* ctx) {
  __shared__ int st;
  ptx::fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0 && threadIdx.y == 0 && threadIdx.z == 0) st = barrier(ctx);
  __syncthreads();
  return st;
}

}  // namespace gicc
