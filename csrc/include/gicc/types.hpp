// types.hpp -- host/device shared types of the runtime.
//
// Buffer / RemoteBufferInfo keep the reference's field names (gicc_types.hpp:13-25).  On
// NVLink there are no memory keys: `lkey` is the local buffer index and `rkey` the
// remote buffer index; `RemoteBufferInfo::addr` is the peer buffer's address *mapped
// into this process* (directly dereferenceable from device code), not the peer's own VA.
#pragma once
#include <cstddef>
#include <cstdint>

#include "gicc/error.hpp"

namespace gicc {

constexpr int GICC_MAX_BUFS = 64;   // registered buffers per rank (reference: 16, gicc_context.cuh:27-30)
constexpr int GICC_MAX_PEERS = 64;  // ranks (reference: gicc_context.cuh:27-30, types.hpp:14)
constexpr int GICC_POOL_SIZE = 32;  // host-queued ops per batch (reference: ofi_runtime.hpp:57)
constexpr int GICC_MAX_ROUNDS = 12; // dissemination rounds, 4096 ranks (reference: gicc_barrier.hpp:55)

struct Buffer {
  void* ptr;
  size_t size;
  uint64_t addr;
  uint32_t lkey;
  uint32_t rkey;
  int index;
};

struct RemoteBufferInfo {
  uint64_t addr;
  uint32_t rkey;
};

// Host-queued put (OFI-style put_no_db): executed on the GPU by flush().
struct QueuedOp {
  uint64_t src;   // local source address
  uint64_t dst;   // destination address (peer memory mapped into this process)
  uint64_t size;  // bytes
  int32_t peer;
  uint32_t slot;  // completion slot
};

struct OpTable {
  uint32_t n_ops;       // ops queued so far in this batch
  uint32_t n_done;      // ops executed by flush() (device-owned)
  uint64_t* completion; // [GICC_POOL_SIZE] epoch per slot; mapped pinned host memory
  uint64_t epoch;       // completion value of this batch
  QueuedOp ops[GICC_POOL_SIZE];
};

// Per-peer device context returned by Runtime::prepare (reference: DeviceStateOpt,
// platform/mlx5/device_opt.cuh:147-185 -- QP, doorbell and CQ state; here peer mappings).
struct DeviceCtx {
  int my_rank;
  int n_ranks;
  int peer;
  int n_bufs;
  uint64_t remote_addr;  // default destination (peer buffer chosen at prepare)
  uint32_t remote_rkey;
  uint32_t checks;      // 1: bounds-check every put (GICC_CHECKS=1 at prepare time)
  uint64_t local_base[GICC_MAX_BUFS];
  uint64_t local_size[GICC_MAX_BUFS];
  uint64_t remote_base[GICC_MAX_BUFS];  // peer's buffers, mapped here
  uint64_t remote_size[GICC_MAX_BUFS];
  uint64_t* sig_local;   // this rank's signal words
  uint64_t* sig_remote;  // the peer's signal words, mapped here
  OpTable* ops;          // host-queued puts (nullptr when none)
  ErrorRecord* err;
  uint64_t timeout_ns;
};

// Whole-job device context (reference: GiccContext, platform/mlx5/gicc_context.cuh:27-61).
struct GiccContext {
  int my_rank;
  int n_ranks;
  int n_bufs;
  int checks;  // 1: bounds-check every put (GICC_CHECKS=1 at build_context time)
  uint64_t local_base[GICC_MAX_BUFS];
  uint64_t size[GICC_MAX_BUFS];
  uint64_t peer_base[GICC_MAX_PEERS][GICC_MAX_BUFS];  // [rank][buf]; [my_rank] = local
  uint64_t mc_base[GICC_MAX_BUFS];                     // NVLS multicast address or 0
  uint64_t* sig_local;
  uint64_t* sig_peer[GICC_MAX_PEERS];
  uint64_t* sig_mc;
  DeviceCtx* peer_ctxs[GICC_MAX_PEERS];
  ErrorRecord* err;
  uint64_t timeout_ns;
};

// Device barrier context (reference: BarrierCtx, platform/ofi/ofi_barrier_device.cuh:31-45).
// Signals carry monotonically increasing epochs, so nothing is re-armed between barriers.
// `expected_signal` is the epoch of the next barrier: the host owns it in single mode
// (Barrier::setup), a continuous-mode kernel owns it and increments it after each
// barrier() -- the reference's contract (examples/ofi/barrier_test.cpp:32-41).
struct BarrierCtx {
  int n_rounds;                              // ceil(log2(size)); 0 with NVLS or one rank
  int rank;
  int size;
  int n_signal_slots;                        // 1 (epochs make a second slot unnecessary)
  uint64_t* signals;                         // [GICC_MAX_ROUNDS] this rank's slots
  uint64_t* trigger_addrs[GICC_MAX_ROUNDS];  // round k: slot k on rank (rank + 2^k) % size
  uint64_t expected_signal;                  // epoch of the next barrier
  uint64_t* done_counter;                    // mapped host word: epoch of the last completed barrier
  uint64_t* ready_counter;                   // kept for API parity; NVLink needs no host re-arm
  uint64_t* mc_counter;                      // NVLS: multicast address of a shared arrival counter (or 0)
  uint64_t* mc_local;                        // NVLS: this rank's copy of that counter
  ErrorRecord* err;
  uint64_t timeout_ns;
  // failure injection (tests only): at barrier epoch inject_epoch this rank applies
  // inject_mode (proto::Inject) to its own signal
  int inject_mode;
  uint64_t inject_epoch;
};

}  // namespace gicc
