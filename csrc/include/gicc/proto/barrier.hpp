// barrier.hpp -- the epoch dissemination barrier, shared by GPU and CPU-rank code.
//
// Round k: store `epoch` (release) into slot k of rank (r + 2^k) mod n, then wait until
// this rank's slot k holds >= epoch (acquire, bounded).  ceil(log2 n) rounds.  Epochs only
// grow, so a slot never needs re-arming and a faster peer's next epoch cannot be lost
// (>= instead of ==).  The reference runs the same dissemination pattern with NIC-side
// puts that the host re-queues for every barrier (platform/ofi/ofi_barrier_device.cuh:
// 61-86, internal/gicc_barrier.hpp:162-223); here each round is one NVLink store.
#pragma once
#include "gicc/error.hpp"
#include "gicc/proto/mem.hpp"

namespace gicc {
namespace proto {

GICC_HD int n_rounds_for(int n) {
  int r = 0;
  while ((1 << r) < n) ++r;
  return r;
}

// Failure injection for the failure-detection tests: this rank's round-0 signal is left
// out (SKIP_SIGNAL) or carries the previous epoch (STALE_EPOCH).  Either way the peer that
// waits for it runs out its bounded wait and reports GICC_ETIMEDOUT; nothing faults.
enum Inject : int { INJECT_NONE = 0, INJECT_SKIP_SIGNAL = 1, INJECT_STALE_EPOCH = 2 };

GICC_PROTO_TEMPLATE
GICC_HD int dissemination_barrier(int n_rounds, uint64_t* const* trigger, uint64_t* signals, uint64_t epoch,
                                  uint64_t timeout_ns, int* fail_round, uint64_t* seen, int inject = INJECT_NONE) {
  Mem::fence();  // everything before the barrier is visible before our first signal
  for (int k = 0; k < n_rounds; ++k) {
    if (k == 0 && inject == INJECT_SKIP_SIGNAL) {
      // signal left out
    } else if (k == 0 && inject == INJECT_STALE_EPOCH) {
      Mem::store_release(trigger[k], epoch - 1);
    } else {
      Mem::store_release(trigger[k], epoch);
    }
    if (!wait_until<Mem>(&signals[k], CMP_GE, epoch, timeout_ns, seen)) {
      if (fail_round) *fail_round = k;
      return GICC_ETIMEDOUT;
    }
  }
  return GICC_OK;
}

// Counter barrier: every rank adds 1 to one shared counter (NVLS multimem.red on the GPU,
// a shared word on CPU ranks); barrier `epoch` completes when the counter reaches
// epoch * n.  `add` performs the release-add on the shared counter.
template <class Mem, class AddFn>
GICC_HD int counter_barrier(AddFn add, const uint64_t* local_counter, int n, uint64_t epoch, uint64_t timeout_ns,
                            uint64_t* seen, int inject = INJECT_NONE) {
  Mem::fence();
  if (inject == INJECT_NONE) add();  // both injections leave this rank's arrival out
  if (!wait_until<Mem>(local_counter, CMP_GE, epoch * (uint64_t)n, timeout_ns, seen)) return GICC_ETIMEDOUT;
  return GICC_OK;
}

}  // namespace proto
}  // namespace gicc
