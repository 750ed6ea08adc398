// barrier.hpp -- gicc::Barrier, the host side of the device barrier.
//
// Method set of the reference's gicc::Barrier (platform/ofi/internal/gicc_barrier.hpp:
// 57-300): init, finalize, setup, wait_completion, reset, start_continuous,
// wait_continuous, device_ctx, count.  The reference needs a monitor thread that re-queues
// NIC operations after every barrier (gicc_barrier.hpp:349-375); with epoch-valued NVLink
// signals nothing has to be re-armed, so setup() is one epoch bump, reset() is a no-op and
// continuous mode runs N barriers with zero host involvement.
#pragma once
#include <cstdint>

#include "gicc/runtime.hpp"

namespace gicc {

class GICC_EXPORT Barrier {
 public:
  // nvls: use the NVSwitch counter barrier (multimem.red) when the runtime has NVLS.
  explicit Barrier(Runtime& rt, bool nvls = false);
  ~Barrier();
  Barrier(const Barrier&) = delete;
  Barrier& operator=(const Barrier&) = delete;

  void init() {}  // nothing to start: no monitor thread is needed
  void finalize();
  void setup();                        // arm the next single barrier (host owns the epoch)
  void wait_completion();              // host wait (bounded) for the armed barrier
  void reset() {}                      // epochs are monotonic: nothing to reset
  void start_continuous(uint64_t n);   // hand the epoch to a kernel that runs n barriers
  void wait_continuous();              // host wait (bounded) until those n completed
  BarrierCtx* device_ctx() const { return dctx_; }
  // Record that n barriers were enqueued by stream-ordered kernels that advance the
  // device epoch themselves (ops::barrier_continuous); no device memory is touched.
  void advance(uint64_t n);
  uint64_t count() const;              // barriers completed on this rank
  // Failure-detection tests: at barrier number `epoch` (the value of expected_signal) this
  // rank leaves its signal out (mode 1) or sends a stale epoch (mode 2); peers then end
  // that barrier with GICC_ETIMEDOUT after timeout_ms (0 = keep the current bound).
  void inject_fault(int mode, uint64_t epoch, uint64_t timeout_ms = 0);
  uint64_t next_epoch() const { return epoch_ + 1; }
  bool uses_nvls() const { return nvls_; }

 private:
  void wait_done(uint64_t target);
  Runtime& rt_;
  BarrierCtx* dctx_ = nullptr;
  uint64_t* done_host_ = nullptr;
  uint64_t epoch_ = 0;   // last epoch handed out
  uint64_t target_ = 0;
  bool nvls_ = false;
  bool finalized_ = false;
};

}  // namespace gicc
