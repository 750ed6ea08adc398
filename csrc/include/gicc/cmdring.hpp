// cmdring.hpp -- gicc::CmdRing: host-queued puts / gets / signals executed on the GPU by a
// persistent one-CTA kernel (the reference's command-ring kernel, persistent.cuh:239-311,
// rebuilt on NVLink peer mappings; protocol in gicc/proto/cmdring.hpp).
//
// Use it when a host thread issues many small transfers: one kernel launch serves them all
// and each command costs a PCIe write of 64 bytes instead of a launch.  The kernel exits on
// stop() or after idle_timeout_ms without commands (status() then reports ETIMEDOUT);
// start() launches it again, and stop() drops commands the kernel did not reach.  Commands
// complete in order; wait(seq) covers seq and all before it.
//
// While the ring kernel is resident, the first launch of a kernel that this process has not
// loaded yet (CUDA lazy module loading, the default) waits until the ring kernel exits.
// Launch such kernels once before start(), or run with CUDA_MODULE_LOADING=EAGER.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "gicc/proto/cmdring.hpp"
#include "gicc/runtime.hpp"

namespace gicc {

class GICC_EXPORT CmdRing {
 public:
  explicit CmdRing(Runtime& rt, int nslots = 64, int threads = 256, uint64_t idle_timeout_ms = 10000);
  ~CmdRing();
  CmdRing(const CmdRing&) = delete;
  CmdRing& operator=(const CmdRing&) = delete;

  void start();  // launch the persistent kernel (on its own stream)
  uint64_t put(const void* src_local, int dst_rank, int dst_buf, size_t dst_off, size_t size, uint64_t user = 0);
  uint64_t get(void* dst_local, int src_rank, int src_buf, size_t src_off, size_t size, uint64_t user = 0);
  uint64_t signal(int dst_rank, size_t word, uint64_t value);  // signal-heap word := value (release)
  uint64_t add(int dst_rank, size_t word, uint64_t value);     // signal-heap word += value (release)
  uint64_t fence();
  void wait(uint64_t seq);        // bounded host wait until command seq finished
  uint64_t completed() const;     // commands finished so far
  void stop();                    // EXIT, then wait for the kernel
  int status() const;             // GICC_OK, GICC_ETIMEDOUT (idle exit), or -1 while running
  bool running() const { return running_; }

 private:
  uint64_t push(const proto::Command& c);
  Runtime& rt_;
  proto::CmdRingView view_{};  // host pointers
  proto::CmdRingView dview_{}; // the same memory, device pointers
  void* host_mem_ = nullptr;
  int threads_;
  uint64_t next_ = 0;
  cudaStream_t stream_ = nullptr;
  bool running_ = false;
};

}  // namespace gicc
