// barrier.cpp -- host side of gicc::Barrier.
#include "gicc/barrier.hpp"

#include "gicc/config.hpp"

#include <chrono>
#include <cstring>
#include <thread>

#include "gicc/host_util.hpp"
#include "gicc/proto/barrier.hpp"

namespace gicc {

Barrier::Barrier(Runtime& rt, bool nvls) : rt_(rt) {
  nvls_ = nvls && rt.multicast_supported() && rt.signal_multicast(0) != nullptr;
  const int n = rt.size(), me = rt.rank();
  const int rounds = proto::n_rounds_for(n);
  if (rounds > GICC_MAX_ROUNDS) throw std::runtime_error("gicc::Barrier: too many ranks");
  // Allocation order is identical on every rank, so the offsets agree.
  const size_t off = rt.signal_alloc(GICC_MAX_ROUNDS + 1);
  BarrierCtx c;
  std::memset(&c, 0, sizeof(c));
  c.rank = me;
  c.size = n;
  c.n_signal_slots = 1;
  c.signals = rt.signal_local(off);
  if (nvls_) {
    c.n_rounds = 0;
    c.mc_counter = rt.signal_multicast(off + GICC_MAX_ROUNDS);
    c.mc_local = rt.signal_local(off + GICC_MAX_ROUNDS);
  } else {
    c.n_rounds = rounds;
    for (int k = 0; k < rounds; ++k) c.trigger_addrs[k] = rt.signal_peer((me + (1 << k)) % n, off + k);
  }
  c.expected_signal = 1;  // epoch of the first barrier
  void* h = nullptr;
  GICC_CUDA(cudaHostAlloc(&h, 2 * sizeof(uint64_t), cudaHostAllocMapped));
  std::memset(h, 0, 2 * sizeof(uint64_t));
  done_host_ = static_cast<uint64_t*>(h);
  void* d = nullptr;
  GICC_CUDA(cudaHostGetDevicePointer(&d, h, 0));
  c.done_counter = static_cast<uint64_t*>(d);
  c.ready_counter = static_cast<uint64_t*>(d) + 1;
  done_host_[1] = ~0ull;  // always "ready"
  c.err = rt.error_record();
  c.timeout_ns = rt.timeout_ns();
  GICC_CUDA(cudaMalloc(reinterpret_cast<void**>(&dctx_), sizeof(BarrierCtx)));
  GICC_CUDA(cudaMemcpy(dctx_, &c, sizeof(c), cudaMemcpyHostToDevice));
  rt.barrier();
}

Barrier::~Barrier() {
  try {
    finalize();
  } catch (...) {
  }
}

void Barrier::finalize() {
  if (finalized_) return;
  finalized_ = true;
  cudaDeviceSynchronize();
  if (dctx_) cudaFree(dctx_);
  if (done_host_) cudaFreeHost(done_host_);
  dctx_ = nullptr;
  done_host_ = nullptr;
}

void Barrier::setup() {
  NvtxRange nvtx("gicc::Barrier::setup");
  ++epoch_;
  GICC_CUDA(cudaMemcpy(&dctx_->expected_signal, &epoch_, sizeof(epoch_), cudaMemcpyHostToDevice));
  target_ = epoch_;
}

void Barrier::start_continuous(uint64_t n) {
  NvtxRange nvtx("gicc::Barrier::start_continuous");
  const uint64_t first = epoch_ + 1;
  GICC_CUDA(cudaMemcpy(&dctx_->expected_signal, &first, sizeof(first), cudaMemcpyHostToDevice));
  epoch_ += n;
  target_ = epoch_;
}

void Barrier::advance(uint64_t n) {
  epoch_ += n;
  target_ = epoch_;
}

void Barrier::wait_done(uint64_t target) {
  NvtxRange nvtx("gicc::Barrier::wait");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(rt_.timeout_ns());
  volatile uint64_t* d = done_host_;
  while (*d < target) {
    if (std::chrono::steady_clock::now() > deadline) {
      rt_.check_device_errors(false);
      throw std::runtime_error("gicc::Barrier: timed out waiting for barrier epoch " + std::to_string(target) +
                               " (done " + std::to_string(*d) + ")");
    }
    std::this_thread::yield();
  }
}

void Barrier::wait_completion() { wait_done(target_); }
void Barrier::wait_continuous() { wait_done(target_); }
void Barrier::inject_fault(int mode, uint64_t epoch, uint64_t timeout_ms) {
  if (mode < proto::INJECT_NONE || mode > proto::INJECT_STALE_EPOCH)
    throw std::runtime_error("gicc::Barrier::inject_fault: mode 0 (none), 1 (skip signal) or 2 (stale epoch)");
  BarrierCtx c;
  GICC_CUDA(cudaMemcpy(&c, dctx_, sizeof(c), cudaMemcpyDeviceToHost));
  c.inject_mode = mode;
  c.inject_epoch = epoch;
  if (timeout_ms) c.timeout_ns = timeout_ms * 1000000ull;
  GICC_CUDA(cudaMemcpy(dctx_, &c, sizeof(c), cudaMemcpyHostToDevice));
}

uint64_t Barrier::count() const { return done_host_ ? *reinterpret_cast<volatile uint64_t*>(done_host_) : 0; }

}  // namespace gicc
