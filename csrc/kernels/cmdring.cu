// cmdring.cu -- the persistent command-ring kernel and gicc::CmdRing (gicc/cmdring.hpp).
#include "gicc/cmdring.hpp"

#include <chrono>
#include <cstring>
#include <stdexcept>
#include <thread>

#include "gicc/config.hpp"
#include "gicc/device/ptx.cuh"
#include "gicc/host_util.hpp"

namespace gicc {
namespace {

using proto::Command;
using proto::DevMem;

__device__ __forceinline__ void block_copy(const Command& c) {
  const uintptr_t s = c.src, d = c.dst;
  if (((s | d | c.size) & 15) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(s);
    uint4* dst = reinterpret_cast<uint4*>(d);
    for (uint64_t i = threadIdx.x; i < c.size / 16; i += blockDim.x) ptx::st_v4(dst + i, ptx::ld_v4(src + i));
  } else {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(s);
    uint8_t* dst = reinterpret_cast<uint8_t*>(d);
    for (uint64_t i = threadIdx.x; i < c.size; i += blockDim.x) dst[i] = src[i];
  }
}

__global__ void k_cmdring(proto::CmdRingView v, uint64_t first) {
  __shared__ Command cmd;
  __shared__ int go;
  for (uint64_t i = first;; ++i) {
    if (threadIdx.x == 0) {
      go = proto::cmdring_next<DevMem>(v, i, &cmd) ? 1 : 0;
      if (!go) ptx::st_release_sys(v.status, (uint64_t)GICC_ETIMEDOUT);
    }
    __syncthreads();
    if (!go) return;
    if (cmd.op == proto::CMD_EXIT) {
      if (threadIdx.x == 0) {
        proto::cmdring_complete<DevMem>(v, i);
        ptx::st_release_sys(v.status, (uint64_t)GICC_OK);
      }
      return;
    }
    switch (cmd.op) {
      case proto::CMD_PUT:
      case proto::CMD_GET:
        block_copy(cmd);
        break;
      case proto::CMD_SIGNAL:
        if (threadIdx.x == 0) ptx::st_release_sys(reinterpret_cast<uint64_t*>(cmd.dst), cmd.value);
        break;
      case proto::CMD_ADD:
        if (threadIdx.x == 0) ptx::red_release_sys_add(reinterpret_cast<uint64_t*>(cmd.dst), cmd.value);
        break;
      default:  // CMD_FENCE, CMD_NOP
        break;
    }
    ptx::fence_acq_rel_sys();  // this thread's stores of the command are performed
    __syncthreads();
    if (threadIdx.x == 0) proto::cmdring_complete<DevMem>(v, i);
    __syncthreads();           // cmd is rewritten by the next iteration
  }
}

}  // namespace

CmdRing::CmdRing(Runtime& rt, int nslots, int threads, uint64_t idle_timeout_ms) : rt_(rt), threads_(threads) {
  if (nslots < 2 || threads < 32 || threads > 1024 || threads % 32)
    throw std::runtime_error("gicc::CmdRing: nslots >= 2, threads a multiple of 32 in [32, 1024]");
  const size_t bytes = (size_t)nslots * sizeof(Command) + 128;
  GICC_CUDA(cudaHostAlloc(&host_mem_, bytes, cudaHostAllocMapped | cudaHostAllocPortable));
  std::memset(host_mem_, 0, bytes);
  void* d = nullptr;
  GICC_CUDA(cudaHostGetDevicePointer(&d, host_mem_, 0));
  auto carve = [&](void* base, proto::CmdRingView& v) {
    v.cmds = static_cast<Command*>(base);
    v.nslots = nslots;
    v.done = reinterpret_cast<uint64_t*>(static_cast<uint8_t*>(base) + (size_t)nslots * sizeof(Command));
    v.status = v.done + 8;  // own cache line
    v.idle_timeout_ns = idle_timeout_ms * 1000000ull;
  };
  carve(host_mem_, view_);
  carve(d, dview_);
  *view_.status = ~0ull;
  GICC_CUDA(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
}

CmdRing::~CmdRing() {
  try {
    stop();
  } catch (...) {
  }
  if (stream_) cudaStreamDestroy(stream_);
  if (host_mem_) cudaFreeHost(host_mem_);
}

void CmdRing::start() {
  NvtxRange nvtx("gicc::CmdRing::start");
  if (running_) return;
  __atomic_store_n(view_.status, ~0ull, __ATOMIC_RELEASE);
  k_cmdring<<<1, threads_, 0, stream_>>>(dview_, __atomic_load_n(view_.done, __ATOMIC_ACQUIRE));
  GICC_CUDA(cudaGetLastError());
  running_ = true;
}

uint64_t CmdRing::push(const Command& c) {
  if (!running_) throw std::runtime_error("gicc::CmdRing: start() the ring first");
  const uint64_t seq = proto::cmdring_push<proto::HostMem>(view_, next_, c, rt_.timeout_ns());
  if (!seq) throw std::runtime_error("gicc::CmdRing: no free slot in time (is the ring kernel running?)");
  ++next_;
  return seq;
}

uint64_t CmdRing::put(const void* src_local, int dst_rank, int dst_buf, size_t dst_off, size_t size, uint64_t user) {
  Command c{};
  c.op = proto::CMD_PUT;
  c.src = reinterpret_cast<uint64_t>(src_local);
  c.dst = reinterpret_cast<uint64_t>(rt_.remote_ptr(dst_rank, dst_buf, dst_off));
  c.size = size;
  c.user = user;
  if (dst_off + size > rt_.buffer(dst_buf).size) throw std::runtime_error("gicc::CmdRing::put: outside the buffer");
  return push(c);
}

uint64_t CmdRing::get(void* dst_local, int src_rank, int src_buf, size_t src_off, size_t size, uint64_t user) {
  Command c{};
  c.op = proto::CMD_GET;
  c.src = reinterpret_cast<uint64_t>(rt_.remote_ptr(src_rank, src_buf, src_off));
  c.dst = reinterpret_cast<uint64_t>(dst_local);
  c.size = size;
  c.user = user;
  if (src_off + size > rt_.buffer(src_buf).size) throw std::runtime_error("gicc::CmdRing::get: outside the buffer");
  return push(c);
}

uint64_t CmdRing::signal(int dst_rank, size_t word, uint64_t value) {
  Command c{};
  c.op = proto::CMD_SIGNAL;
  c.dst = reinterpret_cast<uint64_t>(rt_.signal_peer(dst_rank, word));
  c.value = value;
  return push(c);
}

uint64_t CmdRing::add(int dst_rank, size_t word, uint64_t value) {
  Command c{};
  c.op = proto::CMD_ADD;
  c.dst = reinterpret_cast<uint64_t>(rt_.signal_peer(dst_rank, word));
  c.value = value;
  return push(c);
}

uint64_t CmdRing::fence() {
  Command c{};
  c.op = proto::CMD_FENCE;
  return push(c);
}

uint64_t CmdRing::completed() const { return __atomic_load_n(view_.done, __ATOMIC_ACQUIRE); }

int CmdRing::status() const {
  const uint64_t s = __atomic_load_n(view_.status, __ATOMIC_ACQUIRE);
  return s == ~0ull ? -1 : (int)s;
}

void CmdRing::wait(uint64_t seq) {
  NvtxRange nvtx("gicc::CmdRing::wait");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(rt_.timeout_ns());
  while (completed() < seq) {
    if (status() >= 0) throw std::runtime_error("gicc::CmdRing::wait: the ring kernel exited (idle timeout or stop)");
    if (std::chrono::steady_clock::now() > deadline) throw std::runtime_error("gicc::CmdRing::wait: timed out");
    std::this_thread::yield();
  }
}

void CmdRing::stop() {
  if (!running_) return;
  if (status() < 0) {
    Command c{};
    c.op = proto::CMD_EXIT;
    proto::cmdring_push<proto::HostMem>(view_, next_, c, rt_.timeout_ns());
    ++next_;
  }
  GICC_CUDA(cudaStreamSynchronize(stream_));  // the kernel returns on EXIT or after its idle bound
  // Commands the kernel did not reach (it can only be the EXIT, or commands queued after an
  // idle exit) are dropped, so the next start() begins at an empty ring.
  __atomic_store_n(view_.done, next_, __ATOMIC_RELEASE);
  running_ = false;
}

}  // namespace gicc
