// comm.cu -- communication kernels: barrier (single / continuous), put/get bandwidth,
// ping-pong, quiet latency, queued-op flush, pattern fill/check.
//
// Counterparts of the reference kernels listed in its examples and device headers:
// barrier_test.cpp:20-41 (single/continuous barrier), pingpong_bench.cu:33-79,
// device_opt.cuh:673-796 (burst/multi-WQE puts), gda_put_bw.cpp:75 (windowed put BW),
// benchmark.cpp:41-83 and put_example.cpp:33-70 (pattern init/verify).
#include <cuda_runtime.h>

#include "gicc/device/comm.cuh"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace {

__global__ void k_barrier_single(BarrierCtx* ctx, uint64_t* flag) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (barrier(ctx) != GICC_OK) return;
  ctx->expected_signal++;  // stream-ordered use needs no host re-arm; setup() may still set it
  if (flag) *reinterpret_cast<volatile uint64_t*>(flag) = 42;
}

__global__ void k_barrier_continuous(BarrierCtx* ctx, int n, uint64_t* counter) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int i = 0; i < n; ++i) {
    const uint64_t epoch = ctx->expected_signal;
    if (barrier(ctx, false) != GICC_OK) return;
    ctx->expected_signal++;
    if (counter) *reinterpret_cast<volatile uint64_t*>(counter) = i + 1;
    if (i == n - 1 || (i & 1023) == 1023) *reinterpret_cast<volatile uint64_t*>(ctx->done_counter) = epoch;
  }
}

// Grid-wide copy repeated `iters` times; the final fence makes every store performed at
// system scope before the kernel ends, so kernel time == delivery time.
// window_vec > nvec: repetition `it` works on a different part of a window of window_vec
// vectors (both sides), so repeated small copies do not just hit cached lines.
__global__ void __launch_bounds__(512) k_copy(uint4* dst_base, const uint4* src_base, size_t nvec, int iters,
                                              size_t window_vec) {
  const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const size_t span = window_vec > nvec ? window_vec - nvec + 1 : 1;
  for (int it = 0; it < iters; ++it) {
    const size_t off = ((size_t)it * nvec) % span;
    uint4* dst = dst_base + off;
    const uint4* src = src_base + off;
    size_t i = tid;
    for (; i + 3 * stride < nvec; i += 4 * stride) {
      const uint4 a = src[i], b = src[i + stride], c = src[i + 2 * stride], d = src[i + 3 * stride];
      dst[i] = a;
      dst[i + stride] = b;
      dst[i + 2 * stride] = c;
      dst[i + 3 * stride] = d;
    }
    for (; i < nvec; i += stride) dst[i] = src[i];
  }
  ptx::fence_acq_rel_sys();
}

__global__ void k_copy_bytes(char* dst, const char* src, size_t n, int iters) {
  for (int it = 0; it < iters; ++it)
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
      dst[i] = src[i];
  ptx::fence_acq_rel_sys();
}

// Each block puts its slice and then adds 1 to the peer's signal (release).
__global__ void __launch_bounds__(512) k_put_signal(char* dst, const char* src, size_t bytes, uint64_t* sig) {
  const size_t per = (bytes + gridDim.x - 1) / gridDim.x;
  const size_t lo = per * blockIdx.x;
  const size_t hi = lo + per < bytes ? lo + per : bytes;
  if (lo < hi) copy_bytes<Scope::Block>(dst + lo, src + lo, hi - lo);
  ptx::fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) ptx::red_release_sys_add(sig, 1);
}

__global__ void k_wait_signal(const uint64_t* sig, int cmp, uint64_t value, ErrorRecord* err, uint64_t timeout_ns,
                              int* status) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const int st = signal_wait_until(sig, cmp, value, timeout_ns, err);
  if (status) *status = st;
}

__global__ void k_signal(uint64_t* sig, uint64_t value, int op) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  ptx::fence_acq_rel_sys();
  if (op == SIGNAL_ADD)
    ptx::red_release_sys_add(sig, value);
  else
    ptx::st_release_sys(sig, value);
}

// One warp per side.  Initiator: put, signal, wait for the echo; responder mirrors it.
__global__ void k_pingpong(char* remote_buf, const char* local_buf, size_t bytes, uint64_t* remote_flag,
                           const uint64_t* local_flag, int iters, int initiator, uint64_t base, uint64_t* out_ns,
                           ErrorRecord* err, uint64_t timeout_ns, int rank) {
  const int lane = threadIdx.x & 31;
  uint64_t t0 = 0;
  if (lane == 0) t0 = ptx::globaltimer();
  for (int i = 0; i < iters; ++i) {
    const uint64_t ping = base + 2 * (uint64_t)i + 1, pong = ping + 1;
    if (initiator) {
      put_signal<Scope::Warp>(remote_buf, local_buf, bytes, remote_flag, ping);
      int st = GICC_OK;
      if (lane == 0) st = signal_wait_until(local_flag, proto::CMP_GE, pong, timeout_ns, err, rank, -1, W_PINGPONG);
      st = __shfl_sync(0xffffffffu, st, 0);
      if (st != GICC_OK) return;
    } else {
      int st = GICC_OK;
      if (lane == 0) st = signal_wait_until(local_flag, proto::CMP_GE, ping, timeout_ns, err, rank, -1, W_PINGPONG);
      st = __shfl_sync(0xffffffffu, st, 0);
      if (st != GICC_OK) return;
      put_signal<Scope::Warp>(remote_buf, local_buf, bytes, remote_flag, pong);
    }
  }
  if (lane == 0 && out_ns) *out_ns = ptx::globaltimer() - t0;
}

// Same protocol with a whole CTA moving the message (large sizes).
__global__ void __launch_bounds__(1024) k_pingpong_block(char* remote_buf, const char* local_buf, size_t bytes,
                                                         uint64_t* remote_flag, const uint64_t* local_flag, int iters,
                                                         int initiator, uint64_t base, uint64_t* out_ns,
                                                         ErrorRecord* err, uint64_t timeout_ns, int rank) {
  __shared__ int st;
  uint64_t t0 = 0;
  if (threadIdx.x == 0) t0 = ptx::globaltimer();
  for (int i = 0; i < iters; ++i) {
    const uint64_t ping = base + 2 * (uint64_t)i + 1, pong = ping + 1;
    if (initiator) put_signal<Scope::Block>(remote_buf, local_buf, bytes, remote_flag, ping);
    if (threadIdx.x == 0)
      st = signal_wait_until(local_flag, proto::CMP_GE, initiator ? pong : ping, timeout_ns, err, rank, -1, W_PINGPONG);
    __syncthreads();
    if (st != GICC_OK) return;
    if (!initiator) put_signal<Scope::Block>(remote_buf, local_buf, bytes, remote_flag, pong);
  }
  if (threadIdx.x == 0 && out_ns) *out_ns = ptx::globaltimer() - t0;
}

// Reference-signature put through a DeviceCtx (one warp), then quiet.
__global__ void k_ctx_put(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey,
                          uint32_t size) {
  put<Scope::Warp>(ctx, laddr, lkey, raddr, rkey, size);
  quiet();
}

// put(8 B) + quiet() per iteration, timed on the device.
__global__ void k_quiet_latency(uint64_t* remote, int iters, uint64_t* out_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = ptx::globaltimer();
  for (int i = 0; i < iters; ++i) {
    *reinterpret_cast<volatile uint64_t*>(remote) = (uint64_t)i;
    quiet();
  }
  *out_ns = ptx::globaltimer() - t0;
}

__global__ void k_flush(DeviceCtx* ctx, int* status) {
  flush<Scope::Block>(ctx);
  if (threadIdx.x == 0) {
    const int st = quiet(ctx);
    if (status) *status = st;
  }
}

// Byte pattern (seed + i*mult) -- unique per iteration/stream like the reference's
// (iter + 0xA0 + i) & 0xFF verification (examples/ofi/benchmark.cpp:119-130).
__global__ void k_fill(uint8_t* buf, size_t n, uint32_t seed) {
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    buf[i] = (uint8_t)((seed * 2654435761u + (uint32_t)i * 40503u + (uint32_t)(i >> 16)) >> 13);
}
__global__ void k_check(const uint8_t* buf, size_t n, uint32_t seed, size_t base, unsigned long long* bad) {
  unsigned long long local = 0;
  for (size_t j = (size_t)blockIdx.x * blockDim.x + threadIdx.x; j < n; j += (size_t)gridDim.x * blockDim.x) {
    const size_t i = base + j;  // index in the filled buffer
    const uint8_t e = (uint8_t)((seed * 2654435761u + (uint32_t)i * 40503u + (uint32_t)(i >> 16)) >> 13);
    local += buf[j] != e;
  }
  if (local) atomicAdd(bad, local);
}

}  // namespace

namespace ops {

void barrier_single(BarrierCtx* ctx, uint64_t* flag, cudaStream_t s) {
  k_barrier_single<<<1, 32, 0, s>>>(ctx, flag);
  GICC_CUDA(cudaGetLastError());
}
void barrier_continuous(BarrierCtx* ctx, int n, uint64_t* counter, cudaStream_t s) {
  k_barrier_continuous<<<1, 32, 0, s>>>(ctx, n, counter);
  GICC_CUDA(cudaGetLastError());
}
void copy(void* dst, const void* src, size_t bytes, int iters, int blocks, int threads, cudaStream_t s,
          size_t window) {
  if (bytes == 0) return;
  if (blocks <= 0) blocks = 2 * num_sms();
  if (threads <= 0) threads = 512;
  if ((((uintptr_t)dst | (uintptr_t)src | bytes) & 15) == 0) {
    const size_t nvec = bytes / 16;
    const size_t need = (nvec + threads - 1) / threads;
    if ((size_t)blocks > need) blocks = (int)need;
    k_copy<<<blocks, threads, 0, s>>>(static_cast<uint4*>(dst), static_cast<const uint4*>(src), nvec, iters,
                                      window / 16);
  } else {
    const size_t need = (bytes + threads - 1) / threads;
    if ((size_t)blocks > need) blocks = (int)need;
    k_copy_bytes<<<blocks, threads, 0, s>>>(static_cast<char*>(dst), static_cast<const char*>(src), bytes, iters);
  }
  GICC_CUDA(cudaGetLastError());
}
void put_signal(void* dst, const void* src, size_t bytes, uint64_t* sig_remote, int blocks, cudaStream_t s) {
  if (blocks <= 0) blocks = num_sms();
  k_put_signal<<<blocks, 512, 0, s>>>(static_cast<char*>(dst), static_cast<const char*>(src), bytes, sig_remote);
  GICC_CUDA(cudaGetLastError());
}
void wait_signal(const uint64_t* sig, int cmp, uint64_t value, uint64_t timeout_ns, int* status, cudaStream_t s) {
  k_wait_signal<<<1, 32, 0, s>>>(sig, cmp, value, device_error_record(), timeout_ns, status);
  GICC_CUDA(cudaGetLastError());
}
void signal(uint64_t* sig, uint64_t value, int op, cudaStream_t s) {
  k_signal<<<1, 32, 0, s>>>(sig, value, op);
  GICC_CUDA(cudaGetLastError());
}
void pingpong(void* remote_buf, const void* local_buf, size_t bytes, uint64_t* remote_flag, const uint64_t* local_flag,
              int iters, bool initiator, uint64_t base, uint64_t* out_ns, uint64_t timeout_ns, int rank,
              cudaStream_t s) {
  if (bytes >= 16384)
    k_pingpong_block<<<1, 1024, 0, s>>>(static_cast<char*>(remote_buf), static_cast<const char*>(local_buf), bytes,
                                        remote_flag, local_flag, iters, initiator ? 1 : 0, base, out_ns,
                                        device_error_record(), timeout_ns, rank);
  else
    k_pingpong<<<1, 32, 0, s>>>(static_cast<char*>(remote_buf), static_cast<const char*>(local_buf), bytes,
                                remote_flag, local_flag, iters, initiator ? 1 : 0, base, out_ns, device_error_record(),
                                timeout_ns, rank);
  GICC_CUDA(cudaGetLastError());
}
void quiet_latency(uint64_t* remote, int iters, uint64_t* out_ns, cudaStream_t s) {
  k_quiet_latency<<<1, 32, 0, s>>>(remote, iters, out_ns);
  GICC_CUDA(cudaGetLastError());
}
void ctx_put(DeviceCtx* ctx, uint64_t laddr, uint32_t lkey, uint64_t raddr, uint32_t rkey, uint32_t size,
             cudaStream_t s) {
  k_ctx_put<<<1, 32, 0, s>>>(ctx, laddr, lkey, raddr, rkey, size);
  GICC_CUDA(cudaGetLastError());
}
void flush_queued(DeviceCtx* ctx, int* status, cudaStream_t s) {
  k_flush<<<1, 512, 0, s>>>(ctx, status);
  GICC_CUDA(cudaGetLastError());
}
void fill_pattern(void* buf, size_t n, uint32_t seed, cudaStream_t s) {
  if (!n) return;
  k_fill<<<2 * num_sms(), 256, 0, s>>>(static_cast<uint8_t*>(buf), n, seed);
  GICC_CUDA(cudaGetLastError());
}
void check_pattern(const void* buf, size_t n, uint32_t seed, unsigned long long* bad, cudaStream_t s, size_t base) {
  if (!n) return;
  k_check<<<2 * num_sms(), 256, 0, s>>>(static_cast<const uint8_t*>(buf), n, seed, base, bad);
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
