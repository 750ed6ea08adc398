// examples.cu -- kernels of the reference's measurement programs, rebuilt for NVLink:
//
// * k_phase_loop: the barrier / put / barrier / compute / verify / barrier loop of
//   legacy/ofi/prototype/barrier_put_compute_verify.cpp:465-626, one block per GPU, with a
//   %globaltimer stamp after every phase of every iteration (the host turns them into
//   mean / std / min / max / p50 / p90 / p99 per phase).
// * k_saxpy_put: "compute, then put" fused per CTA (gda-comp.cpp:95-135 runs a SAXPY before
//   a GPU-triggered transfer): each CTA computes y = a*x + y on its chunk, stores the chunk
//   into the peer's buffer and adds one to the peer's arrival counter -- no grid-wide sync.
#include <cuda_runtime.h>

#include "gicc/config.hpp"
#include "gicc/device/comm.cuh"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace {

__device__ __forceinline__ float phase_value(int it, int rank, size_t i) {
  return (float)((it * 7 + rank * 13 + (int)(i % 97)) & 1023);
}

// stamps: [iters][6] = start, after barrier 1, after put + barrier 2, after compute,
// after verify, after barrier 3.
__global__ void __launch_bounds__(1024) k_phase_loop(BarrierCtx* bar, float* x, float* y, const float* recv,
                                                     float* send_remote, size_t n, int iters, float a, int rank,
                                                     int left, uint64_t* stamps, unsigned long long* bad) {
  __shared__ int st;
  auto stamp = [&](int it, int k) {
    if (threadIdx.x == 0) stamps[(size_t)it * 6 + k] = ptx::globaltimer();
  };
  auto barrier = [&]() -> bool {
    ptx::fence_acq_rel_sys();
    __syncthreads();
    if (threadIdx.x == 0) {
      st = gicc::barrier(bar, false);
      bar->expected_signal += 1;
    }
    __syncthreads();
    return st == GICC_OK;
  };
  for (int it = 0; it < iters; ++it) {
    stamp(it, 0);
    if (!barrier()) return;
    stamp(it, 1);
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {  // put: this iteration's data
      const float v = phase_value(it, rank, i);
      x[i] = v;
      send_remote[i] = v;
    }
    if (!barrier()) return;
    stamp(it, 2);
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) y[i] = a * x[i] + y[i];  // compute: SAXPY
    __syncthreads();
    stamp(it, 3);
    unsigned long long mine = 0;  // verify what the left neighbour put
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) mine += recv[i] != phase_value(it, left, i);
    if (mine) atomicAdd(bad, mine);
    __syncthreads();
    stamp(it, 4);
    if (!barrier()) return;
    stamp(it, 5);
  }
  if (threadIdx.x == 0) *reinterpret_cast<volatile uint64_t*>(bar->done_counter) = bar->expected_signal - 1;
}

__global__ void __launch_bounds__(512) k_saxpy_put(const float* x, float* y, float a, size_t n, float* dst_remote,
                                                   uint64_t* arrivals_remote) {
  const size_t chunk = (n + gridDim.x - 1) / gridDim.x;
  const size_t lo = (size_t)blockIdx.x * chunk, hi = min(n, lo + chunk);
  for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    const float v = a * x[i] + y[i];
    y[i] = v;
    dst_remote[i] = v;
  }
  ptx::fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) ptx::red_release_sys_add(arrivals_remote, 1);
}

__global__ void k_wait_count(const uint64_t* counter, uint64_t target, uint64_t timeout_ns, ErrorRecord* err, int rank) {
  uint64_t seen = 0;
  if (!proto::wait_until<proto::DevMem>(counter, proto::CMP_GE, target, timeout_ns, &seen))
    report_error(err, GICC_ETIMEDOUT, W_SIGNAL_WAIT, rank, -1, seen, target);
}

// Bulk tile put: each CTA writes a `tile_bytes` pattern tile into shared memory, one thread
// puts it to dst + blockIdx.x * tile_bytes with put_tile, waits, and releases `sig` (+1).
__global__ void __launch_bounds__(256) k_put_tile(uint8_t* dst, uint32_t tile_bytes, uint32_t seed, uint64_t* sig) {
  extern __shared__ __align__(16) uint8_t tile[];
  const size_t base = (size_t)blockIdx.x * tile_bytes;
  for (uint32_t j = threadIdx.x; j < tile_bytes; j += blockDim.x) {  // the byte pattern of k_fill / k_check
    const size_t i = base + j;
    tile[j] = (uint8_t)((seed * 2654435761u + (uint32_t)i * 40503u + (uint32_t)(i >> 16)) >> 13);
  }
  fence_tile_for_put();
  __syncthreads();
  if (threadIdx.x == 0) {
    put_tile(dst + base, tile, tile_bytes);
    put_tile_wait();
    quiet();
    if (sig) signal_add(sig, 1);
  }
}

__global__ void k_saxpy(const float* x, float* y, float a, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    y[i] = a * x[i] + y[i];
}

}  // namespace

namespace ops {

void phase_loop(BarrierCtx* bar, float* x, float* y, const float* recv, float* send_remote, size_t n, int iters,
                float a, int rank, int left, uint64_t* stamps, unsigned long long* bad, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::phase_loop");
  k_phase_loop<<<1, 1024, 0, s>>>(bar, x, y, recv, send_remote, n, iters, a, rank, left, stamps, bad);
  GICC_CUDA(cudaGetLastError());
}

void saxpy_put(const float* x, float* y, float a, size_t n, float* dst_remote, uint64_t* arrivals_remote, int blocks,
               cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::saxpy_put");
  k_saxpy_put<<<blocks, 512, 0, s>>>(x, y, a, n, dst_remote, arrivals_remote);
  GICC_CUDA(cudaGetLastError());
}

void wait_count(const uint64_t* counter, uint64_t target, uint64_t timeout_ns, int rank, cudaStream_t s) {
  k_wait_count<<<1, 1, 0, s>>>(counter, target, timeout_ns, device_error_record(), rank);
  GICC_CUDA(cudaGetLastError());
}

void put_tile_test(void* dst, int tiles, uint32_t tile_bytes, uint32_t seed, uint64_t* sig, cudaStream_t s) {
  if (tile_bytes == 0 || tile_bytes % 16 || tile_bytes > 96 * 1024 || (reinterpret_cast<uintptr_t>(dst) & 15))
    throw std::runtime_error("gicc::put_tile_test: 16-byte aligned dst, tile_bytes a multiple of 16 up to 96 KiB");
  if (tile_bytes > 48 * 1024)
    GICC_CUDA(cudaFuncSetAttribute(k_put_tile, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)tile_bytes));
  k_put_tile<<<tiles, 256, tile_bytes, s>>>(static_cast<uint8_t*>(dst), tile_bytes, seed, sig);
  GICC_CUDA(cudaGetLastError());
}

void saxpy(const float* x, float* y, float a, size_t n, cudaStream_t s) {
  k_saxpy<<<4 * num_sms(), 256, 0, s>>>(x, y, a, n);
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
