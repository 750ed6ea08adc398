// gicc_pingpong -- native ping-pong latency/bandwidth between ranks 0 and 1 using the
// reference-style device API (put through a DeviceCtx, signal, bounded wait): the
// counterpart of the reference's examples/gicc/pingpong_bench.cu.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gicc_pingpong [iters]
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>

#include "gicc/device/comm.cuh"
#include "gicc/runtime.hpp"

// One warp: put `size` bytes into the peer (DeviceCtx API, warp scope), release the peer's
// flag, wait for the echo.  %globaltimer brackets the loop.
__global__ void pingpong_kernel(gicc::DeviceCtx* ctx, uint64_t laddr, uint32_t size, uint64_t* remote_flag,
                                const uint64_t* local_flag, int iters, int initiator, uint64_t base,
                                unsigned long long* out_ns) {
  const int lane = threadIdx.x & 31;
  unsigned long long t0 = 0;
  if (lane == 0) t0 = gicc::ptx::globaltimer();
  for (int i = 0; i < iters; ++i) {
    const uint64_t ping = base + 2 * (uint64_t)i + 1, pong = ping + 1;
    if (!initiator) {
      int st = 0;
      if (lane == 0) st = gicc::signal_wait_until(local_flag, gicc::proto::CMP_GE, ping, ctx->timeout_ns, ctx->err);
      if (__shfl_sync(0xffffffffu, st, 0)) return;
    }
    gicc::put<gicc::Scope::Warp>(ctx, laddr, 0, size);  // to the default remote buffer
    gicc::ptx::fence_acq_rel_sys();
    __syncwarp();
    if (lane == 0) gicc::signal_set(remote_flag, initiator ? ping : pong);
    if (initiator) {
      int st = 0;
      if (lane == 0) st = gicc::signal_wait_until(local_flag, gicc::proto::CMP_GE, pong, ctx->timeout_ns, ctx->err);
      if (__shfl_sync(0xffffffffu, st, 0)) return;
    }
  }
  if (lane == 0) *out_ns = gicc::ptx::globaltimer() - t0;
}

int main(int argc, char** argv) {
  const int iters = argc > 1 ? std::atoi(argv[1]) : 1000;
  try {
    gicc::Runtime rt;
    const int rank = rt.rank(), n = rt.size();
    if (n < 2) {
      std::fprintf(stderr, "gicc_pingpong needs 2 ranks\n");
      return 1;
    }
    const size_t max_size = 1 << 22;
    gicc::Buffer buf = rt.alloc(max_size);
    rt.exchange();
    const size_t flag_off = rt.signal_alloc(1);
    const int peer = rank == 0 ? 1 : 0;
    gicc::DeviceCtx* ctx = rt.prepare(peer, buf.index);
    unsigned long long* out = nullptr;
    GICC_CUDA(cudaMalloc(&out, sizeof(*out)));
    uint64_t base = 0;
    if (rank == 0) std::printf("%10s %14s %12s\n", "bytes", "half-RTT(us)", "GB/s");
    for (size_t size = 8; size <= max_size; size *= 8) {
      rt.barrier();
      if (rank < 2)
        pingpong_kernel<<<1, 32>>>(ctx, (uint64_t)(uintptr_t)buf.ptr, (uint32_t)size, rt.signal_peer(peer, flag_off),
                                   rt.signal_local(flag_off), iters, rank == 0, base, out);
      GICC_CUDA(cudaDeviceSynchronize());
      base += 2 * (uint64_t)iters;
      unsigned long long ns = 0;
      GICC_CUDA(cudaMemcpy(&ns, out, sizeof(ns), cudaMemcpyDeviceToHost));
      if (rank == 0) {
        const double half = (double)ns / iters / 2.0;
        std::printf("%10zu %14.3f %12.3f\n", size, half / 1e3, size / half);
      }
    }
    rt.check_device_errors();
    cudaFree(out);
    rt.finalize();
    if (rank == 0) std::printf("PASS\n");
    return 0;
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "gicc_pingpong: %s\n", ex.what());
    return 2;
  }
}
