// gicc_barrier_test -- native C++ program using the runtime + device API directly (no
// Python): the counterpart of the reference's examples/ofi/barrier_test.cpp.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gicc_barrier_test [N]
//
// Test 1: single barrier per launch with host setup()/wait_completion() and a flag check.
// Test 2: continuous mode, N barriers in one kernel (the kernel advances expected_signal).
// Exit code 0 and "PASS" on every rank on success.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>

#include "gicc/barrier.hpp"
#include "gicc/device/comm.cuh"
#include "gicc/runtime.hpp"

__global__ void single_barrier_kernel(gicc::BarrierCtx* bctx, volatile uint64_t* flag) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (gicc::barrier(bctx) == gicc::GICC_OK) *flag = 42;
}

__global__ void continuous_barrier_kernel(gicc::BarrierCtx* bctx, int num_barriers, volatile uint64_t* counter) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  for (int i = 0; i < num_barriers; i++) {
    if (gicc::barrier(bctx) != gicc::GICC_OK) return;
    bctx->expected_signal++;
    *counter = i + 1;
  }
}

int main(int argc, char** argv) {
  const int nbar = argc > 1 ? std::atoi(argv[1]) : 10000;
  try {
    gicc::Runtime rt;
    const int rank = rt.rank(), n = rt.size();
    if (rank == 0) std::printf("gicc_barrier_test: %d ranks, GPU %d (%s)\n", n, rt.gpu_id(), rt.gpu_name());
    uint64_t* flag = nullptr;
    GICC_CUDA(cudaMalloc(&flag, 2 * sizeof(uint64_t)));
    GICC_CUDA(cudaMemset(flag, 0, 2 * sizeof(uint64_t)));
    gicc::Barrier barrier(rt);
    barrier.init();
    bool ok = true;
    // Test 1: ten single barriers, one kernel each
    for (int i = 0; i < 10; ++i) {
      barrier.setup();
      single_barrier_kernel<<<1, 32>>>(barrier.device_ctx(), flag);
      barrier.wait_completion();
      GICC_CUDA(cudaDeviceSynchronize());
      uint64_t f = 0;
      GICC_CUDA(cudaMemcpy(&f, flag, sizeof(f), cudaMemcpyDeviceToHost));
      ok = ok && f == 42;
      GICC_CUDA(cudaMemset(flag, 0, sizeof(uint64_t)));
    }
    // Test 2: continuous mode
    rt.barrier();
    barrier.start_continuous(nbar);
    cudaEvent_t s, e;
    cudaEventCreate(&s);
    cudaEventCreate(&e);
    cudaEventRecord(s);
    continuous_barrier_kernel<<<1, 32>>>(barrier.device_ctx(), nbar, flag + 1);
    cudaEventRecord(e);
    barrier.wait_continuous();
    GICC_CUDA(cudaDeviceSynchronize());
    float ms = 0;
    cudaEventElapsedTime(&ms, s, e);
    uint64_t c = 0;
    GICC_CUDA(cudaMemcpy(&c, flag + 1, sizeof(c), cudaMemcpyDeviceToHost));
    ok = ok && c == (uint64_t)nbar;
    rt.check_device_errors();
    std::printf("[rank %d] single x10: %s, continuous %d barriers: %.3f us/barrier, count %llu -> %s\n", rank,
                ok ? "ok" : "FAIL", nbar, 1e3 * ms / nbar, (unsigned long long)barrier.count(), ok ? "PASS" : "FAIL");
    barrier.finalize();
    cudaFree(flag);
    rt.finalize();
    return ok ? 0 : 1;
  } catch (const std::exception& ex) {
    std::fprintf(stderr, "gicc_barrier_test: %s\n", ex.what());
    return 2;
  }
}
