// gicc_queued_put -- the host-queued put path (OFI semantics: Runtime::put_no_db queues a
// transfer, prepare_trigger hands the batch to the GPU, a kernel's flush() runs it, and
// Runtime::wait confirms each op), as in the reference's examples/ofi/test_gicc.cpp (queue,
// flush, quiet, verify) and examples/ofi/benchmark.cpp (32 streams per batch, a byte pattern
// unique per iteration and stream, so a partial or missing write shows up without
// re-initialising the receiver).
//
// Every rank queues 32 puts ("streams") of `-size` bytes from its source buffer into its
// right neighbour's destination buffer per iteration; one block-scope flush kernel runs
// them; the host waits for every token; after a barrier each rank checks what its left
// neighbour wrote.  Reports the batch time (CUDA events around the flush, max over ranks)
// and PASS/FAIL.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gicc_queued_put [-size 1048576] [-iters 20]
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "gicc/coll.hpp"
#include "gicc/device/comm.cuh"
#include "gicc/host_util.hpp"
#include "gicc/runtime.hpp"

namespace {

constexpr int kStreams = gicc::GICC_POOL_SIZE;  // ops per batch

long long arg_ll(int argc, char** argv, const char* name, long long def) {
  for (int i = 1; i + 1 < argc; ++i)
    if (!std::strcmp(argv[i], name)) return std::atoll(argv[i + 1]);
  return def;
}

__host__ __device__ inline uint8_t pattern(int iter, int stream, size_t i) {
  return (uint8_t)((iter + 0xA0 + stream + i * 13) & 0xFF);
}

__global__ void fill(uint8_t* src, size_t size, int iter) {
  const size_t n = size * kStreams;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    src[i] = pattern(iter, (int)(i / size), i % size);
}

__global__ void check(const uint8_t* dst, size_t size, int iter, unsigned long long* bad) {
  const size_t n = size * kStreams;
  unsigned long long mine = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    mine += dst[i] != pattern(iter, (int)(i / size), i % size);
  if (mine) atomicAdd(bad, mine);
}

// one block runs the whole batch (block-scope copies), then waits for its completion words
__global__ void __launch_bounds__(1024) flush_kernel(gicc::DeviceCtx* ctx, int* status) {
  gicc::flush<gicc::Scope::Block>(ctx);
  if (threadIdx.x == 0) *status = gicc::quiet(ctx);
}

}  // namespace

int main(int argc, char** argv) {
  const size_t size = (size_t)arg_ll(argc, argv, "-size", 1 << 20);
  const int iters = (int)arg_ll(argc, argv, "-iters", 20);
  try {
    gicc::Runtime rt;
    const int r = rt.rank(), n = rt.size(), right = (r + 1) % n, left = (r - 1 + n) % n;
    if (size == 0 || iters < 1) throw std::runtime_error("need -size > 0 and -iters >= 1");
    gicc::Buffer src = rt.alloc(size * kStreams);
    gicc::Buffer dst = rt.alloc(size * kStreams);
    rt.exchange();
    int* status = nullptr;
    unsigned long long* bad = nullptr;
    GICC_CUDA(cudaMalloc(&status, sizeof(int)));
    GICC_CUDA(cudaMalloc(&bad, sizeof(*bad)));
    cudaEvent_t e0, e1;
    GICC_CUDA(cudaEventCreate(&e0));
    GICC_CUDA(cudaEventCreate(&e1));
    std::vector<double> ms;
    unsigned long long total_bad = 0;
    int total_status = 0;
    for (int it = 0; it < iters + 1; ++it) {  // iteration 0 is the warm-up
      fill<<<256, 256>>>(static_cast<uint8_t*>(src.ptr), size, it);
      GICC_CUDA(cudaDeviceSynchronize());
      rt.barrier();  // the receiver finished checking the previous iteration
      rt.reset();
      std::vector<gicc::Token> tok;
      for (int s = 0; s < kStreams; ++s) tok.push_back(rt.put_no_db(src, right, dst.index, size, s * size, s * size));
      gicc::DeviceCtx* ctx = rt.prepare_trigger(tok.back());
      GICC_CUDA(cudaEventRecord(e0));
      flush_kernel<<<1, 1024>>>(ctx, status);
      GICC_CUDA(cudaEventRecord(e1));
      for (auto& t : tok) rt.wait(t);
      GICC_CUDA(cudaEventSynchronize(e1));
      float t_ms = 0;
      GICC_CUDA(cudaEventElapsedTime(&t_ms, e0, e1));
      int st = 0;
      GICC_CUDA(cudaMemcpy(&st, status, sizeof(st), cudaMemcpyDeviceToHost));
      total_status |= st;
      rt.barrier();  // every rank's puts have landed
      GICC_CUDA(cudaMemset(bad, 0, sizeof(*bad)));
      check<<<256, 256>>>(static_cast<const uint8_t*>(dst.ptr), size, it, bad);
      unsigned long long b = 0;
      GICC_CUDA(cudaMemcpy(&b, bad, sizeof(b), cudaMemcpyDeviceToHost));
      total_bad += b;
      if (it > 0) ms.push_back(gicc::coll::allreduce_max(rt.boot(), (double)t_ms));
    }
    rt.check_device_errors();
    const int all_bad = gicc::coll::allreduce_sum(rt.boot(), (int)(total_bad != 0 || total_status != 0));
    if (r == 0) {
      std::sort(ms.begin(), ms.end());
      const double med = ms[ms.size() / 2];
      std::printf("gicc_queued_put: %d ranks, %d streams x %zu B per batch (rank -> right neighbour): median %.3f ms "
                  "per batch (flush kernel, max over ranks), %.1f GB/s per rank; min %.3f ms; %s\n",
                  n, kStreams, size, med, (double)kStreams * size / (med * 1e-3) / 1e9, ms.front(),
                  all_bad ? "FAIL" : "PASS");
    }
    (void)left;
    GICC_CUDA(cudaFree(status));
    GICC_CUDA(cudaFree(bad));
    rt.barrier();
    return all_bad ? 1 : 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_queued_put: %s\n", e.what());
    return 1;
  }
}
