// gicc_api_example -- the NVSHMEM-style API (gicc/api.hpp): symmetric malloc, a device
// context, device puts into the right neighbour through it, a barrier, and a check of what
// the left neighbour put.  The reference's counterpart is the gicc_api.hpp usage in its
// MLX5 examples.
//
//   python -m opengda_b200.parallel.launch -n 8 opengda_b200/bin/gicc_api_example
#include <cuda_runtime.h>

#include <cstdio>

#include "gicc/api.hpp"
#include "gicc/device/comm.cuh"

__global__ void put_to_right(gicc::GiccContext* ctx, float* x, size_t n, int right, float tag) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    x[i] = tag + (float)(i % 1000);
  __syncthreads();
  // each block puts its own contiguous slice (block scope: all its threads cooperate)
  const size_t per = (n + gridDim.x - 1) / gridDim.x, lo = blockIdx.x * per;
  const size_t hi = lo + per < n ? lo + per : n;
  if (lo < hi) {
    float* dst = static_cast<float*>(gicc::remote_ptr(ctx, x + n + lo, right));  // second half on the peer
    gicc::put<gicc::Scope::Block>(ctx, dst, x + lo, (uint32_t)((hi - lo) * sizeof(float)), right);
  }
  gicc::quiet(ctx, right);
}

__global__ void count_bad(const float* y, size_t n, float tag, unsigned long long* bad) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    if (y[i] != tag + (float)(i % 1000)) atomicAdd(bad, 1ull);
}

int main() {
  try {
    gicc::init();
    const int me = gicc::my_pe(), n = gicc::n_pes();
    const int right = (me + 1) % n, left = (me + n - 1) % n;
    const size_t count = 1 << 20;
    float* x = static_cast<float*>(gicc::malloc(2 * count * sizeof(float)));
    float* scratch = static_cast<float*>(gicc::malloc(64));
    if (gicc::remote_ptr(x, me) != x) throw std::runtime_error("remote_ptr(self) must be the local address");
    gicc::GiccContext* ctx = gicc::context();
    gicc::barrier();
    put_to_right<<<64, 256>>>(ctx, x, count, right, 100.0f * me);
    GICC_CUDA(cudaGetLastError());
    gicc::barrier();
    unsigned long long* bad = nullptr;
    GICC_CUDA(cudaMalloc(&bad, sizeof(*bad)));
    GICC_CUDA(cudaMemset(bad, 0, sizeof(*bad)));
    count_bad<<<64, 256>>>(x + count, count, 100.0f * left, bad);
    unsigned long long h = 1;
    GICC_CUDA(cudaMemcpy(&h, bad, sizeof(h), cudaMemcpyDeviceToHost));
    GICC_CUDA(cudaFree(bad));
    gicc::runtime().check_device_errors();
    gicc::free(scratch);
    gicc::free(x);
    std::printf("rank %d of %d: %s (%llu bad values)\n", me, n, h == 0 ? "PASS" : "FAIL", h);
    gicc::finalize();
    return h == 0 ? 0 : 1;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_api_example: %s\n", e.what());
    return 1;
  }
}
