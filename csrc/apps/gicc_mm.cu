// gicc_mm -- the distributed matrix-multiply example: C = A * B^T over all ranks with the
// all-gather fused into the tcgen05 GEMM (ops::ag_gemm).  A [M, K] is row-sharded, B [N, K]
// (the nn.Linear layout) column-sharded; rank r computes C[:, r*N/n : (r+1)*N/n].  The
// reference's examples/gicc/mm.cu runs the same all-gather-and-multiply pattern as an fp32
// stripe ring with one put per step; here the shard crosses NVLink once per call (NVLS
// multicast when the node has it, else unicast pushes) while the tensor cores consume it.
//
// Inputs are exactly representable: entries are k/16 for k in [-8, 8], so every product and
// every partial sum is exact in fp32 and the only error is the final bf16 rounding.  The
// analytic check recomputes `--samples` random elements of C on the host in double.
//
// `-ring` runs the reference example's own algorithm instead: fp32, row stripes of A and
// column stripes of B, the B stripes passed around the ring, one column block of C per step
// (ops::ring_mm_step: the stripe push runs inside the step's SGEMM kernel).  With these
// inputs every fp32 sum is exact, so the sampled check there is exact equality.
//
//   python -m opengda_b200.parallel.launch -n 8 opengda_b200/bin/gicc_mm [-n 16384] [-iters 20] [-unicast]
//   python -m opengda_b200.parallel.launch -n 8 opengda_b200/bin/gicc_mm -ring [-n 4096]
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "gicc/coll.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"
#include "gicc/runtime.hpp"

namespace {

int arg_int(int argc, char** argv, const char* name, int def) {
  for (int i = 1; i + 1 < argc; ++i)
    if (!std::strcmp(argv[i], name)) return std::atoi(argv[i + 1]);
  return def;
}
bool arg_flag(int argc, char** argv, const char* name) {
  for (int i = 1; i < argc; ++i)
    if (!std::strcmp(argv[i], name)) return true;
  return false;
}

__host__ __device__ inline float entry(uint32_t which, uint64_t row, uint64_t col, uint64_t ld) {
  uint64_t z = (row * ld + col) * 0x9E3779B97F4A7C15ull + which * 0xD1B54A32D192ED03ull + 1;
  z ^= z >> 31;
  z *= 0xBF58476D1CE4E5B9ull;
  z ^= z >> 29;
  return (float)((int)(z % 17) - 8) / 16.0f;
}

// rows [r0, r0 + rows) of matrix `which` ([*, ld] row-major) into dst
__global__ void fill(__nv_bfloat16* dst, uint32_t which, uint64_t r0, uint64_t rows, uint64_t ld) {
  const uint64_t n = rows * ld;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = __float2bfloat16(entry(which, r0 + i / ld, i % ld, ld));
}

__global__ void fill_f32(float* dst, uint32_t which, uint64_t r0, uint64_t rows, uint64_t c0, uint64_t cols,
                         uint64_t ld) {  // dst[i][j] = entry(which, r0 + i, c0 + j, ld)
  const uint64_t n = rows * cols;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    dst[i] = entry(which, r0 + i / cols, c0 + i % cols, ld);
}

// The fp32 ring: rank r holds A rows [r*Ns, (r+1)*Ns) and B columns [r*Ns, (r+1)*Ns); in step
// s it holds stripe (r - s) mod n and forwards it to the right neighbour.
int run_ring(gicc::Runtime& rt, int N, int iters, int samples) {
  const int r = rt.rank(), n = rt.size(), Ns = N / n;
  if (N % n || Ns % 64 || N % 16) throw std::runtime_error("-ring needs N/ranks % 64 == 0 and N % 16 == 0");
  const size_t stripe = (size_t)N * Ns * sizeof(float);
  gicc::Buffer land[2] = {rt.alloc(stripe), rt.alloc(stripe)};
  rt.exchange();
  const size_t w = rt.signal_alloc(2);  // [0] arrivals (x push CTAs), [1] steps the right rank finished
  float *A = nullptr, *B = nullptr, *C = nullptr;
  unsigned long long* ticket = nullptr;
  GICC_CUDA(cudaMalloc(&A, stripe));
  GICC_CUDA(cudaMalloc(&B, stripe));
  GICC_CUDA(cudaMalloc(&C, stripe));
  GICC_CUDA(cudaMalloc(&ticket, sizeof(*ticket)));
  GICC_CUDA(cudaMemset(ticket, 0, sizeof(*ticket)));
  fill_f32<<<1024, 256>>>(A, 0, (uint64_t)r * Ns, Ns, 0, N, N);
  fill_f32<<<1024, 256>>>(B, 1, 0, N, (uint64_t)r * Ns, Ns, N);
  GICC_CUDA(cudaDeviceSynchronize());
  rt.barrier();
  const int P = 8, left = (r - 1 + n) % n, right = (r + 1) % n;
  const int grid = gicc::ops::ring_mm_grid(Ns, P);
  uint64_t calls = 0, steps = 0;
  auto call = [&]() {
    ++calls;
    for (int s = 0; s < n; ++s) {
      gicc::ops::RingMmStep st;
      st.N = N;
      st.Ns = Ns;
      st.A = A;
      st.C = C;
      st.col_block = (r - s + n) % n;
      st.Bcur = s == 0 ? B : static_cast<const float*>(land[s & 1].ptr);
      if (s > 0) {
        st.arrivals = rt.signal_local(w);
        st.arrivals_target = ((calls - 1) * (n - 1) + s) * (uint64_t)P;
      }
      if (s < n - 1) {
        st.Bnext_remote = static_cast<float*>(rt.remote_ptr(right, land[(s + 1) & 1].index, 0));
        st.arrivals_remote = rt.signal_peer(right, w);
        st.consumed = rt.signal_local(w + 1);
        st.consumed_target = (calls - 1) * n + s;
      }
      st.consumed_left = rt.signal_peer(left, w + 1);
      st.ticket = ticket;
      st.ticket_target = (steps + 1) * (unsigned long long)grid;
      st.push_ctas = P;
      st.timeout_ns = rt.timeout_ns();
      st.rank = r;
      st.left = left;
      st.right = right;
      gicc::ops::ring_mm_step(st, nullptr);
      ++steps;
    }
  };
  for (int i = 0; i < 3; ++i) call();
  GICC_CUDA(cudaDeviceSynchronize());
  rt.barrier();
  cudaEvent_t e0, e1;
  GICC_CUDA(cudaEventCreate(&e0));
  GICC_CUDA(cudaEventCreate(&e1));
  GICC_CUDA(cudaEventRecord(e0));
  for (int i = 0; i < iters; ++i) call();
  GICC_CUDA(cudaEventRecord(e1));
  GICC_CUDA(cudaEventSynchronize(e1));
  float ms = 0;
  GICC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  rt.check_device_errors();
  const double call_ms = gicc::coll::allreduce_max(rt.boot(), (double)ms / iters);
  std::vector<float> c((size_t)Ns * N);
  GICC_CUDA(cudaMemcpy(c.data(), C, stripe, cudaMemcpyDeviceToHost));
  int bad = 0;
  uint64_t z = 777 + r;
  for (int q = 0; q < samples; ++q) {
    z = z * 6364136223846793005ull + 1442695040888963407ull;
    const int i = (int)((z >> 33) % (uint64_t)Ns);
    z = z * 6364136223846793005ull + 1442695040888963407ull;
    const int j = (int)((z >> 33) % (uint64_t)N);
    double ref = 0;
    for (int k = 0; k < N; ++k) ref += (double)entry(0, (uint64_t)r * Ns + i, k, N) * (double)entry(1, k, j, N);
    if ((double)c[(size_t)i * N + j] != ref) ++bad;  // every fp32 partial sum is exact
  }
  const int all_bad = gicc::coll::allreduce_sum(rt.boot(), bad);
  if (r == 0)
    std::printf("gicc_mm -ring: %dx%d fp32 on %d GPUs: %.4f ms per call (max over ranks), %.2f TFLOP/s; "
                "%d exact samples per rank: %s\n",
                N, N, n, call_ms, 2.0 * N * (double)N * N / (call_ms * 1e-3) / 1e12, samples,
                all_bad ? "FAIL" : "PASS");
  GICC_CUDA(cudaFree(A));
  GICC_CUDA(cudaFree(B));
  GICC_CUDA(cudaFree(C));
  GICC_CUDA(cudaFree(ticket));
  rt.barrier();
  return all_bad ? 1 : 0;
}

}  // namespace

int main(int argc, char** argv) {
  if (arg_flag(argc, argv, "-ring")) {
    try {
      gicc::Runtime rt;
      return run_ring(rt, arg_int(argc, argv, "-n", 4096), arg_int(argc, argv, "-iters", 10),
                      arg_int(argc, argv, "-samples", 256));
    } catch (const std::exception& e) {
      std::fprintf(stderr, "gicc_mm -ring: %s\n", e.what());
      return 1;
    }
  }
  const int S = arg_int(argc, argv, "-n", 16384);
  const int iters = arg_int(argc, argv, "-iters", 20);
  const int samples = arg_int(argc, argv, "-samples", 256);
  const bool unicast = arg_flag(argc, argv, "-unicast");
  try {
    gicc::Runtime rt;
    const int r = rt.rank(), n = rt.size();
    const int M = S, N = S, K = S, Ms = M / n, Ns = N / n;
    if (n < 2) throw std::runtime_error("gicc_mm needs at least 2 ranks");
    if (M % (n * 128) || Ns % 256 || K % 64) throw std::runtime_error("need M % (ranks*128) == 0, N/ranks % 256 == 0");
    const bool nvls = !unicast && rt.multicast_supported();
    // two landing buffers (parities) for the gathered A, symmetric
    gicc::Buffer abuf[2] = {rt.alloc((size_t)M * K * 2, nvls), rt.alloc((size_t)M * K * 2, nvls)};
    rt.exchange();
    const int nb = Ms / 128;
    const size_t off = rt.signal_alloc((size_t)n * nb + n + 1);
    __nv_bfloat16 *B = nullptr, *C = nullptr;
    GICC_CUDA(cudaMalloc(&B, (size_t)Ns * K * 2));
    GICC_CUDA(cudaMalloc(&C, (size_t)M * Ns * 2));
    fill<<<1024, 256>>>(B, 1, (uint64_t)r * Ns, Ns, K);
    for (int p = 0; p < 2; ++p)  // this rank's shard, in both parities (zero-copy input)
      fill<<<1024, 256>>>(static_cast<__nv_bfloat16*>(abuf[p].ptr) + (size_t)r * Ms * K, 0, (uint64_t)r * Ms, Ms, K);
    GICC_CUDA(cudaDeviceSynchronize());
    rt.barrier();

    gicc::ops::AgGemmArgs a;
    a.n = n;
    a.r = r;
    a.M = M;
    a.Ns = Ns;
    a.K = K;
    a.B = B;
    a.ldb = K;
    a.C = C;
    a.ldc = Ns;
    for (int q = 0; q < n; ++q) {
      a.arrivals[q] = rt.signal_peer(q, off);
      a.done[q] = rt.signal_peer(q, off + (size_t)n * nb);
    }
    a.tile_counter = rt.signal_local(off + (size_t)n * nb + n);
    a.arrivals_mc = nvls ? rt.signal_multicast(off) : nullptr;
    a.comm_ctas = nvls ? (n >= 8 ? 16 : 8) : 32;
    a.timeout_ns = rt.timeout_ns();
    uint64_t epoch = 0;
    auto call = [&]() {
      ++epoch;
      const int p = (int)(epoch % 2);
      for (int q = 0; q < n; ++q) a.a_full[q] = rt.remote_ptr(q, abuf[p].index, 0);
      a.a_mc = nvls ? rt.multicast_ptr(abuf[p].index) : nullptr;
      a.epoch = epoch;
      gicc::ops::ag_gemm(a, nullptr);
    };
    for (int i = 0; i < 3; ++i) call();
    GICC_CUDA(cudaDeviceSynchronize());
    rt.barrier();
    cudaEvent_t e0, e1;
    GICC_CUDA(cudaEventCreate(&e0));
    GICC_CUDA(cudaEventCreate(&e1));
    GICC_CUDA(cudaEventRecord(e0));
    for (int i = 0; i < iters; ++i) call();
    GICC_CUDA(cudaEventRecord(e1));
    GICC_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    GICC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    rt.check_device_errors();
    const double step_ms = gicc::coll::allreduce_max(rt.boot(), (double)ms / iters);

    // analytic check of sampled elements of this rank's C columns
    std::vector<__nv_bfloat16> c((size_t)M * Ns);
    GICC_CUDA(cudaMemcpy(c.data(), C, c.size() * 2, cudaMemcpyDeviceToHost));
    int bad = 0;
    uint64_t z = 12345 + r;
    for (int s = 0; s < samples; ++s) {
      z = z * 6364136223846793005ull + 1442695040888963407ull;
      const int i = (int)((z >> 33) % (uint64_t)M);
      z = z * 6364136223846793005ull + 1442695040888963407ull;
      const int j = (int)((z >> 33) % (uint64_t)Ns);
      double ref = 0;
      for (int k = 0; k < K; ++k) ref += (double)entry(0, i, k, K) * (double)entry(1, (uint64_t)r * Ns + j, k, K);
      const double got = (double)__bfloat162float(c[(size_t)i * Ns + j]);
      if (std::fabs(got - ref) > std::ldexp(std::fabs(ref), -8) + 1e-6) ++bad;
    }
    const int all_bad = gicc::coll::allreduce_sum(rt.boot(), bad);
    if (r == 0) {
      const double tflops = 2.0 * M * N * K / (step_ms * 1e-3) / 1e12;
      std::printf("gicc_mm: %dx%dx%d bf16 on %d GPUs (%s): %.4f ms per call (max over ranks), %.1f TFLOP/s; "
                  "%d samples per rank: %s\n",
                  M, N, K, n, nvls ? "NVLS multicast" : "unicast", step_ms, tflops, samples,
                  all_bad ? "FAIL" : "PASS");
    }
    GICC_CUDA(cudaFree(B));
    GICC_CUDA(cudaFree(C));
    rt.barrier();
    return all_bad ? 1 : 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_mm: %s\n", e.what());
    return 1;
  }
}
