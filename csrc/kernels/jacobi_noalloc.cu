// jacobi_noalloc.cu -- gicc_jacobi_step_norm_noalloc: a Jacobi sweep plus the squared norm
// of the update, with its working memory (one partial sum per thread block) in a static
// device array instead of memory from the caller or cudaMalloc.  See gicc/noalloc.h for
// who needs this and for the limits.  This entry point has no counterpart in the reference.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "gicc/noalloc.h"

namespace {

constexpr int kThreads = 256;                // 8 warps x 128 columns
constexpr int kColsPerCta = kThreads * 4;    // 1024 columns per block
constexpr int kRun = 16;                     // rows per block
constexpr int kMaxDevices = 64;

// The working memory: one partial sum of squares per block of the sweep.
static __device__ __align__(256) double g_noalloc_partials[GICC_NOALLOC_MAX_BLOCKS];

__device__ __forceinline__ float upd(float e, float w, float n, float s) {
  return __fmul_rn(__fadd_rn(__fadd_rn(e, w), __fadd_rn(n, s)), 0.25f);
}

// Same update (bit for bit) as the library's halo-pushing stencil kernel; every block
// writes its partial sum of (new - old)^2 into its own slot.
__global__ void __launch_bounds__(kThreads) k_jacobi_partials(const float* __restrict__ a, float* __restrict__ b,
                                                             int nx, int rows, double* partials) {
  const int nbx = (nx + kColsPerCta - 1) / kColsPerCta;
  const int bx = blockIdx.x % nbx, by = blockIdx.x / nbx;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j0 = bx * kColsPerCta + threadIdx.x * 4;
  const bool active = j0 < nx;
  const int r0 = 1 + by * kRun;
  const int r1 = min(r0 + kRun, rows + 1);
  float4 rowv[kRun + 2];
  float edge[kRun];
#pragma unroll
  for (int i = 0; i < kRun + 2; ++i) {
    const int r = r0 - 1 + i;
    rowv[i] = (active && r <= r1) ? *reinterpret_cast<const float4*>(a + (size_t)r * nx + j0) : make_float4(0, 0, 0, 0);
  }
  const bool edge_lane = (lane == 0 && active && j0 > 0) || (lane == 31 && active && j0 + 4 < nx);
  const int ecol = lane == 0 ? j0 - 1 : j0 + 4;
#pragma unroll
  for (int i = 0; i < kRun; ++i) edge[i] = (edge_lane && r0 + i < r1) ? a[(size_t)(r0 + i) * nx + ecol] : 0.f;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kRun; ++i) {
    const int r = r0 + i;
    if (r >= r1) break;
    const float4 up = rowv[i], mid = rowv[i + 1], dn = rowv[i + 2];
    float left = __shfl_up_sync(0xffffffffu, mid.w, 1);
    float right = __shfl_down_sync(0xffffffffu, mid.x, 1);
    if (lane == 0 && active && j0 > 0) left = edge[i];
    if (lane == 31 && active && j0 + 4 < nx) right = edge[i];
    float4 o;
    o.x = upd(mid.y, left, up.x, dn.x);
    o.y = upd(mid.z, mid.x, up.y, dn.y);
    o.z = upd(mid.w, mid.y, up.z, dn.z);
    o.w = upd(right, mid.z, up.w, dn.w);
    if (j0 == 0) o.x = mid.x;
    if (j0 + 4 >= nx) o.w = mid.w;
    if (active) {
      *reinterpret_cast<float4*>(b + (size_t)r * nx + j0) = o;
      const float dx = o.x - mid.x, dy = o.y - mid.y, dz = o.z - mid.z, dw = o.w - mid.w;
      sq += dx * dx + dy * dy + dz * dz + dw * dw;
    }
  }
  for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  __shared__ double wsum[kThreads / 32];
  if (lane == 0) wsum[warp] = (double)sq;
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    for (int w = 0; w < kThreads / 32; ++w) s += wsum[w];
    partials[blockIdx.x] = s;
  }
}

// Fixed-order sum of the partials (one block).
__global__ void __launch_bounds__(256) k_sum_partials(const double* partials, int n, double* out) {
  __shared__ double s[256];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partials[i];
  s[threadIdx.x] = acc;
  __syncthreads();
  for (int k = blockDim.x / 2; k > 0; k >>= 1) {
    if ((int)threadIdx.x < k) s[threadIdx.x] += s[threadIdx.x + k];
    __syncthreads();
  }
  if (threadIdx.x == 0) *out = s[0];
}

std::mutex g_mu;
double* g_addr[kMaxDevices] = {};

// Device address of the static array for the current device (looked up once per device).
cudaError_t partials_address(double** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess) return e;
    g_addr[dev] = static_cast<double*>(p);
  }
  *out = g_addr[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) cudaError_t gicc_jacobi_step_norm_noalloc(
    const float* a, float* b, int nx, int rows, double* norm_sq, cudaStream_t stream) {
  if (!a || !b || !norm_sq || nx < 4 || nx % 4 != 0 || rows < 1 ||
      (reinterpret_cast<uintptr_t>(a) & 15) || (reinterpret_cast<uintptr_t>(b) & 15)) {
    std::fprintf(stderr, "gicc_jacobi_step_norm_noalloc: bad arguments (nx must be a multiple of 4, rows >= 1, "
                         "16-byte aligned fields)\n");
    return cudaErrorInvalidValue;
  }
  // 64-bit arithmetic: nx and rows near INT_MAX must fail the size check below, not wrap.
  const long long blocks = (((long long)nx + kColsPerCta - 1) / kColsPerCta) * (((long long)rows + kRun - 1) / kRun);
  if (blocks > GICC_NOALLOC_MAX_BLOCKS) {
    std::fprintf(stderr,
                 "gicc_jacobi_step_norm_noalloc: %d x %d cells need %lld partial sums, more than the %d this "
                 "entry point holds (at most 32768 x 32768 cells)\n",
                 nx, rows, blocks, GICC_NOALLOC_MAX_BLOCKS);
    return cudaErrorInvalidValue;
  }
  const size_t field_bytes = ((size_t)rows + 2) * (size_t)nx * sizeof(float);
  const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
  if (pa < pb + field_bytes && pb < pa + field_bytes) {
    std::fprintf(stderr, "gicc_jacobi_step_norm_noalloc: the input and output fields overlap (the sweep reads "
                         "neighbours of cells it writes; pass two separate fields)\n");
    return cudaErrorInvalidValue;
  }
  double* partials = nullptr;
  cudaError_t e = partials_address(&partials);
  if (e != cudaSuccess) return e;
  k_jacobi_partials<<<(unsigned)blocks, kThreads, 0, stream>>>(a, b, nx, rows, partials);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  k_sum_partials<<<1, 256, 0, stream>>>(partials, (int)blocks, norm_sq);
  return cudaGetLastError();
}
