// ring_mm.cu -- the ring-stripe fp32 matrix multiply of the reference's distributed-matmul
// example (examples/gicc/mm.cu:116-225: every rank holds a row stripe of A and a column
// stripe of B, the B stripes travel around the ring, and each step adds one column block of
// C), here as one kernel per step with the transfer inside it:
//
// * the first `push_ctas` CTAs forward the stripe held this step to the right neighbour's
//   other landing buffer (16-byte stores into its HBM over NVLink) and release-add its
//   arrival word, once that neighbour has reported finishing the step that last read the
//   buffer;
// * the other CTAs compute the column block C[:, b*Ns : (b+1)*Ns] = A_s . B_b with a
//   register-tiled SIMT SGEMM (64 x 64 per CTA, fp32 in and out);
// * the last CTA to finish reports the step as consumed to the left neighbour.
//
// Every wait is bounded; a timeout records an error (where = W_RING_MM) and the CTA skips
// its work.  Stripes move to the right neighbour, so in step s rank r holds (and writes the
// column block of) stripe (r - s) mod n.
#include <cuda_runtime.h>

#include "gicc/config.hpp"
#include "gicc/device/comm.cuh"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace {

constexpr int kTile = 64;   // output tile edge
constexpr int kKStep = 16;  // k per shared-memory stage
constexpr int kThreads = 256;

__device__ bool ring_wait(const uint64_t* word, uint64_t target, const ops::RingMmStep& a, ErrorRecord* err,
                          int peer) {
  uint64_t seen = 0;
  if (proto::wait_until<proto::DevMem>(word, proto::CMP_GE, target, a.timeout_ns, &seen)) return true;
  report_error(err, GICC_ETIMEDOUT, W_RING_MM, a.rank, peer, seen, target);
  return false;
}

// C[i0:i0+64, col0 + j0 : ... + 64] = A[i0:i0+64, :] . B[:, j0:j0+64]
__device__ void sgemm_tile(const ops::RingMmStep& a, int tile) {
  __shared__ float As[kKStep][kTile + 4];
  __shared__ __align__(16) float Bs[kKStep][kTile];
  const int tiles_n = a.Ns / kTile;
  const int i0 = (tile / tiles_n) * kTile, j0 = (tile % tiles_n) * kTile;
  const int t = threadIdx.x, ty = t / 16, tx = t % 16;
  const int ar = t / 4, ak = (t % 4) * 4;    // A: row, first k of this thread's float4
  const int bk = t / 16, bc = (t % 16) * 4;  // B: k row, first column
  float acc[4][4] = {};
  for (int k0 = 0; k0 < a.N; k0 += kKStep) {
    const float4 va = *reinterpret_cast<const float4*>(a.A + (size_t)(i0 + ar) * a.N + k0 + ak);
    const float4 vb = *reinterpret_cast<const float4*>(a.Bcur + (size_t)(k0 + bk) * a.Ns + j0 + bc);
    As[ak + 0][ar] = va.x;
    As[ak + 1][ar] = va.y;
    As[ak + 2][ar] = va.z;
    As[ak + 3][ar] = va.w;
    *reinterpret_cast<float4*>(&Bs[bk][bc]) = vb;
    __syncthreads();
#pragma unroll
    for (int k = 0; k < kKStep; ++k) {
      float x[4], y[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = As[k][ty * 4 + i];
      const float4 w = *reinterpret_cast<const float4*>(&Bs[k][tx * 4]);
      y[0] = w.x;
      y[1] = w.y;
      y[2] = w.z;
      y[3] = w.w;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
    }
    __syncthreads();
  }
  const size_t col = (size_t)a.col_block * a.Ns + j0 + tx * 4;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    *reinterpret_cast<float4*>(a.C + (size_t)(i0 + ty * 4 + i) * a.N + col) =
        make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
}

__device__ void push_stripe(const ops::RingMmStep& a) {
  const size_t nvec = (size_t)a.N * a.Ns / 4;
  const uint4* src = reinterpret_cast<const uint4*>(a.Bcur);
  uint4* dst = reinterpret_cast<uint4*>(a.Bnext_remote);
  const size_t stride = (size_t)a.push_ctas * kThreads;
  size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x;
  for (; i + 3 * stride < nvec; i += 4 * stride) {  // four 16-byte loads in flight per thread
    uint4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = src[i + j * stride];
#pragma unroll
    for (int j = 0; j < 4; ++j) dst[i + j * stride] = v[j];
  }
  for (; i < nvec; i += stride) dst[i] = src[i];
}

__global__ void __launch_bounds__(kThreads) k_ring_mm_step(ops::RingMmStep a, ErrorRecord* err) {
  __shared__ int landed_s, free_s;
  if (threadIdx.x == 0) {
    landed_s = !a.arrivals || ring_wait(a.arrivals, a.arrivals_target, a, err, a.left);  // Bcur has landed
    free_s = 0;
  }
  __syncthreads();
  const bool landed = landed_s != 0;  // every thread reads it before anyone writes free_s
  if ((int)blockIdx.x < a.push_ctas) {
    if (landed && a.Bnext_remote) {
      // the right neighbour finished every step that read the buffer this push overwrites
      if (threadIdx.x == 0) free_s = !a.consumed || ring_wait(a.consumed, a.consumed_target, a, err, a.right);
      __syncthreads();
      if (free_s) {
        push_stripe(a);
        ptx::fence_acq_rel_sys();
        __syncthreads();
        if (threadIdx.x == 0) ptx::red_release_sys_add(a.arrivals_remote, 1);
      }
    }
  } else if (landed) {
    sgemm_tile(a, (int)blockIdx.x - a.push_ctas);
  }
  // Every thread of this CTA is done reading Bcur; the last CTA of the step tells the left
  // neighbour (the one that writes into this rank's landing buffers).
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0 && a.consumed_left) {
    const unsigned long long old = atomicAdd(a.ticket, 1ull);
    if (old + 1 == a.ticket_target) {
      ptx::fence_acq_rel_sys();
      ptx::red_release_sys_add(a.consumed_left, 1);
    }
  }
}

}  // namespace

namespace ops {

int ring_mm_grid(int Ns, int push_ctas) { return push_ctas + (Ns / kTile) * (Ns / kTile); }

void ring_mm_step(const RingMmStep& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::ring_mm_step");
  if (a.Ns <= 0 || a.N <= 0 || a.Ns % kTile || a.N % kKStep)
    throw std::runtime_error("gicc::ring_mm_step: need Ns % 64 == 0 and N % 16 == 0");
  if (!a.A || !a.Bcur || !a.C) throw std::runtime_error("gicc::ring_mm_step: A, Bcur and C are required");
  if (a.Bnext_remote && (!a.arrivals_remote || a.push_ctas <= 0))
    throw std::runtime_error("gicc::ring_mm_step: a push needs arrivals_remote and push_ctas > 0");
  if (a.consumed_left && !a.ticket) throw std::runtime_error("gicc::ring_mm_step: consumed_left needs ticket");
  if (a.push_ctas < 0) throw std::runtime_error("gicc::ring_mm_step: push_ctas < 0");
  k_ring_mm_step<<<ring_mm_grid(a.Ns, a.push_ctas), kThreads, 0, s>>>(a, device_error_record());
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
