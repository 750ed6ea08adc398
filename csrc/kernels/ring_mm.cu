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
//   register-tiled SIMT SGEMM, fp32 in and out: 128 x 128 per CTA (8 x 8 per thread,
//   double-buffered shared memory, two CTAs per SM) when a step has at least 120 such
//   tiles, else 64 x 64 (4 x 4 per thread) so that small stripes still fill the GPU;
// * or, in tensor-core mode (RingMmStep::Bsplit), the other CTAs write the stripe transposed
//   as its tf32 parts (hi, lo, hi) and the step's column block is then one kind::tf32 GEMM
//   over 3N with A_s's parts (hi, hi, lo): fp32 accuracy to about 2^-21 of |A||B| per term
//   at tensor-core speed (ops::gemm_tf32, launched after the step kernel on its stream);
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

// 128 x 128 tile: C[i0:i0+128, col0 + j0 : ... + 128] = A[i0:i0+128, :] . B[:, j0:j0+128].
// The 8 warps form a 4 x 2 grid of 32 x 64 warp tiles; lane (ty, tx) of a 4 x 8 lane grid
// owns rows ty*4 + {0..3, 16..19} and columns tx*4 + {0..3, 32..35} of its warp tile, 8 x 8
// in all.  So a warp's four 16-byte shared-memory reads per k touch 4 or 8 distinct vectors
// (one wavefront each): 4 wavefronts per 2048 FMAs, which the shared-memory pipe sustains
// at full FMA rate.  A k-step is 8 deep; A is stored k-major (transposed) with rows padded to
// 132 floats, so the transposing stores of a warp fall in distinct banks; the next k-step's
// operands are loaded into registers while the current one is multiplied.
constexpr int kT2 = 128;
constexpr int kK2 = 8;
constexpr int kPadA = kT2 + 4;

__device__ void sgemm_tile_128(const ops::RingMmStep& a, int tile) {
  __shared__ __align__(16) float As[2][kK2][kPadA];
  __shared__ __align__(16) float Bs[2][kK2][kT2];
  const int tiles_n = a.Ns / kT2;
  const int i0 = (tile / tiles_n) * kT2, j0 = (tile % tiles_n) * kT2;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int wr = (warp >> 1) * 32 + (lane >> 3) * 4;  // first row of this thread (and +16)
  const int wc = (warp & 1) * 64 + (lane & 7) * 4;    // first column (and +32)
  const int ar = t >> 1, ak = (t & 1) * 4;    // A: row, first k of this thread's float4
  const int bk = t >> 5, bc = (t & 31) * 4;   // B: k row, first column
  const float* pa = a.A + (size_t)(i0 + ar) * a.N + ak;
  const float* pb = a.Bcur + (size_t)bk * a.Ns + j0 + bc;
  float acc[8][8] = {};
  float4 va = *reinterpret_cast<const float4*>(pa);
  float4 vb = *reinterpret_cast<const float4*>(pb);
  As[0][ak + 0][ar] = va.x;
  As[0][ak + 1][ar] = va.y;
  As[0][ak + 2][ar] = va.z;
  As[0][ak + 3][ar] = va.w;
  *reinterpret_cast<float4*>(&Bs[0][bk][bc]) = vb;
  __syncthreads();
  int cur = 0;
  for (int k0 = 0; k0 < a.N; k0 += kK2) {
    const bool more = k0 + kK2 < a.N;
    if (more) {
      va = *reinterpret_cast<const float4*>(pa + k0 + kK2);
      vb = *reinterpret_cast<const float4*>(pb + (size_t)(k0 + kK2) * a.Ns);
    }
#pragma unroll
    for (int k = 0; k < kK2; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][k][wr]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][k][wr + 16]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][k][wc]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][k][wc + 32]);
      const float x[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float y[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(x[i], y[j], acc[i][j]);
    }
    if (more) {
      // the other buffer was last read before the previous barrier
      As[cur ^ 1][ak + 0][ar] = va.x;
      As[cur ^ 1][ak + 1][ar] = va.y;
      As[cur ^ 1][ak + 2][ar] = va.z;
      As[cur ^ 1][ak + 3][ar] = va.w;
      *reinterpret_cast<float4*>(&Bs[cur ^ 1][bk][bc]) = vb;
    }
    __syncthreads();
    cur ^= 1;
  }
  const size_t col = (size_t)a.col_block * a.Ns + j0 + wc;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float* row = a.C + (size_t)(i0 + wr + (i < 4 ? i : 16 + i - 4)) * a.N + col;
    *reinterpret_cast<float4*>(row) = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
    *reinterpret_cast<float4*>(row + 32) = make_float4(acc[i][4], acc[i][5], acc[i][6], acc[i][7]);
  }
}

// Tensor-core mode: Bcur [N][Ns] -> Bsplit [Ns][3N], row j = (hi, lo, hi) of Bcur's column
// j, in 32 x 32 tiles through shared memory (loads and stores 128 bytes per warp row).
constexpr int kSplitCtas = 128;

__device__ void split_transpose(const ops::RingMmStep& a, int cta, int nctas) {
  __shared__ float tile[32][33];
  const int tiles_j = a.Ns / 32, tiles = (a.N / 32) * tiles_j;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const size_t N3 = 3 * (size_t)a.N;
  for (int t = cta; t < tiles; t += nctas) {
    const int k0 = (t / tiles_j) * 32, j0 = (t % tiles_j) * 32;
    for (int r = ty; r < 32; r += kThreads / 32) tile[r][tx] = a.Bcur[(size_t)(k0 + r) * a.Ns + j0 + tx];
    __syncthreads();
    for (int r = ty; r < 32; r += kThreads / 32) {
      const float x = tile[tx][r];
      const float hi = ptx::to_tf32(x), lo = x - hi;
      float* d = a.Bsplit + (size_t)(j0 + r) * N3 + k0 + tx;
      d[0] = hi;
      d[a.N] = lo;
      d[2 * (size_t)a.N] = hi;
    }
    __syncthreads();
  }
}

// Output tile edge for a step of Ns x Ns: 128 when that gives at least 120 tiles.
__host__ __device__ inline int ring_tile(int Ns) { return (Ns % kT2 == 0 && (Ns / kT2) * (Ns / kT2) >= 120) ? kT2 : kTile; }

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

template <int T>
__global__ void __launch_bounds__(kThreads, 2) k_ring_mm_step(ops::RingMmStep a, ErrorRecord* err) {
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
    if constexpr (T == 0) split_transpose(a, (int)blockIdx.x - a.push_ctas, (int)gridDim.x - a.push_ctas);
    else if constexpr (T == kT2) sgemm_tile_128(a, (int)blockIdx.x - a.push_ctas);
    else sgemm_tile(a, (int)blockIdx.x - a.push_ctas);
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

int ring_mm_grid_tc(int push_ctas) { return push_ctas + kSplitCtas; }

int ring_mm_grid(int Ns, int push_ctas) {
  const int T = ring_tile(Ns);
  return push_ctas + (Ns / T) * (Ns / T);
}

void ring_mm_step(const RingMmStep& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::ring_mm_step");
  if (a.Ns <= 0 || a.N <= 0 || a.Ns % kTile || a.N % kKStep)
    throw std::runtime_error("gicc::ring_mm_step: need Ns % 64 == 0 and N % 16 == 0");
  if (!a.A || !a.Bcur || !a.C) throw std::runtime_error("gicc::ring_mm_step: A, Bcur and C are required");
  if (a.Bnext_remote && (!a.arrivals_remote || a.push_ctas <= 0))
    throw std::runtime_error("gicc::ring_mm_step: a push needs arrivals_remote and push_ctas > 0");
  if (a.consumed_left && !a.ticket) throw std::runtime_error("gicc::ring_mm_step: consumed_left needs ticket");
  if (a.push_ctas < 0) throw std::runtime_error("gicc::ring_mm_step: push_ctas < 0");
  if (a.Bsplit) {
    if (!a.Asplit || a.N % 32 || a.Ns % 32 || (reinterpret_cast<uintptr_t>(a.Asplit) & 15) ||
        (reinterpret_cast<uintptr_t>(a.Bsplit) & 15))
      throw std::runtime_error("gicc::ring_mm_step: tensor-core mode needs Asplit, N % 32 == 0 and aligned buffers");
    k_ring_mm_step<0><<<ring_mm_grid_tc(a.push_ctas), kThreads, 0, s>>>(a, device_error_record());
    GICC_CUDA(cudaGetLastError());
    const long long k3 = 3LL * a.N;
    gemm_tf32(a.Asplit, a.Bsplit, a.C + (size_t)a.col_block * a.Ns, a.Ns, a.Ns, (int)k3, k3, k3, a.N, 1.0f, s);
    return;
  }
  if (ring_tile(a.Ns) == kT2)
    k_ring_mm_step<kT2><<<ring_mm_grid(a.Ns, a.push_ctas), kThreads, 0, s>>>(a, device_error_record());
  else
    k_ring_mm_step<kTile><<<ring_mm_grid(a.Ns, a.push_ctas), kThreads, 0, s>>>(a, device_error_record());
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
