// gemm.cu -- single-GPU tcgen05 GEMM (the compute core of every distributed GEMM mode).
//
//   C[M,N] = alpha * A[M,K] * B[N,K]^T,  bf16 inputs, f32 accumulation, bf16 or f32 output.
//
// Host entry points: gicc::ops::gemm_bf16 (C++, throws) and gicc_gemm_bf16 (C ABI).
#include <algorithm>
#include <cuda.h>
#include <cuda_runtime.h>

#include "gicc/device/gemm_core.cuh"
#include "gicc/device/gemm_core2.cuh"
#include "gicc/config.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace gemm {

// Epilogue: row-major bf16/f32 store of alpha * acc.
struct StoreEpi {
  static constexpr bool kNeedsTileDone = false;
  static constexpr bool kPairHalves = false;
  static constexpr bool kStagedStore = true;  // the CTA-pair core may store bf16 C through TMA
  void* C;
  long long ldc;
  int M, N;
  float alpha;
  int out_f32;
  int vec = 1;                       // C's base and row pitch are multiples of 16 bytes
  int use_tma = 0;                   // bf16 C stored as 32 x 32 boxes by TMA (tmC valid)
  const CUtensorMap* tmC = nullptr;  // set by the kernel (a __grid_constant__ parameter)
  __device__ bool staged() const { return use_tma != 0; }
  __device__ const CUtensorMap* tmap() const { return tmC; }
  // A box whose first row or column lies past C's edge is not stored (TMA clips the rest).
  __device__ bool chunk_in_bounds(const TileInfo& ti, int row0, int c) const {
    return ti.m0 + row0 < M && ti.n0 + c < N;
  }
  __device__ __forceinline__ void pack(const uint32_t* r, uint4* v) const {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j].x = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 0]), alpha * __uint_as_float(r[8 * j + 1]));
      v[j].y = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 2]), alpha * __uint_as_float(r[8 * j + 3]));
      v[j].z = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 4]), alpha * __uint_as_float(r[8 * j + 5]));
      v[j].w = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 6]), alpha * __uint_as_float(r[8 * j + 7]));
    }
  }
  __device__ static void fence_before_done() {}
  __device__ void tile_done(const TileInfo&) {}
  __device__ void begin_tile(const TileInfo&, int) {}
  __device__ void end_tile(const TileInfo&, int) {}
  __device__ __forceinline__ void store(const TileInfo& ti, int row, int c, const uint32_t* r) {
    const int gm = ti.m0 + row;
    if (gm >= M) return;
    const int gn = ti.n0 + c;
    // 16-byte vector stores where C's base and row pitch allow them (vec) and the group lies
    // inside C; element stores otherwise (unaligned views, the last N % 8 (bf16) or N % 4
    // (f32) columns).
    if (out_f32) {
      float* p = static_cast<float*>(C) + (size_t)gm * ldc + gn;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (vec && gn + 4 * j + 4 <= N) {
          uint4 v;
          v.x = __float_as_uint(alpha * __uint_as_float(r[4 * j + 0]));
          v.y = __float_as_uint(alpha * __uint_as_float(r[4 * j + 1]));
          v.z = __float_as_uint(alpha * __uint_as_float(r[4 * j + 2]));
          v.w = __float_as_uint(alpha * __uint_as_float(r[4 * j + 3]));
          ptx::st_v4(p + 4 * j, v);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (gn + 4 * j + e < N) p[4 * j + e] = alpha * __uint_as_float(r[4 * j + e]);
        }
      }
    } else {
      uint16_t* p = static_cast<uint16_t*>(C) + (size_t)gm * ldc + gn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (vec && gn + 8 * j + 8 <= N) {
          uint4 v;
          v.x = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 0]), alpha * __uint_as_float(r[8 * j + 1]));
          v.y = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 2]), alpha * __uint_as_float(r[8 * j + 3]));
          v.z = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 4]), alpha * __uint_as_float(r[8 * j + 5]));
          v.w = ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + 6]), alpha * __uint_as_float(r[8 * j + 7]));
          ptx::st_v4(p + 8 * j, v);
        } else {
#pragma unroll
          for (int e = 0; e < 8; ++e)
            if (gn + 8 * j + e < N) p[8 * j + e] = static_cast<uint16_t>(ptx::pack_bf16x2(alpha * __uint_as_float(r[8 * j + e]), 0.f) & 0xffffu);
        }
      }
    }
  }
};

// 16-byte vector (and TMA) stores of C need a 16-byte aligned base and row pitch.
static bool c_vector_ok(const void* C, long long ldc, bool out_f32) {
  return (reinterpret_cast<uintptr_t>(C) & 15) == 0 && ((ldc * (out_f32 ? 4 : 2)) & 15) == 0;
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_bf16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, PlainSched sched,
                StoreEpi epi, ErrorRecord* err, uint64_t timeout_ns) {
  gemm_core<BN>(&tmA, &tmB, sched, epi, err, timeout_ns, -1);
}

template <int BN>
static void launch_plain(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                         long long ldc, bool out_f32, float alpha, cudaStream_t stream) {
  using Cf = Cfg<BN>;
  const CUtensorMap tA = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, ldb, BN, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  PlainSched s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.bn = BN;
  s.num_m = (M + BM - 1) / BM;
  s.num_n = (N + BN - 1) / BN;
  const ops::GemmTuning tune = ops::gemm_tuning();
  s.group_m = tune.group_m;
  s.l2hint = tune.l2_hint;
  StoreEpi e;
  e.C = C;
  e.ldc = ldc;
  e.M = M;
  e.N = N;
  e.alpha = alpha;
  e.out_f32 = out_f32 ? 1 : 0;
  e.vec = c_vector_ok(C, ldc, out_f32) ? 1 : 0;
  static bool attr_set[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_bf16<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmemBytes));
    attr_set[dev] = true;
  }
  const int tiles = s.num_m * s.num_n;
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  k_gemm_bf16<BN><<<grid, kThreads, Cf::kSmemBytes, stream>>>(tA, tB, s, e, device_error_record(),
                                                               default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}

// ---- CTA-pair (cta_group::2) variants: 256 x 256 (NH = 1) or 256 x 512 (NH = 2) tiles per
// cluster of two CTAs ----
struct PairPlainSched {
  int M, N, K;
  int num_m, num_n, group_m;
  int cols;  // output columns per pair tile (NH * 256)
  pair::PairLoadOpts lopt;
  static constexpr int kCommWarps = 0;
  __device__ int num_tiles() const { return num_m * num_n; }
  __device__ TileInfo tile(int t) const {
    int mb, nb;
    raster(t, num_m, num_n, group_m, mb, nb);
    TileInfo ti;
    ti.m0 = mb * 2 * BM;
    ti.n0 = nb * cols;
    ti.a_row = ti.m0;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = 0;
    ti.aux2 = 0;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo&, int, uint64_t, volatile int*, ErrorRecord*) const { return true; }
};

template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::PairCfg<NH>::kThreads, 1)
    k_gemm_bf16_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmC, PairPlainSched sched, StoreEpi epi, ErrorRecord* err,
                     uint64_t timeout_ns) {
  epi.tmC = &tmC;
  pair::gemm_core_pair<NH>(&tmA, &tmB, sched, epi, err, timeout_ns, -1, sched.lopt);
}

template <int NH>
static void launch_pair(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                        long long ldc, bool out_f32, float alpha, cudaStream_t stream) {
  using Cf = pair::PairCfg<NH>;
  const CUtensorMap tA = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, ldb, pair::BN2 / 2, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  PairPlainSched s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.cols = Cf::kCols;
  s.num_m = (M + 2 * BM - 1) / (2 * BM);
  s.num_n = (N + Cf::kCols - 1) / Cf::kCols;
  const ops::GemmTuning tune = ops::gemm_tuning();
  s.group_m = tune.pair_group_m;
  s.lopt.l2hint = tune.pair_l2_hint;
  s.lopt.prefetch = tune.pair_prefetch;
  StoreEpi e;
  e.C = C;
  e.ldc = ldc;
  e.M = M;
  e.N = N;
  e.alpha = alpha;
  e.out_f32 = out_f32 ? 1 : 0;
  e.vec = c_vector_ok(C, ldc, out_f32) ? 1 : 0;
  // bf16 C whose base and row pitch suit TMA is stored in 32 x 32 boxes through shared
  // memory (whole 128-byte lines to L2); otherwise each thread stores its row directly.
  const bool tma_c = !out_f32 && tune.pair_tma_store != 0 && e.vec;
  e.use_tma = tma_c ? 1 : 0;
  const CUtensorMap tC = tma_c ? make_tmap_2d(C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, N, ldc, 32, 32,
                                              CU_TENSOR_MAP_SWIZZLE_NONE)
                               : tA;  // unused
  static bool attr_set[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_bf16_pair<NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cf::kSmemBytesStaged));
    attr_set[dev] = true;
  }
  const int pairs_max = num_sms(dev) / 2;
  const int tiles = s.num_m * s.num_n;
  const int grid = 2 * (tiles < pairs_max ? tiles : pairs_max);
  k_gemm_bf16_pair<NH><<<grid, Cf::kThreads, Cf::kSmemBytesStaged, stream>>>(tA, tB, tC, s, e, device_error_record(),
                                                                              default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}

// ---- self-test of the core's tile-done ordering (used by the distributed epilogues) ----
// Each epilogue warp records that it finished a tile; the core's tile_done hook must then
// run exactly once per tile, after all four warps.  Warp 0 is delayed on every other tile
// so that the other warps run ahead into the tile held in the other accumulator.
struct TileDoneCheckEpi {
  static constexpr bool kNeedsTileDone = true;
  static constexpr bool kPairHalves = false;
  int num_n, bn;
  uint32_t* warps_done;  // [tiles]
  uint32_t* published;   // [tiles]
  uint32_t* bad;         // tile_done ran before all four warps finished
  uint32_t skew_ns;
  __device__ static void fence_before_done() { __threadfence(); }
  __device__ int index(const TileInfo& ti) const { return (ti.m0 / BM) * num_n + ti.n0 / bn; }
  __device__ void begin_tile(const TileInfo&, int) {}
  __device__ void store(const TileInfo&, int, int, const uint32_t*) {}
  __device__ void end_tile(const TileInfo& ti, int row) {
    const int idx = index(ti);
    if (row < 32 && (idx & 1) == 0 && skew_ns) {
      for (uint32_t t = 0; t < skew_ns; t += 1000) __nanosleep(1000);
    }
    __syncwarp();
    if ((row & 31) == 0) atomicAdd(&warps_done[idx], 1u);
  }
  __device__ void tile_done(const TileInfo& ti) {
    const int idx = index(ti);
    if (atomicAdd(&warps_done[idx], 0u) != 4u) atomicAdd(bad, 1u);
    atomicAdd(&published[idx], 1u);
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tile_done_check(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                           PlainSched sched, TileDoneCheckEpi epi, ErrorRecord* err, uint64_t timeout_ns) {
  gemm_core<256>(&tmA, &tmB, sched, epi, err, timeout_ns, -1);
}

// ---- fp32 GEMM on the tensor cores (3 x tf32) ----
// x = hi + lo with hi = x rounded to tf32 (cvt.rna) and lo = x - hi (exact, |lo| <= 2^-11 |x|);
// A.B^T = Ahi.Bhi^T + Ahi.Blo^T + Alo.Bhi^T + Alo.Blo^T, and the last term (below 2^-22 of
// |A||B|) is dropped.  The three remaining products are one tf32 GEMM over K' = 3K of the
// operands [Ahi | Ahi | Alo] and [Bhi | Blo | Bhi], accumulated in f32 in TMEM: the error is
// about 2^-21 of |A||B| per product term (lo's own tf32 rounding in the MMA), against 2^-24
// for fp32 FMA.

// dst [rows][3K] = three K-long segments of src's rows: (hi, hi, lo) with order 0 or
// (hi, lo, hi) with order 1.  src rows are 16-byte aligned (ld % 4 == 0), K % 4 == 0.
__global__ void __launch_bounds__(256) k_tf32_split(const float* __restrict__ src, long long ld, int rows, int K,
                                                    float* __restrict__ dst, int order) {
  const int k4 = K / 4;
  const size_t total = (size_t)rows * k4;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / k4), c = (int)(i - (size_t)r * k4) * 4;
    const float4 v = *reinterpret_cast<const float4*>(src + (size_t)r * ld + c);
    float4 hi, lo;
    hi.x = ptx::to_tf32(v.x);
    hi.y = ptx::to_tf32(v.y);
    hi.z = ptx::to_tf32(v.z);
    hi.w = ptx::to_tf32(v.w);
    lo.x = v.x - hi.x;
    lo.y = v.y - hi.y;
    lo.z = v.z - hi.z;
    lo.w = v.w - hi.w;
    float* d = dst + (size_t)r * 3 * K + c;
    *reinterpret_cast<float4*>(d) = hi;
    *reinterpret_cast<float4*>(d + K) = order == 0 ? hi : lo;
    *reinterpret_cast<float4*>(d + 2 * K) = order == 0 ? lo : hi;
  }
}

// The plain schedule over fp32 operands (32 elements per 128-byte k-block) for kind::tf32.
struct PlainSchedTf32 : PlainSched {
  static constexpr bool kTf32 = true;
  __device__ TileInfo tile(int t) const {
    TileInfo ti = PlainSched::tile(t);
    ti.kb1 = (K + 31) / 32;
    return ti;
  }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * 32, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * 32, ti.b_row);
  }
};

// The CTA-pair schedule over fp32 operands for kind::tf32.
struct PairPlainSchedTf32 : PairPlainSched {
  static constexpr bool kTf32 = true;
  __device__ TileInfo tile(int t) const {
    TileInfo ti = PairPlainSched::tile(t);
    ti.kb1 = (K + 31) / 32;
    return ti;
  }
};

template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::PairCfg<NH>::kThreads, 1)
    k_gemm_tf32_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     PairPlainSchedTf32 sched, StoreEpi epi, ErrorRecord* err, uint64_t timeout_ns) {
  pair::gemm_core_pair<NH>(&tmA, &tmB, sched, epi, err, timeout_ns, -1);
}

__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tf32(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, PlainSchedTf32 sched,
                StoreEpi epi, ErrorRecord* err, uint64_t timeout_ns) {
  gemm_core<256>(&tmA, &tmB, sched, epi, err, timeout_ns, -1);
}

}  // namespace gemm

namespace ops {

void tf32_split(const float* src, long long ld, int rows, int K, float* dst, int order, cudaStream_t stream) {
  if (rows <= 0 || K <= 0 || K % 4 || ld % 4 || (reinterpret_cast<uintptr_t>(src) & 15) ||
      (reinterpret_cast<uintptr_t>(dst) & 15) || order < 0 || order > 1)
    throw std::runtime_error("gicc::tf32_split: K % 4 == 0, ld % 4 == 0, 16-byte aligned src and dst, order 0 or 1");
  const size_t vecs = (size_t)rows * (K / 4);
  const int grid = (int)std::min<size_t>((vecs + 255) / 256, (size_t)num_sms() * 8);
  gemm::k_tf32_split<<<grid, 256, 0, stream>>>(src, ld, rows, K, dst, order);
  GICC_CUDA(cudaGetLastError());
}

static int default_tile(int M, int N);  // tile by shape (defined with gemm_bf16)

namespace {
template <int NH>
void launch_tf32_pair(const float* A, const float* B, float* C, int M, int N, int K, long long lda, long long ldb,
                      long long ldc, float alpha, cudaStream_t stream) {
  using namespace gemm;
  using Cf = pair::PairCfg<NH>;
  const CUtensorMap tA = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, K, lda, BM, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K, ldb, pair::BN2 / 2, 32,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  PairPlainSchedTf32 s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.cols = Cf::kCols;
  s.num_m = (M + 2 * BM - 1) / (2 * BM);
  s.num_n = (N + Cf::kCols - 1) / Cf::kCols;
  s.group_m = gemm_tuning().pair_group_m;
  StoreEpi e;
  e.C = C;
  e.ldc = ldc;
  e.M = M;
  e.N = N;
  e.alpha = alpha;
  e.out_f32 = 1;
  e.vec = c_vector_ok(C, ldc, true) ? 1 : 0;
  static bool attr_set[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_tf32_pair<NH>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmemBytes));
    attr_set[dev] = true;
  }
  const int pairs_max = num_sms(dev) / 2;
  const int tiles = s.num_m * s.num_n;
  const int grid = 2 * (tiles < pairs_max ? tiles : pairs_max);
  k_gemm_tf32_pair<NH><<<grid, Cf::kThreads, Cf::kSmemBytes, stream>>>(tA, tB, s, e, device_error_record(),
                                                                        default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}
}  // namespace

void gemm_tf32(const float* A, const float* B, float* C, int M, int N, int K, long long lda, long long ldb,
               long long ldc, float alpha, cudaStream_t stream, int bn) {
  NvtxRange nvtx("gicc::ops::gemm_tf32");
  using namespace gemm;
  using Cf = Cfg<256>;
  if (M <= 0 || N <= 0 || K <= 0) throw std::runtime_error("gicc::gemm_tf32: empty shape");
  if (lda % 4 || ldb % 4 || ldc < N || (reinterpret_cast<uintptr_t>(A) & 15) || (reinterpret_cast<uintptr_t>(B) & 15))
    throw std::runtime_error("gicc::gemm_tf32: 16-byte aligned A/B rows (lda, ldb % 4 == 0), ldc >= N");
  if (bn == 0) bn = default_tile(M, N);
  if (bn == 1024 || bn == 512) {
    if (bn == 1024) launch_tf32_pair<2>(A, B, C, M, N, K, lda, ldb, ldc, alpha, stream);
    else launch_tf32_pair<1>(A, B, C, M, N, K, lda, ldb, ldc, alpha, stream);
    return;
  }
  if (bn != 256) throw std::runtime_error("gicc::gemm_tf32: bn must be 0, 256, 512 or 1024");
  const CUtensorMap tA = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, M, K, lda, BM, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, N, K, ldb, 256, 32, CU_TENSOR_MAP_SWIZZLE_128B);
  PlainSchedTf32 s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.bn = 256;
  s.num_m = (M + BM - 1) / BM;
  s.num_n = (N + 255) / 256;
  s.group_m = gemm_tuning().group_m;
  s.l2hint = 0;
  StoreEpi e;
  e.C = C;
  e.ldc = ldc;
  e.M = M;
  e.N = N;
  e.alpha = alpha;
  e.out_f32 = 1;
  e.vec = c_vector_ok(C, ldc, true) ? 1 : 0;
  static bool attr_set[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr_set[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_tf32, cudaFuncAttributeMaxDynamicSharedMemorySize, Cf::kSmemBytes));
    attr_set[dev] = true;
  }
  const int tiles = s.num_m * s.num_n;
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  k_gemm_tf32<<<grid, kThreads, Cf::kSmemBytes, stream>>>(tA, tB, s, e, device_error_record(), default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}

void gemm_fp32(const float* A, const float* B, float* C, int M, int N, int K, long long lda, long long ldb,
               long long ldc, float alpha, float* work, cudaStream_t stream, int bn) {
  NvtxRange nvtx("gicc::ops::gemm_fp32");
  if (K % 4) throw std::runtime_error("gicc::gemm_fp32: K % 4 == 0");
  float* Ap = work;                          // [M][3K] = (hi, hi, lo)
  float* Bp = work + (size_t)M * 3 * K;      // [N][3K] = (hi, lo, hi)
  tf32_split(A, lda, M, K, Ap, 0, stream);
  tf32_split(B, ldb, N, K, Bp, 1, stream);
  gemm_tf32(Ap, Bp, C, M, N, 3 * K, 3LL * K, 3LL * K, ldc, alpha, stream, bn);
}

void gemm_tile_done_selftest(const void* A, const void* B, int M, int N, int K, uint32_t* counters, uint32_t skew_ns,
                             cudaStream_t stream) {
  using Cf = gemm::Cfg<256>;
  if (M % gemm::BM || N % 256 || K % gemm::BK) throw std::runtime_error("gicc::gemm_tile_done_selftest: M%128, N%256, K%64");
  const CUtensorMap tA = make_tmap_2d(A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, M, K, K, gemm::BM, gemm::BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, N, K, K, 256, gemm::BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  gemm::PlainSched s;
  s.M = M;
  s.N = N;
  s.K = K;
  s.bn = 256;
  s.num_m = M / gemm::BM;
  s.num_n = N / 256;
  s.group_m = 16;
  const int tiles = s.num_m * s.num_n;
  gemm::TileDoneCheckEpi e;
  e.num_n = s.num_n;
  e.bn = 256;
  e.warps_done = counters;
  e.published = counters + tiles;
  e.bad = counters + 2 * tiles;
  e.skew_ns = skew_ns;
  GICC_CUDA(cudaFuncSetAttribute(gemm::k_gemm_tile_done_check, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 Cf::kSmemBytes));
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  const int grid = tiles < num_sms(dev) ? tiles : num_sms(dev);
  gemm::k_gemm_tile_done_check<<<grid, gemm::kThreads, Cf::kSmemBytes, stream>>>(tA, tB, s, e, device_error_record(),
                                                                          default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}


namespace {
GemmTuning g_tuning;
bool g_tuning_set = false;  // set_gemm_tuning() wins over the environment
}
void set_gemm_tuning(const GemmTuning& t) {
  if (t.group_m < 1 || t.l2_hint < 0 || t.l2_hint > 2 || t.pair_group_m < 1 || t.pair_l2_hint < 0 ||
      t.pair_l2_hint > 2 || t.pair_prefetch < 0 || t.pair_prefetch > 64 || t.pair_tma_store < 0 ||
      t.pair_tma_store > 1)
    throw std::runtime_error(
        "gicc::set_gemm_tuning: group_m >= 1, l2_hint in 0..2, pair_group_m >= 1, pair_l2_hint in 0..2, "
        "pair_prefetch in 0..64, pair_tma_store 0 or 1");
  g_tuning = t;
  g_tuning_set = true;
}
GemmTuning gemm_tuning() {
  if (!g_tuning_set) {  // GICC_GEMM_GROUP_M / GICC_GEMM_L2_HINT, read once
    const Config c = config();
    g_tuning.group_m = c.gemm_group_m;
    g_tuning.l2_hint = c.gemm_l2_hint;
    g_tuning.pair_group_m = c.gemm_pair_group_m;
    g_tuning.pair_l2_hint = c.gemm_pair_l2_hint;
    g_tuning.pair_prefetch = c.gemm_pair_prefetch;
    g_tuning.pair_tma_store = c.gemm_pair_tma_store;
    g_tuning_set = true;
  }
  return g_tuning;
}

// Default tile for an M x N output: the 256 x 512 pair tile moves half the operand bytes
// per FLOP of the 128 x 256 single-CTA tile (and runs faster under the power cap), unless
// its coarser tiles leave a markedly larger share of the last wave of CTA pairs idle.
static int default_tile(int M, int N) {
  const int sms = num_sms();
  auto fill = [](long long tiles, int slots) {
    const long long waves = (tiles + slots - 1) / slots;
    return (double)tiles / (double)(waves * slots);
  };
  const long long t1024 = (long long)((M + 255) / 256) * ((N + 511) / 512);
  const long long t256 = (long long)((M + 127) / 128) * ((N + 255) / 256);
  if (t1024 < sms / 2) return 256;
  return fill(t1024, sms / 2) >= fill(t256, sms) - 0.05 ? 1024 : 256;
}

void gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
               long long ldc, bool out_f32, float alpha, int bn, cudaStream_t stream) {
  NvtxRange nvtx("gicc::ops::gemm_bf16");
  if (M <= 0 || N <= 0 || K <= 0) throw std::runtime_error("gicc::gemm_bf16: empty shape");
  if (K % 8 != 0 || lda % 8 != 0 || ldb % 8 != 0)
    throw std::runtime_error("gicc::gemm_bf16: K and leading dimensions of A/B must be multiples of 8 (16-byte TMA rows)");
  if (ldc < N) throw std::runtime_error("gicc::gemm_bf16: ldc < N");
  if (bn == 0) bn = default_tile(M, N);
  switch (bn) {
    case 256: gemm::launch_plain<256>(A, B, C, M, N, K, lda, ldb, ldc, out_f32, alpha, stream); break;
    case 128: gemm::launch_plain<128>(A, B, C, M, N, K, lda, ldb, ldc, out_f32, alpha, stream); break;
    case 512: gemm::launch_pair<1>(A, B, C, M, N, K, lda, ldb, ldc, out_f32, alpha, stream); break;   // pairs, 256 x 256
    case 1024: gemm::launch_pair<2>(A, B, C, M, N, K, lda, ldb, ldc, out_f32, alpha, stream); break;  // pairs, 256 x 512
    default: throw std::runtime_error("gicc::gemm_bf16: bn must be 128, 256, 512 (CTA pairs, 256 x 256) or 1024 "
                                      "(CTA pairs, 256 x 512)");
  }
}

}  // namespace ops
}  // namespace gicc

GICC_API int gicc_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                            long long ldc, int out_f32, float alpha, cudaStream_t stream) {
  return gicc::guarded([&] { gicc::ops::gemm_bf16(A, B, C, M, N, K, lda, ldb, ldc, out_f32 != 0, alpha, 0, stream); });
}
