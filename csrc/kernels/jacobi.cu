// jacobi.cu -- 2-D 5-point Jacobi (fp32) with halo puts fused into the stencil kernel.
//
// Reference: examples/gicc/jacobi.cu:66-162 -- a 32x32-thread SIMT stencil whose *last*
// finishing block (atomicInc counter) RDMA-writes both halo rows after every block is done,
// followed by a host MPI barrier per iteration (jacobi.cu:430-471).
//
// Here:
//  * one thread updates 4 adjacent columns (one float4) for RUN consecutive rows, keeping
//    the rows above/below in registers (every interior value is read from HBM once);
//    left/right neighbours come from warp shuffles;
//  * the CTAs that own this rank's first / last row run first (lowest block ids) and
//    store those rows straight into the neighbour's halo row over NVLink as they are
//    computed, then bump the neighbour's arrival counter with a release add;
//  * the next iteration's boundary CTAs wait (bounded) on their own arrival counter
//    before reading the halo -- no host barrier, no separate copy kernel;
//  * the update is ((e + w) + (n + s)) * 0.25 with explicit round-to-nearest adds/muls,
//    bit-identical to the CPU oracle.
#include <cuda_runtime.h>

#include "gicc/device/comm.cuh"
#include "gicc/config.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace {

constexpr int kThreads = 256;           // 8 warps x 128 columns = 1024 columns per CTA
constexpr int kColsPerCta = kThreads * 4;
constexpr int kRun = 16;                // rows per CTA

struct JacobiArgs {
  const float* a;  // [rows+2][nx] read buffer (row 0 / rows+1 are halos)
  float* b;        // [rows+2][nx] write buffer
  int nx, rows;
  float* top_dst;                // upper neighbour's bottom halo row in its write buffer (or null)
  float* bot_dst;                // lower neighbour's top halo row in its write buffer (or null)
  uint64_t* top_sig_remote;      // upper neighbour's bottom-halo arrival counter
  uint64_t* bot_sig_remote;      // lower neighbour's top-halo arrival counter
  const uint64_t* top_flag;      // my top-halo arrival counter
  const uint64_t* bot_flag;      // my bottom-halo arrival counter
  uint64_t wait_top, wait_bot;   // counts that make the halos of the previous iteration valid
  double* norm;                  // optional: sum of (new-old)^2
  ErrorRecord* err;
  uint64_t timeout_ns;
  int rank;
};

__device__ __forceinline__ float upd(float e, float w, float n, float s) {
  return __fmul_rn(__fadd_rn(__fadd_rn(e, w), __fadd_rn(n, s)), 0.25f);
}

// Rows [r0, r1) of column chunk bx (r1 <= rows + 1): reads a (rows r0-1 .. r1), writes b;
// row 1 and row `rows` also go to top_dst / bot_dst when those are set.  Returns this
// thread's sum of squared updates when want_norm, else 0.
__device__ __forceinline__ float jacobi_rows(const float* A, float* B, int nx_, int nrows, int bx, int r0, int r1,
                                             float* top_dst, float* bot_dst, bool want_norm) {
  const int lane = threadIdx.x & 31;
  const int j0 = bx * kColsPerCta + threadIdx.x * 4;  // first column of this thread
  const bool active = j0 < nx_;
  const size_t nx = (size_t)nx_;

  // Issue every load of the run up front (kRun + 2 rows, plus the warp-edge columns) so
  // ~20 independent 16-byte loads per thread are in flight: HBM latency is hidden by
  // memory-level parallelism instead of occupancy.
  float4 rows[kRun + 2];
  float edge[kRun];
#pragma unroll
  for (int i = 0; i < kRun + 2; ++i) {
    const int r = r0 - 1 + i;
    rows[i] = (active && r <= r1) ? __ldcs(reinterpret_cast<const float4*>(A + (size_t)r * nx + j0))
                                  : make_float4(0, 0, 0, 0);
  }
  const bool edge_lane = (lane == 0 && active && j0 > 0) || (lane == 31 && active && j0 + 4 < nx_);
  const int ecol = lane == 0 ? j0 - 1 : j0 + 4;
#pragma unroll
  for (int i = 0; i < kRun; ++i) edge[i] = (edge_lane && r0 + i < r1) ? A[(size_t)(r0 + i) * nx + ecol] : 0.f;
  float sq = 0.f;
#pragma unroll
  for (int i = 0; i < kRun; ++i) {
    const int r = r0 + i;
    if (r >= r1) break;
    const float4 up = rows[i], mid = rows[i + 1], dn = rows[i + 2];
    float left = __shfl_up_sync(0xffffffffu, mid.w, 1);
    float right = __shfl_down_sync(0xffffffffu, mid.x, 1);
    if (lane == 0 && active && j0 > 0) left = edge[i];
    if (lane == 31 && active && j0 + 4 < nx_) right = edge[i];
    float4 o;
    o.x = upd(mid.y, left, up.x, dn.x);
    o.y = upd(mid.z, mid.x, up.y, dn.y);
    o.z = upd(mid.w, mid.y, up.z, dn.z);
    o.w = upd(right, mid.z, up.w, dn.w);
    // Dirichlet columns keep their value
    if (j0 == 0) o.x = mid.x;
    if (j0 + 4 >= nx_) o.w = mid.w;
    if (active) {
      __stcs(reinterpret_cast<float4*>(B + (size_t)r * nx + j0), o);
      if (r == 1 && top_dst) *reinterpret_cast<float4*>(top_dst + j0) = o;
      if (r == nrows && bot_dst) *reinterpret_cast<float4*>(bot_dst + j0) = o;
      if (want_norm) {
        const float dx = o.x - mid.x, dy = o.y - mid.y, dz = o.z - mid.z, dw = o.w - mid.w;
        sq += dx * dx + dy * dy + dz * dz + dw * dw;
      }
    }
  }
  return sq;
}

__global__ void __launch_bounds__(kThreads) k_jacobi(JacobiArgs p) {
  const int nbx = (p.nx + kColsPerCta - 1) / kColsPerCta;
  const int nby = (p.rows + kRun - 1) / kRun;
  // boundary CTAs first: by = 0, then by = nby-1, then the rest
  int bid = blockIdx.x, bx, by;
  if (bid < nbx) {
    bx = bid;
    by = 0;
  } else if (nby > 1 && bid < 2 * nbx) {
    bx = bid - nbx;
    by = nby - 1;
  } else {
    const int rest = bid - (nby > 1 ? 2 : 1) * nbx;
    bx = rest % nbx;
    by = 1 + rest / nbx;
  }
  const bool has_top = by == 0, has_bot = by == nby - 1;
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (has_top && p.top_flag &&
        signal_wait_until(p.top_flag, proto::CMP_GE, p.wait_top, p.timeout_ns, p.err, p.rank, p.rank - 1,
                          W_JACOBI_HALO) != GICC_OK)
      ok = 0;
    if (has_bot && p.bot_flag &&
        signal_wait_until(p.bot_flag, proto::CMP_GE, p.wait_bot, p.timeout_ns, p.err, p.rank, p.rank + 1,
                          W_JACOBI_HALO) != GICC_OK)
      ok = 0;
  }
  __syncthreads();
  if (!ok) return;

  const int lane = threadIdx.x & 31;
  const int r0 = 1 + by * kRun;                         // first local row of the run
  const int r1 = min(r0 + kRun, p.rows + 1);            // one past the last
  float sq = jacobi_rows(p.a, p.b, p.nx, p.rows, bx, r0, r1, p.top_dst, p.bot_dst, p.norm != nullptr);
  if (p.norm) {
    for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
    if (lane == 0 && sq != 0.f) atomicAdd(p.norm, (double)sq);
  }
  if ((has_top && p.top_dst) || (has_bot && p.bot_dst)) {
    ptx::fence_acq_rel_sys();  // this thread's halo stores are visible system-wide
    __syncthreads();
    if (threadIdx.x == 0) {
      if (has_top && p.top_dst) ptx::red_release_sys_add(p.top_sig_remote, 1);
      if (has_bot && p.bot_dst) ptx::red_release_sys_add(p.bot_sig_remote, 1);
    }
  }
}

// Persistent multi-iteration variant: one cooperative launch runs `iters` iterations.  CTA
// c owns a contiguous block of rows; before iteration gi it waits until the CTAs owning the
// blocks above and below finished iteration gi-1 (per-CTA monotonic done counters, local
// memory, acquire/release at GPU scope) -- that covers both the rows it reads and the rows
// it overwrites -- and, if it owns row 1 or row `rows`, until the neighbour rank's halo row
// of iteration gi-1 arrived.  The CTA that owns row 1 does its first run of every column
// chunk first and the one that owns row `rows` its last run, so the halo rows leave early;
// each pusher then adds one arrival per column chunk, the same count the one-launch-per-
// iteration kernel produces, so the two kernels can be mixed on the same counters.
struct JacobiPArgs {
  float* buf[2];        // [rows+2][nx]; iteration gi reads buf[gi & 1] and writes the other
  int nx, rows;
  float* top_dst[2];    // upper neighbour's bottom halo row in its buffer p (null: none)
  float* bot_dst[2];    // lower neighbour's top halo row in its buffer p
  uint64_t* top_sig_remote;
  uint64_t* bot_sig_remote;
  const uint64_t* top_flag;
  const uint64_t* bot_flag;
  uint64_t iter0;       // global index of the first iteration of this launch
  int iters;
  uint64_t* done;       // [gridDim.x] iterations finished per CTA (monotonic)
  double* norm;         // optional: sum of squared updates of the last iteration
  ErrorRecord* err;
  uint64_t timeout_ns;
  int rank;
};

__global__ void __launch_bounds__(kThreads, 2) k_jacobi_persistent(JacobiPArgs p) {
  const int G = gridDim.x, c = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int nbx = (p.nx + kColsPerCta - 1) / kColsPerCta;
  const int per = (p.rows + G - 1) / G;
  const int lo = min(1 + c * per, p.rows + 1), hi = min(1 + (c + 1) * per, p.rows + 1);  // rows [lo, hi)
  const bool own_top = lo == 1 && lo < hi, own_bot = lo <= p.rows && p.rows < hi;
  const int nrun = (hi - lo + kRun - 1) / kRun;
  __shared__ int ok_s;
  for (int it = 0; it < p.iters; ++it) {
    const uint64_t gi = p.iter0 + it;
    const int rd = (int)(gi & 1), wr = rd ^ 1;
    if (threadIdx.x == 0) {
      int ok = 1;
      if (it > 0) {  // the previous launch finished before this one started
        if (c > 0 && !proto::wait_until<proto::DevMem>(p.done + c - 1, proto::CMP_GE, gi, p.timeout_ns, nullptr))
          ok = 0;
        if (c + 1 < G && !proto::wait_until<proto::DevMem>(p.done + c + 1, proto::CMP_GE, gi, p.timeout_ns, nullptr))
          ok = 0;
        if (!ok) report_error(p.err, GICC_ETIMEDOUT, W_JACOBI_HALO, p.rank, p.rank, 0, gi);
      }
      if (ok && own_top && p.top_flag &&
          signal_wait_until(p.top_flag, proto::CMP_GE, gi * (uint64_t)nbx, p.timeout_ns, p.err, p.rank, p.rank - 1,
                            W_JACOBI_HALO) != GICC_OK)
        ok = 0;
      if (ok && own_bot && p.bot_flag &&
          signal_wait_until(p.bot_flag, proto::CMP_GE, gi * (uint64_t)nbx, p.timeout_ns, p.err, p.rank, p.rank + 1,
                            W_JACOBI_HALO) != GICC_OK)
        ok = 0;
      ok_s = ok;
    }
    __syncthreads();
    if (!ok_s) return;  // the error is recorded; every CTA that waits on this one times out too
    const float* A = p.buf[rd];
    float* B = p.buf[wr];
    float* tdst = own_top ? p.top_dst[wr] : nullptr;
    float* bdst = own_bot ? p.bot_dst[wr] : nullptr;
    const bool want_norm = p.norm && it == p.iters - 1;
    float sq = 0.f;
    for (int k = 0; k < nrun; ++k) {
      // the bottom-row owner (unless it also owns row 1) walks its runs upwards
      const int run = (own_bot && !own_top) ? nrun - 1 - k : k;
      const int r0 = lo + run * kRun, r1 = min(r0 + kRun, hi);
      for (int bx = 0; bx < nbx; ++bx) sq += jacobi_rows(A, B, p.nx, p.rows, bx, r0, r1, tdst, bdst, want_norm);
      // a halo row of this iteration is complete in every column chunk: publish it with one
      // arrival per chunk (the count of the one-launch-per-iteration kernel)
      const bool pub_top = tdst && r0 == 1;
      const bool pub_bot = bdst && r0 <= p.rows && p.rows < r1;
      if (pub_top || pub_bot) {
        ptx::fence_acq_rel_sys();
        __syncthreads();
        if (threadIdx.x == 0) {
          if (pub_top) ptx::red_release_sys_add(p.top_sig_remote, (uint64_t)nbx);
          if (pub_bot) ptx::red_release_sys_add(p.bot_sig_remote, (uint64_t)nbx);
        }
      }
    }
    if (want_norm) {
      for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
      if (lane == 0 && sq != 0.f) atomicAdd(p.norm, (double)sq);
    }
    __syncthreads();  // every thread of this CTA finished reading and writing iteration gi
    if (threadIdx.x == 0) {
      __threadfence();
      ptx::st_release_gpu(p.done + c, gi + 1);
    }
  }
}

// splitmix64 of (seed, global index) -> uniform [0,1) with 24 random bits.
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t idx) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ull + idx + 1;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

// Initialise local rows [0, rows+2) = global rows [g0-1, g0+rows]: top edge 1.0, other
// edges 0, interior U[0,1) from `seed` keyed by the global index.
__global__ void k_jacobi_init(float* a, float* b, int nx, int ny, int rows, int g0, uint64_t seed) {
  const size_t total = (size_t)(rows + 2) * nx;
  for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (size_t)gridDim.x * blockDim.x) {
    const int lr = (int)(k / nx), j = (int)(k % nx);
    const int g = g0 - 1 + lr;
    float v;
    if (g <= 0)
      v = 1.0f;
    else if (g >= ny - 1 || j == 0 || j == nx - 1)
      v = 0.0f;
    else
      v = hash_uniform(seed, (uint64_t)g * (uint64_t)nx + j);
    a[k] = v;
    if (b) b[k] = v;
  }
}

}  // namespace

namespace ops {

void jacobi_init(float* a, float* b, int nx, int ny, int rows, int g0, uint64_t seed, cudaStream_t s) {
  k_jacobi_init<<<4 * num_sms(), 256, 0, s>>>(a, b, nx, ny, rows, g0, seed);
  GICC_CUDA(cudaGetLastError());
}

void jacobi_step(const JacobiStep& st, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::jacobi_step");
  if (st.nx % 4 != 0) throw std::runtime_error("gicc::jacobi: nx must be a multiple of 4");
  if (st.rows < 1) throw std::runtime_error("gicc::jacobi: a rank needs at least one row");
  JacobiArgs p;
  p.a = st.a;
  p.b = st.b;
  p.nx = st.nx;
  p.rows = st.rows;
  p.top_dst = st.top_dst;
  p.bot_dst = st.bot_dst;
  p.top_sig_remote = st.top_sig_remote;
  p.bot_sig_remote = st.bot_sig_remote;
  p.top_flag = st.top_flag;
  p.bot_flag = st.bot_flag;
  p.wait_top = st.wait_top;
  p.wait_bot = st.wait_bot;
  p.norm = st.norm;
  p.err = device_error_record();
  p.timeout_ns = st.timeout_ns ? st.timeout_ns : default_timeout_ns();
  p.rank = st.rank;
  const int nbx = (st.nx + kColsPerCta - 1) / kColsPerCta;
  const int nby = (st.rows + kRun - 1) / kRun;
  k_jacobi<<<nbx * nby, kThreads, 0, s>>>(p);
  GICC_CUDA(cudaGetLastError());
}

int jacobi_ctas_per_row(int nx) { return (nx + kColsPerCta - 1) / kColsPerCta; }

int jacobi_persistent_grid(int rows) {
  // every CTA resident at once (cooperative launch), never more CTAs than rows
  static int per_sm[64] = {0};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && !per_sm[dev])
    GICC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm[dev], k_jacobi_persistent, kThreads, 0));
  const int resident = (dev < 64 ? per_sm[dev] : 1) * num_sms(dev);
  return rows < resident ? rows : resident;
}

void jacobi_run(const JacobiRun& r, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::jacobi_run");
  if (r.nx % 4 != 0) throw std::runtime_error("gicc::jacobi_run: nx must be a multiple of 4");
  if (r.rows < 1) throw std::runtime_error("gicc::jacobi_run: a rank needs at least one row");
  if (!r.buf[0] || !r.buf[1] || !r.done) throw std::runtime_error("gicc::jacobi_run: buf[2] and done are required");
  if ((r.top_dst[0] || r.top_dst[1]) && (!r.top_dst[0] || !r.top_dst[1] || !r.top_sig_remote))
    throw std::runtime_error("gicc::jacobi_run: top_dst needs both parities and top_sig_remote");
  if ((r.bot_dst[0] || r.bot_dst[1]) && (!r.bot_dst[0] || !r.bot_dst[1] || !r.bot_sig_remote))
    throw std::runtime_error("gicc::jacobi_run: bot_dst needs both parities and bot_sig_remote");
  if (r.iters <= 0) return;
  JacobiPArgs p;
  for (int i = 0; i < 2; ++i) {
    p.buf[i] = r.buf[i];
    p.top_dst[i] = r.top_dst[i];
    p.bot_dst[i] = r.bot_dst[i];
  }
  p.nx = r.nx;
  p.rows = r.rows;
  p.top_sig_remote = r.top_sig_remote;
  p.bot_sig_remote = r.bot_sig_remote;
  p.top_flag = r.top_flag;
  p.bot_flag = r.bot_flag;
  p.iter0 = r.iter0;
  p.iters = r.iters;
  p.done = r.done;
  p.norm = r.norm;
  p.err = device_error_record();
  p.timeout_ns = r.timeout_ns ? r.timeout_ns : default_timeout_ns();
  p.rank = r.rank;
  void* args[] = {&p};
  GICC_CUDA(cudaLaunchCooperativeKernel((const void*)k_jacobi_persistent, dim3(jacobi_persistent_grid(r.rows)),
                                        dim3(kThreads), args, 0, s));
}

}  // namespace ops
}  // namespace gicc
