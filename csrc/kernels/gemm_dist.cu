// gemm_dist.cu -- distributed GEMM with the NVLink transfer fused into the tcgen05 kernel.
//
// all-gather -> GEMM (AG):  C[:, cols_r] = A_full[M,K] * B_r[Ns,K]^T
//   A is row-sharded; rank r's shard already sits in rows [r*Ms, (r+1)*Ms) of its
//   symmetric A_full buffer.  The communication warps of `comm_ctas` CTAs move that shard
//   in 128-row bands (units of a band spread over those CTAs):
//   * NVLS (default when the node has it): each unit is written once through the landing
//     buffer's multicast view (multimem.st) and one multimem.red bumps the (source, band)
//     arrival counter on every GPU; all shards arrive at once, band by band, so consumers
//     take the local shard first and then go band-major over the other sources;
//   * unicast: 16-byte stores into every peer's A_full, release add on that peer's
//     counter; pushes go to rank r-1 first, r-2 next, ..., the order in which each receiver
//     consumes them (local shard first, then shard r+1, r+2, ...);
//   * copy engines (ops::ag_transfer_ce, an option): a side stream copies the bands and
//     writes the counters with stream memory operations, and the kernel only waits.
//   Tiles come from a global counter (dynamic schedule), so the CTAs that push take fewer
//   tiles; an SM whose warps store to NVLink also slows its own TMA loads.  The TMA producer
//   waits (bounded, acquire) on a band's counter before loading it, so band b+1 travels
//   while the tensor cores work on band b.
//
// GEMM -> reduce-scatter (RS): rank r owns output rows [r*Mr, (r+1)*Mr); K is sharded.
//   * NVLS (default when available): every rank stores its bf16 partial of the whole output
//     in its own staging buffer; when the last tile of band (o, b) is stored, rank r tells
//     owner o; the owner's reduce warps (in `comm_ctas` CTAs, or -- with the join option --
//     in every CTA that has run out of tiles) sum the band of all ranks inside the switch
//     with multimem.ld_reduce once all ranks reported it, and write the result;
//   * unicast: tiles walked owner by owner (r+1, r+2, ..., own rows last); the epilogue
//     stores a remote owner's tile into that owner's slot for source r and releases a
//     (source, band) counter; for its own rows it waits for every source's tiles, adds them
//     to its TMEM accumulator and writes the bf16 result.
//
// Both use epoch counters (one epoch per call) and double-buffered landing / staging areas;
// a rank writes an area of parity p only after every rank that reads it reported (per-CTA
// done counters) that it finished the call that last used parity p.
//
// The reference's distributed matmul (examples/gicc/mm.cu:116-225) rotates fp32 B stripes
// around a ring with one <<<1,1>>> put per step and a SIMT atomicAdd kernel; this is the
// same all-gather-and-multiply pattern with tensor-core tiles and fine-grained overlap.
#include <cuda_runtime.h>

#include "gicc/device/comm.cuh"
#include "gicc/device/gemm_core.cuh"
#include "gicc/device/gemm_core2.cuh"
#include "gicc/config.hpp"
#include "gicc/driver.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace gemm {
namespace {

constexpr int kMaxR = 16;
constexpr int kCommWarpsAG = 4;

struct DoneTable {
  uint64_t* p[kMaxR];  // each rank's [n] CTA-done counters, mapped here
};

__device__ __forceinline__ bool wait_counter(const uint64_t* p, uint64_t target, uint64_t timeout_ns,
                                             volatile int* abort_flag) {
  if (ptx::ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = ptx::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (ptx::ld_acquire_sys(p) >= target) return true;
    if ((i & 63) == 0) {
      if (abort_flag && *abort_flag) return false;
      if (ptx::globaltimer() - t0 > timeout_ns) return false;
    }
  }
}

// Copy nv 16-byte vectors with the 128 threads of the communication warps, software-
// pipelined: the loads of batch b+1 (8 vectors per thread) are in flight while batch b is
// stored, so each thread keeps 16 vectors moving and the SM's push rate is not bound by
// one load latency per batch.
template <int kT>
__device__ __forceinline__ void copy_unit(const uint4* __restrict__ src, uint4* __restrict__ dst, size_t nv, int tid) {
  constexpr size_t step = 8 * kT;
  const size_t nbatch = nv / step;
  uint4 va[8], vb[8];
  auto load = [&](uint4* v, size_t b) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ptx::ld_v4_nc(src + b * step + tid + j * kT);
  };
  auto store = [&](const uint4* v, size_t b) {
#pragma unroll
    for (int j = 0; j < 8; ++j) ptx::st_v4_na(dst + b * step + tid + j * kT, v[j]);
  };
  if (nbatch > 0) load(va, 0);
  size_t b = 0;
  for (; b + 1 < nbatch; b += 2) {
    load(vb, b + 1);
    store(va, b);
    if (b + 2 < nbatch) load(va, b + 2);
    store(vb, b + 1);
  }
  if (b < nbatch) store(va, b);  // odd count: the last batch is loaded, not yet stored
  for (size_t i = nbatch * step + tid; i < nv; i += kT) ptx::st_v4_na(dst + i, ptx::ld_v4_nc(src + i));
}

// Same, with the stores going through an NVLS multicast view (multimem.st: one store,
// delivered by the NVSwitch to every GPU of the multicast object).
template <int kT>
__device__ __forceinline__ void copy_unit_mc(const uint4* __restrict__ src, uint4* dst_mc, size_t nv, int tid) {
  constexpr size_t step = 8 * kT;
  const size_t nbatch = nv / step;
  uint4 va[8], vb[8];
  auto load = [&](uint4* v, size_t b) {
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = ptx::ld_v4_nc(src + b * step + tid + j * kT);
  };
  auto store = [&](const uint4* v, size_t b) {
#pragma unroll
    for (int j = 0; j < 8; ++j) ptx::multimem_st_v4(dst_mc + b * step + tid + j * kT, v[j]);
  };
  if (nbatch > 0) load(va, 0);
  size_t b = 0;
  for (; b + 1 < nbatch; b += 2) {
    load(vb, b + 1);
    store(va, b);
    if (b + 2 < nbatch) load(va, b + 2);
    store(vb, b + 1);
  }
  if (b < nbatch) store(va, b);
  for (size_t i = nbatch * step + tid; i < nv; i += kT) ptx::multimem_st_v4(dst_mc + i, ptx::ld_v4_nc(src + i));
}

// ------------------------------------------------------------------------------------------
// all-gather -> GEMM
// ------------------------------------------------------------------------------------------
struct AgSched {
  static constexpr int kCommWarps = kCommWarpsAG;
  static constexpr bool kDynamic = true;  // CTAs that push take fewer tiles
  int n, r, M, Ns, K, Ms, nb, bn, num_n, Q, G;
  int C;                           // CTAs that push (blockIdx.x < C); the rest only compute
  const uint16_t* a_local;         // my A_full (this parity)
  uint16_t* a_peer[kMaxR];         // every rank's A_full (this parity), mapped here
  const uint64_t* arrivals;        // my counters [n][nb]
  uint64_t* arrivals_peer[kMaxR];  // each rank's counter base
  const uint64_t* done_local;      // [n] CTA-exit counts received from each rank
  uint64_t epoch;                  // this call, >= 1
  // Diagnostics (both off in normal use).  trace: %globaltimer stamps, layout in
  // AgTrace below.  diag bit 0: skip the transfer and the arrival waits, which times the
  // tensor-core work of the fused kernel alone (the output is then not the product).
  uint64_t* trace;
  int diag;
  unsigned long long* tile_counter;  // local word, monotonic over calls
  unsigned long long tile_base;      // (epoch - 1) * (tiles + grid): every CTA takes one index past the end
  // NVLS mode (both non-null): the shard is written once through the multicast view of
  // A_full and lands in every GPU; one multimem.red bumps every GPU's arrival counter.
  uint16_t* a_mc;
  uint64_t* arrivals_mc;

  __device__ int num_tiles() const { return n * nb * num_n; }
  __device__ int num_units() const { return (diag & 3) ? 0 : (a_mc ? nb * Q : (n - 1) * nb * Q); }
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(tile_counter, 1ull) - tile_base;
    return v < (unsigned long long)num_tiles() ? (int)v : num_tiles();
  }
  __device__ int trace_tile(const TileInfo& ti) const { return (ti.m0 / BM) * num_n + ti.n0 / bn; }
  __device__ TileInfo tile(int t) const {
    // Local shard first.  Unicast push: then shard r+1, r+2, ... (each source pushes to
    // its consumers in that order).  NVLS: every shard arrives at once, band by band, so
    // the remote tiles go band-major over the sources.  Grouped rasterisation (16 rows of
    // tiles) throughout, for L2 reuse of A and B.
    const int per = nb * num_n;
    int k, b, nbk;
    if (a_mc && t >= per) {
      int vm;
      raster(t - per, nb * (n - 1), num_n, 16, vm, nbk);
      b = vm / (n - 1);
      k = 1 + vm - b * (n - 1);
    } else {
      k = t / per;
      raster(t - k * per, nb, num_n, 16, b, nbk);
    }
    const int s = (r + k) % n;
    TileInfo ti;
    ti.m0 = s * Ms + b * BM;
    ti.a_row = ti.m0;
    ti.n0 = nbk * bn;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = s;
    ti.aux2 = b;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo& ti, uint64_t timeout_ns, volatile int* abort_flag,
                                ErrorRecord* err) const {
    uint64_t* tr = trace ? trace + 2 * (size_t)trace_tile(ti) : nullptr;
    if (tr) tr[0] = ptx::globaltimer();
    if (ti.aux != r && !(diag & 1)) {
      const uint64_t* c = arrivals + (size_t)ti.aux * nb + ti.aux2;
      const uint64_t target = epoch * (uint64_t)Q;
      if (!wait_counter(c, target, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_AG_FLAG, r, ti.aux, ptx::ld_relaxed_sys(c), target);
        return false;
      }
      ptx::fence_proxy_async_global();  // peer's generic-proxy stores -> our TMA reads
    }
    if (tr) tr[1] = ptx::globaltimer();
    return true;
  }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
  }

  // Push this rank's shard to the peers: unit u = ((k-1)*nb + b)*Q + q goes to rank r-k.
  __device__ void comm(int cw, int lane, volatile int* abort_flag, ErrorRecord* err, uint64_t timeout_ns) const {
    __shared__ int comm_stop;
    const int tid = cw * 32 + lane;
    constexpr int kT = kCommWarps * 32;
    const size_t band_bytes = (size_t)BM * K * 2;
    const size_t unit_bytes = band_bytes / Q;
    const int U = num_units();
    uint64_t* tr = trace ? trace + 3 * (size_t)num_tiles() : nullptr;
    int last_d = -1;
    if ((int)blockIdx.x >= C) return;
    if (a_mc) {
      // NVLS: unit u = b*Q + q of my shard, written to every GPU at once.  First make sure
      // that every peer finished the call that last used this parity.
      if (tid == 0) {
        int stop = *abort_flag;
        for (int d = 0; d < n && !stop && epoch > 2 && U > 0; ++d) {
          if (d == r) continue;
          const uint64_t target = (epoch - 2) * (uint64_t)G;
          if (!wait_counter(done_local + d, target, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_AG_FLAG, r, d, ptx::ld_relaxed_sys(done_local + d), target);
            *abort_flag = 1;
            stop = 1;
          }
        }
        comm_stop = stop;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (comm_stop) return;
      for (int u = blockIdx.x; u < U && !*abort_flag; u += C) {
        const int b = u / Q, q = u - (u / Q) * Q;
        if (tr && tid == 0) tr[2 * u] = ptx::globaltimer();
        const size_t off = ((size_t)(r * Ms + b * BM) * K * 2) + (size_t)q * unit_bytes;
        copy_unit_mc<kT>(reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a_local) + off),
                         reinterpret_cast<uint4*>(reinterpret_cast<char*>(a_mc) + off), unit_bytes / 16, tid);
        ptx::fence_acq_rel_sys();
        asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
        if (tid == 0) ptx::multimem_red_release_add_u64(arrivals_mc + (size_t)r * nb + b, 1);
        if (tr && tid == 0) tr[2 * u + 1] = ptx::globaltimer();
      }
      return;
    }
    for (int u = blockIdx.x; u < U; u += C) {
      const int k = 1 + u / (nb * Q);
      const int rem = u - (k - 1) * nb * Q;
      const int b = rem / Q, q = rem - (rem / Q) * Q;
      const int d = (r - k + n) % n;
      if (tid == 0) {
        int stop = *abort_flag;
        if (!stop && d != last_d && epoch > 2) {
          const uint64_t target = (epoch - 2) * (uint64_t)G;
          if (!wait_counter(done_local + d, target, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_AG_FLAG, r, d, ptx::ld_relaxed_sys(done_local + d), target);
            *abort_flag = 1;
            stop = 1;
          }
        }
        comm_stop = stop;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (comm_stop) break;
      last_d = d;
      if (tr && tid == 0) tr[2 * u] = ptx::globaltimer();
      const size_t off = ((size_t)(r * Ms + b * BM) * K * 2) + (size_t)q * unit_bytes;
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const char*>(a_local) + off);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<char*>(a_peer[d]) + off);
      copy_unit<kT>(src, dst, unit_bytes / 16, tid);
      ptx::fence_acq_rel_sys();
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (tid == 0) ptx::red_release_sys_add(arrivals_peer[d] + (size_t)r * nb + b, 1);
      if (tr && tid == 0) tr[2 * u + 1] = ptx::globaltimer();
    }
  }
};
// The same all-gather GEMM on CTA pairs (cta_group::2): tiles of 256 rows x NH*256 columns,
// numbered like AgSched's (local shard first, then band-major over the other shards) over
// pair bands of 256 rows.  Each CTA of a pair loads its own 128-row band of A, so each
// producer waits for its own band's arrival counter.  The transfer (comm warps) is AgSched's.
template <int NH>
struct AgPairSched : AgSched {
  int nb2;  // 256-row pair bands per shard
  __device__ int num_tiles() const { return n * nb2 * num_n; }
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(tile_counter, 1ull) - tile_base;
    return v < (unsigned long long)num_tiles() ? (int)v : num_tiles();
  }
  __device__ TileInfo tile(int t) const {
    const int per = nb2 * num_n;
    int k, b, nbk;
    if (a_mc && t >= per) {
      int vm;
      raster(t - per, nb2 * (n - 1), num_n, 8, vm, nbk);
      b = vm / (n - 1);
      k = 1 + vm - b * (n - 1);
    } else {
      k = t / per;
      raster(t - k * per, nb2, num_n, 8, b, nbk);
    }
    const int s = (r + k) % n;
    TileInfo ti;
    ti.m0 = s * Ms + b * 2 * BM;
    ti.a_row = ti.m0;
    ti.n0 = nbk * NH * 256;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = s;
    ti.aux2 = 2 * b;  // the pair's first 128-row band
    return ti;
  }
  __device__ bool producer_wait(const TileInfo& ti, int crank, uint64_t timeout_ns, volatile int* abort_flag,
                                ErrorRecord* err) const {
    if (ti.aux != r && !(diag & 1)) {
      const uint64_t* c = arrivals + (size_t)ti.aux * nb + ti.aux2 + crank;
      const uint64_t target = epoch * (uint64_t)Q;
      if (!wait_counter(c, target, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_AG_FLAG, r, ti.aux, ptx::ld_relaxed_sys(c), target);
        return false;
      }
      ptx::fence_proxy_async_global();  // peer's generic-proxy stores -> our TMA reads
    }
    return true;
  }
};

// Trace layout (uint64 %globaltimer ns), T = tiles (m-block major), U = (n-1)*nb*Q units:
//   [2t, 2t+1]        producer: before / after the wait for tile t's A band
//   [2T + t]          epilogue: tile t stored (first epilogue warp)
//   [3T + 2u, +1]     comm: unit u push start / arrival released
//   [3T + 2U + 2c, +1] CTA c: start / end

struct PlainStoreEpi {
  static constexpr bool kNeedsTileDone = false;
  static constexpr bool kPairHalves = false;
  static constexpr bool kStagedStore = true;  // the CTA-pair core may store C through TMA
  uint16_t* C;
  long long ldc;
  int M, N;
  uint64_t* trace_epi;  // diagnostics: [tile] stamp when stored, or null
  int num_n, bn;
  int use_tma = 0;                   // C stored as 32 x 32 boxes by TMA (tmC valid; pair kernels)
  const CUtensorMap* tmC = nullptr;  // set by the kernel (a __grid_constant__ parameter)
  __device__ bool staged() const { return use_tma != 0; }
  __device__ const CUtensorMap* tmap() const { return tmC; }
  __device__ bool chunk_in_bounds(const TileInfo& ti, int row0, int c) const {
    return ti.m0 + row0 < M && ti.n0 + c < N;
  }
  __device__ __forceinline__ void pack(const uint32_t* r, uint4* v) const {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      v[j].x = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
      v[j].y = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
      v[j].z = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
      v[j].w = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
    }
  }
  __device__ static void fence_before_done() {}
  __device__ void tile_done(const TileInfo&) {}
  __device__ void begin_tile(const TileInfo&, int) {}
  __device__ void end_tile(const TileInfo& ti, int row) {
    if (trace_epi && row == 0) trace_epi[(ti.m0 / BM) * num_n + ti.n0 / bn] = ptx::globaltimer();
  }
  __device__ __forceinline__ void store(const TileInfo& ti, int row, int c, const uint32_t* r) {
    const int gm = ti.m0 + row;
    if (gm >= M) return;
    const int gn = ti.n0 + c;
    uint16_t* p = C + (size_t)gm * ldc + gn;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (gn + 8 * j + 8 <= N) {
        uint4 v;
        v.x = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 0]), __uint_as_float(r[8 * j + 1]));
        v.y = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 2]), __uint_as_float(r[8 * j + 3]));
        v.z = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 4]), __uint_as_float(r[8 * j + 5]));
        v.w = ptx::pack_bf16x2(__uint_as_float(r[8 * j + 6]), __uint_as_float(r[8 * j + 7]));
        ptx::st_v4(p + 8 * j, v);
      }
    }
  }
};

// Each CTA tells every rank that it is done with this call (it will not read any landing
// area of this parity again).
__device__ __forceinline__ void signal_cta_done(uint64_t* const* done_peer, int n, int r) {
  __syncthreads();
  if (threadIdx.x < (unsigned)n) ptx::red_release_sys_add(done_peer[threadIdx.x] + r, 1);
}

template <int BN>
__global__ void __launch_bounds__(cta_threads(kCommWarpsAG), 1)
    k_ag_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, AgSched sched,
              PlainStoreEpi epi, DoneTable done_peer, ErrorRecord* err, uint64_t timeout_ns) {
  uint64_t* tr = sched.trace ? sched.trace + 3 * (size_t)sched.num_tiles() + 2 * (size_t)sched.num_units() : nullptr;
  if (tr && threadIdx.x == 0) tr[2 * blockIdx.x] = ptx::globaltimer();
  gemm_core<BN>(&tmA, &tmB, sched, epi, err, timeout_ns, sched.r);
  signal_cta_done(done_peer.p, sched.n, sched.r);
  if (tr && threadIdx.x == 0) tr[2 * blockIdx.x + 1] = ptx::globaltimer();
}

template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::PairCfg<NH>::threads(kCommWarpsAG), 1)
    k_ag_gemm_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                   const __grid_constant__ CUtensorMap tmC, AgPairSched<NH> sched, PlainStoreEpi epi,
                   DoneTable done_peer, ErrorRecord* err, uint64_t timeout_ns) {
  epi.tmC = &tmC;
  pair::gemm_core_pair<NH>(&tmA, &tmB, sched, epi, err, timeout_ns, sched.r);
  signal_cta_done(done_peer.p, sched.n, sched.r);
}

// ------------------------------------------------------------------------------------------
// GEMM -> reduce-scatter
// ------------------------------------------------------------------------------------------
struct RsSched {
  static constexpr int kCommWarps = 0;
  int n, r, M, N, K, Mr, nbo, bn, num_n;
  __device__ int num_tiles() const { return n * nbo * num_n; }
  __device__ TileInfo tile(int t) const {
    // owner-major (owners r+1, r+2, ..., own rows last), grouped rasterisation per owner
    const int per = nbo * num_n;
    const int k = t / per;
    int b, nbk;
    raster(t - k * per, nbo, num_n, 16, b, nbk);
    const int o = (r + 1 + k) % n;
    TileInfo ti;
    ti.m0 = o * Mr + b * BM;
    ti.a_row = ti.m0;
    ti.n0 = nbk * bn;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = o;
    ti.aux2 = b;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo&, uint64_t, volatile int*, ErrorRecord*) const { return true; }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
  }
  __device__ void comm(int, int, volatile int*, ErrorRecord*, uint64_t) const {}
};

struct RsEpi {
  static constexpr bool kNeedsTileDone = true;
  static constexpr bool kPairHalves = false;
  int n, r, Mr, N, nbo, num_n, G;
  uint16_t* slots_peer[kMaxR];     // owner o's slot area [n][Mr][N] (this parity), mapped here
  const uint16_t* slots_local;     // my slot area
  uint64_t* arrivals_peer[kMaxR];  // owner o's counters [n][nbo]
  const uint64_t* arrivals;        // mine
  const uint64_t* done_local;      // [n]
  uint16_t* out;                   // [Mr][N] bf16
  long long ldo;
  uint64_t epoch;
  uint64_t timeout_ns;
  ErrorRecord* err;
  volatile int* abort_flag;
  int checked_owner;  // per-thread cache: owner whose previous-call readers are known done
  int skip;           // per-thread: current tile aborted

  __device__ static void fence_before_done() { ptx::fence_acq_rel_sys(); }
  __device__ void begin_tile(const TileInfo& ti, int) {
    skip = 0;
    const int o = ti.aux;
    if (o != r) {
      if (o != checked_owner && epoch > 2) {
        const uint64_t target = (epoch - 2) * (uint64_t)G;
        if (!wait_counter(done_local + o, target, timeout_ns, abort_flag)) {
          report_error(err, GICC_ETIMEDOUT, W_RS_FLAG, r, o, ptx::ld_relaxed_sys(done_local + o), target);
          skip = 1;
          return;
        }
      }
      checked_owner = o;
    } else {
      const uint64_t target = epoch * (uint64_t)num_n;
      for (int s = 0; s < n && !skip; ++s) {
        if (s == r) continue;
        const uint64_t* c = arrivals + (size_t)s * nbo + ti.aux2;
        if (!wait_counter(c, target, timeout_ns, abort_flag)) {
          report_error(err, GICC_ETIMEDOUT, W_RS_FLAG, r, s, ptx::ld_relaxed_sys(c), target);
          skip = 1;
        }
      }
    }
  }
  __device__ void end_tile(const TileInfo&, int) {}
  __device__ __forceinline__ void store(const TileInfo& ti, int row, int c, const uint32_t* acc) {
    if (skip) return;
    const int o = ti.aux;
    const int lrow = ti.m0 - o * Mr + row;  // row within the owner's block
    const int gn = ti.n0 + c;
    if (o != r) {
      uint16_t* p = slots_peer[o] + ((size_t)r * Mr + lrow) * N + gn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 v;
        v.x = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 0]), __uint_as_float(acc[8 * j + 1]));
        v.y = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 2]), __uint_as_float(acc[8 * j + 3]));
        v.z = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 4]), __uint_as_float(acc[8 * j + 5]));
        v.w = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 6]), __uint_as_float(acc[8 * j + 7]));
        ptx::st_v4_na(p + 8 * j, v);
      }
      return;
    }
    float f[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(acc[i]);
    for (int s = 0; s < n; ++s) {
      if (s == r) continue;
      const uint16_t* p = slots_local + ((size_t)s * Mr + lrow) * N + gn;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 v = ptx::ld_v4(p + 8 * j);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          f[8 * j + 2 * h] += ptx::bf16_lo(w[h]);
          f[8 * j + 2 * h + 1] += ptx::bf16_hi(w[h]);
        }
      }
    }
    uint16_t* q = out + (size_t)lrow * ldo + gn;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 v;
      v.x = ptx::pack_bf16x2(f[8 * j + 0], f[8 * j + 1]);
      v.y = ptx::pack_bf16x2(f[8 * j + 2], f[8 * j + 3]);
      v.z = ptx::pack_bf16x2(f[8 * j + 4], f[8 * j + 5]);
      v.w = ptx::pack_bf16x2(f[8 * j + 6], f[8 * j + 7]);
      ptx::st_v4(q + 8 * j, v);
    }
  }
  __device__ void tile_done(const TileInfo& ti) {
    if (ti.aux != r) ptx::red_release_sys_add(arrivals_peer[ti.aux] + (size_t)r * nbo + ti.aux2, 1);
  }
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_rs(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, RsSched sched, RsEpi epi,
              DoneTable done_peer, ErrorRecord* err, uint64_t timeout_ns) {
  epi.checked_owner = -1;
  epi.skip = 0;
  gemm_core<BN>(&tmA, &tmB, sched, epi, err, timeout_ns, sched.r);
  signal_cta_done(done_peer.p, sched.n, sched.r);
}

// ------------------------------------------------------------------------------------------
// GEMM -> reduce-scatter over NVLS
// ------------------------------------------------------------------------------------------
// Every rank writes its bf16 partial of the whole [M, N] output into its own staging
// buffer (local HBM, no NVLink traffic from the epilogue).  Tiles go band-major over the
// owners (band b of owner 0, 1, ..., n-1, then band b+1), the same order on every rank,
// so a band is finished everywhere at about the same time.  The CTA that completes a
// band's last tile tells the owner (one release add).  On the owner, `comm_ctas` CTAs run
// reduce warps: once all n ranks reported a band, multimem.ld_reduce reads the band
// through the staging buffer's multicast view -- the NVSwitch fetches the n partials and
// adds them (f32) -- and the bf16 sum is stored into the owner's output rows.  The
// reduction of band b overlaps the MMAs of the bands after it.
struct RsNvSched {
  static constexpr int kCommWarps = kCommWarpsAG;
  static constexpr bool kDynamic = true;
  int n, r, M, N, K, Mr, nbo, bn, num_n, Q, G, C;
  const uint16_t* staging_mc;      // multicast view of the staging buffers (this parity)
  const uint64_t* arrivals;        // mine: [nbo] ranks that finished my band b (monotonic)
  const uint64_t* done_local;      // [n] CTA-exit counts received from each rank
  uint16_t* out;                   // [Mr][N] bf16
  long long ldo;
  uint64_t epoch;
  unsigned long long* tile_counter;
  unsigned long long tile_base;
  // Diagnostics: %globaltimer stamps or null.  Layout (uint64), T = tiles (m-block major),
  // U = nbo * Q reduce units: [T] tile stored, [2U] unit start / end, [2G] CTA start / end.
  uint64_t* trace;
  // join != 0: reduce units are handed out by a global counter (base (epoch-1) * (U + grid):
  // every CTA takes one index past the end) and a CTA whose producer has taken its last
  // GEMM tile joins the reduction, so the bands that finish last are reduced by many SMs.
  int join;
  unsigned long long* unit_counter;
  unsigned long long unit_base;
  int group;  // m-blocks per raster group

  __device__ int num_tiles() const { return n * nbo * num_n; }
  __device__ int num_units() const { return nbo * Q; }
  __device__ volatile int* gemm_done_flag() const {
    __shared__ int gemm_done;  // set to 0 at kernel entry; 1 once the producer ran out of tiles
    return &gemm_done;
  }
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(tile_counter, 1ull) - tile_base;
    if (v >= (unsigned long long)num_tiles()) {
      if (join) *gemm_done_flag() = 1;
      return num_tiles();
    }
    return (int)v;
  }
  __device__ TileInfo tile(int t) const {
    int vm, nbk;
    raster(t, nbo * n, num_n, group, vm, nbk);
    const int b = vm / n, o = vm - b * n;
    TileInfo ti;
    ti.m0 = o * Mr + b * BM;
    ti.a_row = ti.m0;
    ti.n0 = nbk * bn;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = o;
    ti.aux2 = b;
    return ti;
  }
  // Before this CTA's first tile: every owner finished reading (ld_reduce) the staging
  // parity this call writes, i.e. finished call epoch-2.
  __device__ int* checked_flag() const {
    __shared__ int checked;  // set to 0 at kernel entry
    return &checked;
  }
  __device__ bool producer_wait(const TileInfo&, uint64_t timeout_ns, volatile int* abort_flag,
                                ErrorRecord* err) const {
    int* checked = checked_flag();
    if (*checked) return true;
    for (int d = 0; d < n && epoch > 2; ++d) {
      if (d == r) continue;
      const uint64_t target = (epoch - 2) * (uint64_t)G;
      if (!wait_counter(done_local + d, target, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_RS_FLAG, r, d, ptx::ld_relaxed_sys(done_local + d), target);
        return false;
      }
    }
    *checked = 1;
    return true;
  }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
  }
  // Reduce warps: unit u = b*Q + q covers rows [q*128/Q, (q+1)*128/Q) of my band b.
  __device__ void comm(int cw, int lane, volatile int* abort_flag, ErrorRecord* err, uint64_t timeout_ns) const {
    __shared__ int comm_stop;
    __shared__ int comm_unit;
    const int tid = cw * 32 + lane;
    constexpr int kT = kCommWarps * 32;
    if (!join && (int)blockIdx.x >= C) return;
    const int U = nbo * Q;
    const int rows = BM / Q;
    const int vpr = N / 8;  // 16-byte vectors per row
    const size_t nv = (size_t)rows * vpr;
    if (join && (int)blockIdx.x >= C) {
      // not a dedicated reducer: join once this CTA's producer has taken its last tile
      if (tid == 0) {
        const uint64_t t0 = ptx::globaltimer();
        while (!*gemm_done_flag() && !*abort_flag) {
          __nanosleep(1000);
          if (ptx::globaltimer() - t0 > timeout_ns) break;  // the producer's own waits report
        }
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
    }
    for (int it = 0;; ++it) {
      if (tid == 0) {
        int u;
        if (join) {
          const unsigned long long v = atomicAdd(unit_counter, 1ull) - unit_base;
          u = v < (unsigned long long)U ? (int)v : U;
        } else {
          u = (int)blockIdx.x + it * C;
          if (u > U) u = U;
        }
        int stop = *abort_flag || u >= U;
        if (!stop) {
          const uint64_t target = epoch * (uint64_t)n;
          const int b = u / Q;
          if (!wait_counter(arrivals + b, target, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_RS_FLAG, r, -1, ptx::ld_relaxed_sys(arrivals + b), target);
            *abort_flag = 1;
            stop = 1;
          }
        }
        comm_unit = u;
        comm_stop = stop;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (comm_stop) break;
      const int u = comm_unit;
      const int b = u / Q, q = u - (u / Q) * Q;
      uint64_t* tr = trace ? trace + (size_t)num_tiles() + 2 * (size_t)u : nullptr;
      if (tr && tid == 0) tr[0] = ptx::globaltimer();
      const int lrow0 = b * BM + q * rows;  // first row within my block
      const uint4* src = reinterpret_cast<const uint4*>(staging_mc + ((size_t)r * Mr + lrow0) * N);
      size_t i = tid;
      for (; i + 15 * kT < nv; i += 16 * kT) {
        uint4 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = ptx::multimem_ld_reduce_bf16x8(src + i + j * kT);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const size_t e = i + j * kT;
          const int rr = (int)(e / vpr), cc = (int)(e - (size_t)rr * vpr);
          ptx::st_v4(out + (size_t)(lrow0 + rr) * ldo + (size_t)cc * 8, v[j]);
        }
      }
      for (; i < nv; i += kT) {
        const int rr = (int)(i / vpr), cc = (int)(i - (size_t)rr * vpr);
        ptx::st_v4(out + (size_t)(lrow0 + rr) * ldo + (size_t)cc * 8, ptx::multimem_ld_reduce_bf16x8(src + i));
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (tr && tid == 0) tr[1] = ptx::globaltimer();
    }
  }
};

struct RsNvEpi {
  static constexpr bool kNeedsTileDone = true;
  static constexpr bool kPairHalves = false;
  int N, nbo, num_n;
  uint16_t* staging;                   // mine [M][N] (this parity)
  unsigned long long* band_tiles;      // mine [n][nbo]: tiles of band (o, b) finished here (monotonic)
  uint64_t* arrivals_peer[kMaxR];      // owner o's [nbo] counters, mapped here
  uint64_t epoch;
  uint64_t* trace_epi;                 // diagnostics: [tile] stamp when stored, or null
  __device__ static void fence_before_done() { ptx::fence_acq_rel_sys(); }
  __device__ void begin_tile(const TileInfo&, int) {}
  __device__ void end_tile(const TileInfo& ti, int row) {
    if (trace_epi && row == 0) trace_epi[(ti.m0 / BM) * num_n + ti.n0 / 256] = ptx::globaltimer();
  }
  __device__ __forceinline__ void store(const TileInfo& ti, int row, int c, const uint32_t* acc) {
    uint16_t* p = staging + (size_t)(ti.m0 + row) * N + ti.n0 + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 v;
      v.x = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 0]), __uint_as_float(acc[8 * j + 1]));
      v.y = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 2]), __uint_as_float(acc[8 * j + 3]));
      v.z = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 4]), __uint_as_float(acc[8 * j + 5]));
      v.w = ptx::pack_bf16x2(__uint_as_float(acc[8 * j + 6]), __uint_as_float(acc[8 * j + 7]));
      ptx::st_v4(p + 8 * j, v);
    }
  }
  // Last epilogue warp of a tile: count it; the CTA that completes the band tells the owner.
  __device__ void tile_done(const TileInfo& ti) {
    unsigned long long* c = band_tiles + (size_t)ti.aux * nbo + ti.aux2;
    const unsigned long long old = ptx::atom_add_acq_rel_sys(reinterpret_cast<uint64_t*>(c), 1);
    if (old + 1 == epoch * (unsigned long long)num_n) ptx::red_release_sys_add(arrivals_peer[ti.aux] + ti.aux2, 1);
  }
};

// The NVLS reduce-scatter GEMM on CTA pairs: pair tiles of 256 rows (two 128-row bands of
// one owner) x NH*256 columns in the same band-major order; each CTA publishes its own band.
// The join option is not available here (only the leader's producer sees the tile counter).
template <int NH>
struct RsNvPairSched : RsNvSched {
  int nbo2;  // 256-row pair bands per owner
  __device__ int num_tiles() const { return n * nbo2 * num_n; }
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(tile_counter, 1ull) - tile_base;
    return v < (unsigned long long)num_tiles() ? (int)v : num_tiles();
  }
  __device__ TileInfo tile(int t) const {
    int vm, nbk;
    raster(t, nbo2 * n, num_n, group, vm, nbk);
    const int b = vm / n, o = vm - b * n;
    TileInfo ti;
    ti.m0 = o * Mr + b * 2 * BM;
    ti.a_row = ti.m0;
    ti.n0 = nbk * NH * 256;
    ti.b_row = ti.n0;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = o;
    ti.aux2 = 2 * b;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo& ti, int, uint64_t timeout_ns, volatile int* abort_flag,
                                ErrorRecord* err) const {
    return RsNvSched::producer_wait(ti, timeout_ns, abort_flag, err);
  }
};

// RsNvEpi for pair tiles: the band that a CTA publishes follows from its first row.
struct RsNvPairEpi : RsNvEpi {
  int Mr;
  __device__ void end_tile(const TileInfo&, int) {}
  __device__ void tile_done(const TileInfo& ti) {
    TileInfo t = ti;
    t.aux2 = (ti.m0 - ti.aux * Mr) / BM;
    RsNvEpi::tile_done(t);
  }
};

template <int NH>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(pair::PairCfg<NH>::threads(kCommWarpsAG), 1)
    k_gemm_rs_nvls_pair(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        RsNvPairSched<NH> sched, RsNvPairEpi epi, DoneTable done_peer, ErrorRecord* err,
                        uint64_t timeout_ns) {
  if (threadIdx.x == 0) {  // ordered by the core's set-up barrier
    *sched.checked_flag() = 0;
    *sched.gemm_done_flag() = 0;
  }
  pair::gemm_core_pair<NH>(&tmA, &tmB, sched, epi, err, timeout_ns, sched.r);
  signal_cta_done(done_peer.p, sched.n, sched.r);
}

template <int BN>
__global__ void __launch_bounds__(cta_threads(kCommWarpsAG), 1)
    k_gemm_rs_nvls(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, RsNvSched sched,
                   RsNvEpi epi, DoneTable done_peer, ErrorRecord* err, uint64_t timeout_ns) {
  if (threadIdx.x == 0) {  // ordered by the core's set-up barrier
    *sched.checked_flag() = 0;
    *sched.gemm_done_flag() = 0;
  }
  uint64_t* tr = sched.trace ? sched.trace + (size_t)sched.num_tiles() + 2 * (size_t)sched.num_units() : nullptr;
  if (tr && threadIdx.x == 0) tr[2 * blockIdx.x] = ptx::globaltimer();
  gemm_core<BN>(&tmA, &tmB, sched, epi, err, timeout_ns, sched.r);
  signal_cta_done(done_peer.p, sched.n, sched.r);
  if (tr && threadIdx.x == 0) tr[2 * blockIdx.x + 1] = ptx::globaltimer();
}

}  // namespace
}  // namespace gemm

namespace ops {

namespace {
// The CTA-pair variant of ag_gemm: same schedule fields, pair tiles, grid of whole pairs.
template <int NH>
void launch_ag_pair(const AgGemmArgs& a, const gemm::AgSched& base, const gemm::PlainStoreEpi& e0,
                    const gemm::DoneTable& dt, int G, cudaStream_t s) {
  using namespace gemm;
  using Cf = pair::PairCfg<NH>;
  const int Ms = a.M / a.n;
  if (Ms % (2 * BM) || a.Ns % (NH * 256) || a.trace)
    throw std::runtime_error("gicc::ag_gemm (pairs): need M/ranks % 256 == 0, N/ranks % (pair*256) == 0, no trace");
  const int Gp = G & ~1;  // whole CTA pairs
  const CUtensorMap tA = make_tmap_2d(a.a_full[a.r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.K, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.Ns, a.K, a.ldb, pair::BN2 / 2, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  AgPairSched<NH> sc;
  static_cast<AgSched&>(sc) = base;
  sc.G = Gp;
  sc.C = a.comm_ctas > 0 && a.comm_ctas < Gp ? a.comm_ctas : Gp;
  sc.nb2 = Ms / (2 * BM);
  sc.num_n = a.Ns / (NH * 256);
  sc.bn = NH * 256;
  // every leader takes one index past the end of each call
  sc.tile_base = (unsigned long long)(a.epoch - 1) * (unsigned long long)(a.n * sc.nb2 * sc.num_n + Gp / 2);
  PlainStoreEpi e = e0;
  e.trace_epi = nullptr;
  // C in 32 x 32 boxes through shared memory and TMA (whole lines to L2), as the plain GEMM
  e.use_tma = ops::gemm_tuning().pair_tma_store != 0 ? 1 : 0;
  const CUtensorMap tC = e.use_tma ? make_tmap_2d(a.C, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.Ns, a.ldc, 32, 32,
                                                  CU_TENSOR_MAP_SWIZZLE_NONE)
                                   : tA;  // unused
  static bool attr[2][64] = {};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr[NH - 1][dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_ag_gemm_pair<NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cf::kSmemBytesStaged));
    attr[NH - 1][dev] = true;
  }
  k_ag_gemm_pair<NH><<<Gp, Cf::threads(kCommWarpsAG), Cf::kSmemBytesStaged, s>>>(
      tA, tB, tC, sc, e, dt, device_error_record(), a.timeout_ns ? a.timeout_ns : default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}
}  // namespace

namespace {
// The CTA-pair variant of the NVLS reduce-scatter GEMM.
template <int NH>
void launch_rs_pair(const GemmRsArgs& a, const gemm::RsNvSched& base, const gemm::RsNvEpi& e0,
                    const gemm::DoneTable& dt, int G, cudaStream_t s) {
  using namespace gemm;
  using Cf = pair::PairCfg<NH>;
  const int Mr = a.M / a.n;
  if (Mr % (2 * BM) || a.N % (NH * 256) || a.trace || a.join_reduce)
    throw std::runtime_error("gicc::gemm_rs (pairs): need M/ranks % 256 == 0, N % (pair*256) == 0, no join, no trace");
  const int Gp = G & ~1;
  const CUtensorMap tA = make_tmap_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, pair::BN2 / 2, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  RsNvPairSched<NH> sc;
  static_cast<RsNvSched&>(sc) = base;
  sc.G = Gp;
  sc.C = a.comm_ctas > 0 && a.comm_ctas < Gp ? a.comm_ctas : 16;
  sc.nbo2 = Mr / (2 * BM);
  sc.num_n = a.N / (NH * 256);
  sc.bn = NH * 256;
  sc.tile_base = (unsigned long long)(a.epoch - 1) * (unsigned long long)(a.n * sc.nbo2 * sc.num_n + Gp / 2);
  sc.group = a.raster_group > 0 ? a.raster_group : 8;
  RsNvPairEpi e;
  static_cast<RsNvEpi&>(e) = e0;
  e.trace_epi = nullptr;
  e.num_n = sc.num_n;
  e.Mr = Mr;
  static bool attr[2][64] = {};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr[NH - 1][dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_rs_nvls_pair<NH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   Cf::kSmemBytes));
    attr[NH - 1][dev] = true;
  }
  k_gemm_rs_nvls_pair<NH><<<Gp, Cf::threads(kCommWarpsAG), Cf::kSmemBytes, s>>>(
      tA, tB, sc, e, dt, device_error_record(), a.timeout_ns ? a.timeout_ns : default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}
}  // namespace

void ag_gemm(const AgGemmArgs& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::ag_gemm");
  using namespace gemm;
  constexpr int BN_ = 256;
  if (a.n < 2 || a.n > kMaxR) throw std::runtime_error("gicc::ag_gemm: 2..16 ranks");
  if (a.M % (a.n * BM) || a.Ns % BN_ || a.K % BK)
    throw std::runtime_error("gicc::ag_gemm: need M % (ranks*128) == 0, N/ranks % 256 == 0, K % 64 == 0");
  if ((reinterpret_cast<uintptr_t>(a.C) & 15) || (a.ldc % 8) || a.ldc < a.Ns)
    throw std::runtime_error("gicc::ag_gemm: C needs a 16-byte aligned base and ldc % 8 == 0, ldc >= N/ranks");
  const int Ms = a.M / a.n, nb = Ms / BM;
  const int Q = a.units_per_band > 0 ? a.units_per_band : 4;
  if (((long long)BM * a.K * 2 / 16) % Q) throw std::runtime_error("gicc::ag_gemm: units_per_band must divide a band's 16-byte vectors");
  const CUtensorMap tA = make_tmap_2d(a.a_full[a.r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.K, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.Ns, a.K, a.ldb, BN_, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const int G = a.grid > 0 ? a.grid : num_sms();
  // One CTA per SM (the shared-memory ring allows no second); the CTAs wait on one another's
  // tiles and arrivals, so all of them must be resident at once.
  if (G > num_sms()) throw std::runtime_error("gicc: a persistent distributed GEMM needs grid <= number of SMs");
  AgSched sc{};
  sc.n = a.n;
  sc.r = a.r;
  sc.M = a.M;
  sc.Ns = a.Ns;
  sc.K = a.K;
  sc.Ms = Ms;
  sc.nb = nb;
  sc.bn = BN_;
  sc.num_n = a.Ns / BN_;
  sc.Q = Q;
  sc.G = G;
  sc.C = a.comm_ctas > 0 && a.comm_ctas < G ? a.comm_ctas : G;
  sc.a_local = static_cast<const uint16_t*>(a.a_full[a.r]);
  for (int i = 0; i < a.n; ++i) {
    sc.a_peer[i] = static_cast<uint16_t*>(a.a_full[i]);
    sc.arrivals_peer[i] = a.arrivals[i];
  }
  sc.arrivals = a.arrivals[a.r];
  sc.done_local = a.done[a.r];
  sc.epoch = a.epoch;
  sc.trace = a.trace;
  sc.diag = a.diag;
  if (!a.tile_counter) throw std::runtime_error("gicc::ag_gemm: tile_counter (one zeroed local word) is required");
  sc.tile_counter = reinterpret_cast<unsigned long long*>(a.tile_counter);
  sc.tile_base = (unsigned long long)(a.epoch - 1) * (unsigned long long)(a.n * nb * (a.Ns / BN_) + G);
  sc.a_mc = static_cast<uint16_t*>(a.a_mc);
  sc.arrivals_mc = a.arrivals_mc;
  if ((sc.a_mc == nullptr) != (sc.arrivals_mc == nullptr))
    throw std::runtime_error("gicc::ag_gemm: NVLS mode needs both a_mc and arrivals_mc");
  PlainStoreEpi e{static_cast<uint16_t*>(a.C), a.ldc, a.M, a.Ns, a.trace ? a.trace + 2 * (size_t)a.n * nb * (a.Ns / BN_) : nullptr,
                  a.Ns / BN_, BN_};
  DoneTable dt{};
  for (int i = 0; i < a.n; ++i) dt.p[i] = a.done[i];
  if (a.pair) {
    if (a.pair == 1) launch_ag_pair<1>(a, sc, e, dt, G, s);
    else launch_ag_pair<2>(a, sc, e, dt, G, s);
    return;
  }
  constexpr uint32_t smem = Cfg<BN_>::kSmemBytes;
  static bool attr[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_ag_gemm<BN_>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  k_ag_gemm<BN_><<<G, cta_threads(kCommWarpsAG), smem, s>>>(tA, tB, sc, e, dt, device_error_record(),
                                                             a.timeout_ns ? a.timeout_ns : default_timeout_ns());
  GICC_CUDA(cudaGetLastError());
}

void ag_transfer_ce(const AgCeArgs& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::ag_transfer_ce");
  using namespace gemm;
  if (a.n < 2 || a.n > kMaxR || a.M % (a.n * BM)) throw std::runtime_error("gicc::ag_transfer_ce: bad shape");
  const DriverApi& d = driver();
  if (!d.StreamWriteValue64) throw std::runtime_error("gicc::ag_transfer_ce: stream memory operations unavailable");
  const uint64_t timeout_ns = a.timeout_ns ? a.timeout_ns : default_timeout_ns();
  const int Ms = a.M / a.n, nb = Ms / BM;
  const int chunks = a.chunks > 0 && a.chunks <= nb ? a.chunks : 1;
  const size_t row_bytes = (size_t)a.K * 2;
  const uint64_t target = a.epoch * (uint64_t)(a.units_per_band > 0 ? a.units_per_band : 4);
  for (int k = 1; k < a.n; ++k) {
    const int dst = (a.r - k + a.n) % a.n;
    // dst finished the call that last used this parity (its CTAs' exit counts).  The wait
    // is a one-thread kernel bounded by timeout_ns: on timeout it records GICC_ETIMEDOUT in
    // the device error record (read by the host after the call) and the stream goes on.
    if (a.epoch > 2)
      wait_signal(a.done_local + dst, proto::CMP_GE, (a.epoch - 2) * (uint64_t)a.grid, timeout_ns, nullptr, s);
    for (int c = 0; c < chunks; ++c) {
      const int b0 = nb * c / chunks, b1 = nb * (c + 1) / chunks;
      const size_t off = ((size_t)a.r * Ms + (size_t)b0 * BM) * row_bytes;
      GICC_CUDA(cudaMemcpyAsync(static_cast<char*>(a.a_full[dst]) + off, static_cast<const char*>(a.a_full[a.r]) + off,
                                (size_t)(b1 - b0) * BM * row_bytes, cudaMemcpyDeviceToDevice, s));
      for (int b = b0; b < b1; ++b)  // default write: ordered after the copy's stores
        GICC_DRV(d.StreamWriteValue64(s, reinterpret_cast<CUdeviceptr>(a.arrivals[dst] + (size_t)a.r * nb + b), target,
                                      CU_STREAM_WRITE_VALUE_DEFAULT));
    }
  }
}

void gemm_rs(const GemmRsArgs& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::gemm_rs");
  using namespace gemm;
  constexpr int BN_ = 256;
  if (a.n < 2 || a.n > kMaxR) throw std::runtime_error("gicc::gemm_rs: 2..16 ranks");
  if (a.M % (a.n * BM) || a.N % BN_ || a.K % BK)
    throw std::runtime_error("gicc::gemm_rs: need M % (ranks*128) == 0, N % 256 == 0, K/ranks % 64 == 0");
  const int Mr = a.M / a.n;
  const CUtensorMap tA = make_tmap_2d(a.A, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.M, a.K, a.lda, BM, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB = make_tmap_2d(a.B, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.N, a.K, a.ldb, BN_, BK,
                                      CU_TENSOR_MAP_SWIZZLE_128B);
  const int G = a.grid > 0 ? a.grid : num_sms();
  // One CTA per SM (the shared-memory ring allows no second); the CTAs wait on one another's
  // tiles and arrivals, so all of them must be resident at once.
  if (G > num_sms()) throw std::runtime_error("gicc: a persistent distributed GEMM needs grid <= number of SMs");
  if (a.staging_mc) {
    const int Q = a.units_per_band > 0 ? a.units_per_band : 4;
    if (BM % Q || !a.band_tiles || !a.tile_counter || !a.slots[a.r])
      throw std::runtime_error("gicc::gemm_rs (NVLS): units_per_band | 128, band_tiles, tile_counter, staging required");
    RsNvSched sc{};
    sc.n = a.n; sc.r = a.r; sc.M = a.M; sc.N = a.N; sc.K = a.K; sc.Mr = Mr; sc.nbo = Mr / BM; sc.bn = BN_;
    sc.num_n = a.N / BN_; sc.Q = Q; sc.G = G;
    sc.C = a.comm_ctas > 0 && a.comm_ctas < G ? a.comm_ctas : 16;
    sc.staging_mc = static_cast<const uint16_t*>(a.staging_mc);
    sc.arrivals = a.arrivals[a.r];
    sc.done_local = a.done[a.r];
    sc.out = static_cast<uint16_t*>(a.out);
    sc.ldo = a.ldo;
    sc.epoch = a.epoch;
    sc.tile_counter = reinterpret_cast<unsigned long long*>(a.tile_counter);
    sc.tile_base = (unsigned long long)(a.epoch - 1) * (unsigned long long)(a.n * sc.nbo * sc.num_n + G);
    sc.trace = a.trace;
    sc.join = a.join_reduce ? 1 : 0;
    if (sc.join && !a.unit_counter) throw std::runtime_error("gicc::gemm_rs (NVLS): join_reduce needs unit_counter");
    sc.unit_counter = reinterpret_cast<unsigned long long*>(a.unit_counter);
    sc.unit_base = (unsigned long long)(a.epoch - 1) * (unsigned long long)(sc.nbo * Q + G);
    sc.group = a.raster_group > 0 ? a.raster_group : 16;
    RsNvEpi e{};
    e.trace_epi = a.trace;  // first T words
    e.N = a.N; e.nbo = sc.nbo; e.num_n = sc.num_n;
    e.staging = static_cast<uint16_t*>(a.slots[a.r]);
    e.band_tiles = reinterpret_cast<unsigned long long*>(a.band_tiles);
    for (int i = 0; i < a.n; ++i) e.arrivals_peer[i] = a.arrivals[i];
    e.epoch = a.epoch;
    DoneTable dt{};
    for (int i = 0; i < a.n; ++i) dt.p[i] = a.done[i];
    if (a.pair) {
      if (a.pair == 1) launch_rs_pair<1>(a, sc, e, dt, G, s);
      else launch_rs_pair<2>(a, sc, e, dt, G, s);
      return;
    }
    constexpr uint32_t smem = Cfg<BN_>::kSmemBytes;
    static bool attr_nv[64] = {false};
    int dev = 0;
    GICC_CUDA(cudaGetDevice(&dev));
    if (!attr_nv[dev]) {
      GICC_CUDA(cudaFuncSetAttribute(k_gemm_rs_nvls<BN_>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr_nv[dev] = true;
    }
    k_gemm_rs_nvls<BN_><<<G, cta_threads(kCommWarpsAG), smem, s>>>(tA, tB, sc, e, dt, device_error_record(),
                                                                   a.timeout_ns ? a.timeout_ns : default_timeout_ns());
    GICC_CUDA(cudaGetLastError());
    return;
  }
  RsSched sc{a.n, a.r, a.M, a.N, a.K, Mr, Mr / BM, BN_, a.N / BN_};
  RsEpi e{};
  e.n = a.n;
  e.r = a.r;
  e.Mr = Mr;
  e.N = a.N;
  e.nbo = Mr / BM;
  e.num_n = a.N / BN_;
  e.G = G;
  for (int i = 0; i < a.n; ++i) {
    e.slots_peer[i] = static_cast<uint16_t*>(a.slots[i]);
    e.arrivals_peer[i] = a.arrivals[i];
  }
  e.slots_local = static_cast<const uint16_t*>(a.slots[a.r]);
  e.arrivals = a.arrivals[a.r];
  e.done_local = a.done[a.r];
  e.out = static_cast<uint16_t*>(a.out);
  e.ldo = a.ldo;
  e.epoch = a.epoch;
  e.timeout_ns = a.timeout_ns ? a.timeout_ns : default_timeout_ns();
  e.err = device_error_record();
  e.abort_flag = nullptr;
  DoneTable dt{};
  for (int i = 0; i < a.n; ++i) dt.p[i] = a.done[i];
  constexpr uint32_t smem = Cfg<BN_>::kSmemBytes;
  static bool attr[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(k_gemm_rs<BN_>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  k_gemm_rs<BN_><<<G, kThreads, smem, s>>>(tA, tB, sc, e, dt, e.err, e.timeout_ns);
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
