// moe.cu -- expert-parallel MoE layer: routing, dispatch all-to-all fused into the first
// grouped GEMM, SwiGLU in its epilogue, and the gate-weighted combine all-to-all fused into
// the second grouped GEMM's epilogue.  None of this exists in the reference; it is an
// expert-parallel layer (e.g. 4096 tokens per GPU, hidden 7168, 256 experts, top-8) built on
// the same NVLink primitives (peer stores + release/acquire counters, every wait bounded).
//
// Per call (epoch e), on every rank r of n, with El = E/n local experts:
//  1. k_route      softmax over the E router logits of each token, top-k, per-expert counts.
//  2. k_plan       one CTA: pushes its counts row into every rank's count table, waits for
//                  everybody's row, then derives (a) where its rows land on each owner
//                  (sources ordered by rank inside an expert segment, segments padded to
//                  128 rows), (b) the local experts' row ranges and m-block prefix for the
//                  grouped GEMMs, (c) the send order (expert-major, so every owner gets
//                  expert 0 from all sources first).
//  3. k_sort       places every (token, k) pair into the send list.
//  4. k_moe_gemm1  4 communication warps per CTA copy the token rows (16-byte NVLink
//                  stores) into the owners' receive buffers, with (source, slot, gate) meta,
//                  and release-add a per-(source, expert) row counter; the TMA producer
//                  waits on the counters of an expert before its first tile; tcgen05 MMAs
//                  compute [gate | up] = X W1^T tile-wise and the epilogue writes
//                  silu(gate) * up.
//  5. k_moe_gemm2  Y = H W2^T; the epilogue scales each row by its gate and stores it into
//                  the source rank's combine buffer (slot t*k+j), then release-adds the
//                  per-source arrival count (rows x column tiles).
//  6. k_combine    the source waits for all its rows and sums the k weighted rows per token.
//
// Options (MoeArgs): dispatch_ctas confines step 4's NVLink stores to a few CTAs and lets
// the first GEMM take tiles dynamically; combine_ctas makes step 5 stage its rows locally
// (k_moe_gemm2_staged) and queue each finished tile for a few pushing CTAs; comm_only runs
// steps 1-3, then k_moe_dispatch (step 4's dispatch alone), k_moe_return (each received row
// back to its source, scaled by its gate) and step 6 -- the all-to-all round trip with
// identity experts.
#include <cuda_runtime.h>

#include <cstring>

#include "gicc/device/comm.cuh"
#include "gicc/device/gemm_core.cuh"
#include "gicc/config.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace moe {
namespace {

using namespace gicc::gemm;
constexpr int kMaxR = 8;
constexpr int kMaxLocalExperts = 256;
constexpr int kCommWarps = 4;

struct Ptrs8 {
  void* p[kMaxR];
};
struct Words8 {
  uint64_t* p[kMaxR];
};

__device__ __forceinline__ bool wait_ge(const uint64_t* p, uint64_t target, uint64_t timeout_ns,
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

// ---------------------------------------------------------------------------------------
// 1. routing: one warp per token (E <= 1024, E % 32 == 0), k <= 8
// ---------------------------------------------------------------------------------------
__global__ void k_route(const float* logits, int T, int E, int topk, int* topk_idx, float* topk_w, int* counts) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= T) return;
  const float* l = logits + (size_t)warp * E;
  constexpr int kMaxPer = 32;
  float v[kMaxPer];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i) {
    v[i] = (i < per && i * 32 + lane < E) ? l[i * 32 + lane] : -INFINITY;
    mx = fmaxf(mx, v[i]);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < kMaxPer; ++i)
    if (i < per && i * 32 + lane < E) sum += expf(v[i] - mx);
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  for (int k = 0; k < topk; ++k) {
    // lane-local best (lowest index on ties), then warp argmax
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < kMaxPer; ++i)
      if (i < per && v[i] > bv) {
        bv = v[i];
        bi = i * 32 + lane;
      }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((bi & 31) == lane) v[bi >> 5] = -INFINITY;  // remove the winner
    if (lane == 0) {
      topk_idx[(size_t)warp * topk + k] = bi;
      topk_w[(size_t)warp * topk + k] = expf(bv - mx) / sum;
      atomicAdd(&counts[bi], 1);
    }
  }
}

// ---------------------------------------------------------------------------------------
// 2. plan: one CTA of 256 threads
// ---------------------------------------------------------------------------------------
struct PlanArgs {
  int n, r, E, El;
  const int* counts;        // [E] this rank's pair counts per global expert
  Ptrs8 count_tab;          // each rank's [n][E] int32 table (peer views)
  Words8 flags;             // each rank's [n] flag words (peer views)
  uint64_t epoch;
  int* dest_row_base;       // [E] out: first row of my rows for expert g on its owner
  int* key_base;            // [El*n + 1] out: send-list offsets per key
  int* key_cursor;          // [El*n] out: zeroed
  int* expert_base;         // [El] out
  int* expert_rows;         // [El] out
  int* mblk_prefix;         // [El+1] out
  uint64_t* cum_rows;       // [n][El] in/out: cumulative rows expected from each source
  uint64_t* cum_pairs;      // [1] in/out: cumulative pairs this rank sent (for combine)
  int pairs;                // T * topk
  ErrorRecord* err;
  uint64_t timeout_ns;
};

__device__ __forceinline__ int pad128(int x) { return (x + 127) & ~127; }

__global__ void __launch_bounds__(256) k_plan(PlanArgs a) {
  const int t = threadIdx.x;
  const int n = a.n, r = a.r, E = a.E, El = a.El;
  // (1) my counts row -> every rank's table, then a release flag
  for (int i = t; i < E; i += blockDim.x) {
    const int c = a.counts[i];
    for (int d = 0; d < n; ++d) reinterpret_cast<int*>(a.count_tab.p[d])[(size_t)r * E + i] = c;
  }
  ptx::fence_acq_rel_sys();
  __syncthreads();
  if (t < n) ptx::st_release_sys(a.flags.p[t] + r, a.epoch);
  // (2) wait for every rank's row
  __shared__ int ok;
  if (t == 0) ok = 1;
  __syncthreads();
  if (t < n) {
    if (!wait_ge(a.flags.p[r] + t, a.epoch, a.timeout_ns, nullptr)) {
      report_error(a.err, GICC_ETIMEDOUT, W_MOE_COUNT, r, t, ptx::ld_relaxed_sys(a.flags.p[r] + t), a.epoch);
      ok = 0;
    }
  }
  __syncthreads();
  if (!ok) return;
  const int* C = reinterpret_cast<const int*>(a.count_tab.p[r]);  // [n][E], complete now
  // (3) per global expert g: where my rows start on its owner.  Segment sizes go to shared
  // memory first; one thread per owner scans its segment list (no dependent global loads).
  __shared__ int seg[1024];  // E <= 1024: padded rows of expert g on its owner, then its base
  for (int g = t; g < E; g += blockDim.x) {
    int rows = 0;
    for (int s = 0; s < n; ++s) rows += C[(size_t)s * E + g];
    seg[g] = pad128(rows);
  }
  __syncthreads();
  if (t < n) {
    int base = 0;
    for (int e = 0; e < El; ++e) {
      const int sz = seg[t * El + e];
      seg[t * El + e] = base;
      base += sz;
    }
  }
  __syncthreads();
  for (int g = t; g < E; g += blockDim.x) {
    int base = seg[g];
    for (int s = 0; s < r; ++s) base += C[(size_t)s * E + g];
    a.dest_row_base[g] = base;
  }
  // (4) my local experts
  __shared__ int rows_s[kMaxLocalExperts];
  for (int e = t; e < El; e += blockDim.x) {
    int rows = 0;
    for (int s = 0; s < n; ++s) {
      const int c = C[(size_t)s * E + r * El + e];
      rows += c;
      a.cum_rows[(size_t)s * El + e] += (uint64_t)c;
    }
    rows_s[e] = rows;
    a.expert_rows[e] = rows;
  }
  __shared__ int cnt_s[1024];  // this rank's pair counts per global expert (E <= 1024)
  for (int g = t; g < E; g += blockDim.x) cnt_s[g] = a.counts[g];
  __syncthreads();
  // (5) prefix sums by warp 0 (each lane scans a contiguous range from shared memory, then
  // one shuffle scan over the lanes' totals): expert bases / m-block prefix over my experts,
  // and the send-list offsets over keys e * n + j, j = (r - d) mod n (local first, then
  // r-1, r-2, ...).
  if (t < 32) {
    const unsigned full = 0xffffffffu;
    auto excl_scan = [&](int v, int* total) {
      int incl = v;
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(full, incl, o);
        if (t >= o) incl += u;
      }
      *total = __shfl_sync(full, incl, 31);
      return incl - v;
    };
    const int pe = (El + 31) / 32, e0 = min(t * pe, El), e1 = min(e0 + pe, El);
    int sum = 0, total = 0;
    for (int e = e0; e < e1; ++e) sum += pad128(rows_s[e]);
    int base = excl_scan(sum, &total);
    for (int e = e0; e < e1; ++e) {
      a.expert_base[e] = base;
      a.mblk_prefix[e] = base / 128;  // every segment is a multiple of 128 rows
      base += pad128(rows_s[e]);
    }
    if (t == 0) a.mblk_prefix[El] = total / 128;
    const int K = El * n, pk = (K + 31) / 32, k0 = min(t * pk, K), k1 = min(k0 + pk, K);
    auto key_count = [&](int key) {
      const int e = key / n, j = key - e * n, d = (r - j + n) % n;
      return cnt_s[d * El + e];
    };
    sum = 0;
    for (int k = k0; k < k1; ++k) sum += key_count(k);
    int off = excl_scan(sum, &total);
    for (int k = k0; k < k1; ++k) {
      a.key_base[k] = off;
      off += key_count(k);
    }
    if (t == 0) {
      a.key_base[K] = total;
      *a.cum_pairs += (uint64_t)a.pairs;
    }
  }
  for (int i = t; i < El * n; i += blockDim.x) a.key_cursor[i] = 0;
}

// ---------------------------------------------------------------------------------------
// 3. sort pairs into the send list
// ---------------------------------------------------------------------------------------
__global__ void k_sort(const int* topk_idx, int pairs, int n, int r, int El, const int* key_base, int* key_cursor,
                       const int* dest_row_base, int* send_pair, int* send_row) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= pairs) return;
  const int g = topk_idx[i];
  const int d = g / El, e = g % El;
  const int key = e * n + (r - d + n) % n;
  const int k = atomicAdd(&key_cursor[key], 1);
  const int pos = key_base[key] + k;
  send_pair[pos] = i;
  send_row[pos] = dest_row_base[g] + k;
}

// ---------------------------------------------------------------------------------------
// 4. grouped GEMM 1: dispatch (comm warps) + X W1^T + SwiGLU
// ---------------------------------------------------------------------------------------
// Dyn = true: only C CTAs dispatch, and tiles come from a global counter so those CTAs take
// fewer tiles.  The tile count changes from call to call (it follows the routing), so the
// counter is one of a pair: call e counts on tile_ctr[e & 1] and zeroes the other one, which
// call e+1 uses.
template <bool Dyn>
struct G1SchedT {
  static constexpr int kCommWarps = moe::kCommWarps;
  static constexpr bool kDynamic = Dyn;
  int n, r, El, H, I2, num_n;  // H = hidden (K), I2 = 2*inter (N), num_n = I2 / 256
  int topk, G;
  int C;                       // CTAs that dispatch (G when not Dyn)
  unsigned long long* tile_ctr;  // Dyn: this call's counter
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(tile_ctr, 1ull);
    return v < (unsigned long long)num_tiles() ? (int)v : num_tiles();
  }
  const int* mblk_prefix;      // [El+1]
  const int* expert_base;      // [El]
  const uint64_t* arrivals;    // my [n][El] row counters
  const uint64_t* cum_rows;    // [n][El] targets
  // dispatch
  int npairs;
  const int* send_pair;        // [npairs] pair id (t*topk + j)
  const int* send_row;         // [npairs] row on the owner
  const int* topk_idx;
  const float* topk_w;
  const uint16_t* x;           // [T][H] my tokens
  Ptrs8 recv;                  // each rank's receive buffer [cap][H]
  Ptrs8 meta;                  // each rank's meta [cap] int4 {src, pair, gate_bits, 0}
  Words8 arrivals_peer;        // each rank's [n][El] counters

  __device__ int num_tiles() const { return mblk_prefix[El] * num_n; }
  __device__ int expert_of_mblock(int mb) const {
    int lo = 0, hi = El - 1;
    while (lo < hi) {  // last e with prefix[e] <= mb
      const int mid = (lo + hi + 1) >> 1;
      if (mblk_prefix[mid] <= mb) lo = mid; else hi = mid - 1;
    }
    return lo;
  }
  __device__ TileInfo tile(int t) const {
    // tiles ordered (expert, n-block, m-block): the m-blocks of an expert vary fastest so
    // one W1 tile is reused from L2 by all of them; expert e owns tiles
    // [prefix[e]*num_n, prefix[e+1]*num_n)
    const int e = expert_of_mblock(t / num_n);
    const int rem = t - mblk_prefix[e] * num_n;
    const int mbs = mblk_prefix[e + 1] - mblk_prefix[e];
    const int nb = mbs ? rem / mbs : 0, mb = mbs ? rem - nb * mbs : 0;
    TileInfo ti;
    ti.a_row = expert_base[e] + mb * BM;
    ti.m0 = ti.a_row;
    ti.n0 = nb * 256;
    ti.b_row = e * I2 + nb * 256;
    ti.kb0 = 0;
    ti.kb1 = H / BK;
    ti.aux = e;
    ti.aux2 = mb;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo& ti, uint64_t timeout_ns, volatile int* abort_flag,
                                ErrorRecord* err) const {
    const int e = ti.aux;
    for (int s = 0; s < n; ++s) {
      const uint64_t* c = arrivals + (size_t)s * El + e;
      const uint64_t target = cum_rows[(size_t)s * El + e];
      if (!wait_ge(c, target, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_MOE_COUNT, r, s, ptx::ld_relaxed_sys(c), target);
        return false;
      }
    }
    ptx::fence_proxy_async_global();
    return true;
  }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
  }
  // Dispatch: pairs in send order, dispatching CTA c takes pairs c, c+C, ...
  __device__ void comm(int cw, int lane, volatile int* abort_flag, ErrorRecord*, uint64_t) const {
    __shared__ int comm_stop;
    const int tid = cw * 32 + lane;
    constexpr int kT = kCommWarps * 32;
    const int nvec = H / 8;  // 16-byte vectors per row
    constexpr int kBatch = 16;  // rows per fence / barrier (a fence waits for every store in flight)
    constexpr int kVec = 8;    // vectors in flight per thread
    if ((int)blockIdx.x >= C) return;
    // CTA c owns pairs c, c+C, c+2C, ... (send order, so every owner's first expert
    // completes first); kBatch of them share one fence and one barrier.
    for (int p0 = blockIdx.x; p0 < npairs; p0 += C * kBatch) {
      // one thread samples the CTA's abort flag; all comm threads leave together
      if (tid == 0) comm_stop = *abort_flag;
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (comm_stop) break;
#pragma unroll 1
      for (int j = 0; j < kBatch; ++j) {
        const int p = p0 + j * C;
        if (p >= npairs) break;
        const int pair = send_pair[p];
        const int row = send_row[p];
        const int tok = pair / topk;
        const int d = topk_idx[pair] / El;
        const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok * H);
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(recv.p[d]) + (size_t)row * H);
        for (int i0 = 0; i0 < nvec; i0 += kVec * kT) {
          uint4 v[kVec];
#pragma unroll
          for (int u = 0; u < kVec; ++u) {
            const int i = i0 + u * kT + tid;
            if (i < nvec) v[u] = ptx::ld_v4_nc(src + i);
          }
#pragma unroll
          for (int u = 0; u < kVec; ++u) {
            const int i = i0 + u * kT + tid;
            if (i < nvec) ptx::st_v4_na(dst + i, v[u]);
          }
        }
        if (tid == 0) {
          int4 m;
          m.x = r;
          m.y = pair;
          m.z = __float_as_int(topk_w[pair]);
          m.w = 0;
          reinterpret_cast<int4*>(meta.p[d])[row] = m;
        }
      }
      ptx::fence_acq_rel_sys();
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (tid < kBatch) {
        const int p = p0 + tid * C;
        if (p < npairs) {
          const int g = topk_idx[send_pair[p]];
          ptx::red_release_sys_add(arrivals_peer.p[g / El] + (size_t)r * El + (g - (g / El) * El), 1);
        }
      }
    }
  }
};

struct G1Epi {
  static constexpr bool kNeedsTileDone = false;
  static constexpr bool kPairHalves = true;
  uint16_t* h;            // [cap][I] activations
  int I;                  // inter
  const int* expert_rows;
  const int* expert_base;
  __device__ static void fence_before_done() {}
  __device__ void tile_done(const TileInfo&) {}
  __device__ void begin_tile(const TileInfo&, int) {}
  __device__ void end_tile(const TileInfo&, int) {}
  __device__ void store(const TileInfo&, int, int, const uint32_t*) {}
  __device__ __forceinline__ void store_pair(const TileInfo& ti, int row, int c, const uint32_t* g, const uint32_t* u) {
    const int e = ti.aux;
    if (ti.aux2 * BM + row >= expert_rows[e]) return;  // padding row of the expert segment
    uint16_t* p = h + (size_t)(ti.a_row + row) * I + ti.n0 / 2 + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float a[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float gv = __uint_as_float(g[8 * j + q]);
        a[q] = gv / (1.0f + expf(-gv)) * __uint_as_float(u[8 * j + q]);
      }
      uint4 v;
      v.x = ptx::pack_bf16x2(a[0], a[1]);
      v.y = ptx::pack_bf16x2(a[2], a[3]);
      v.z = ptx::pack_bf16x2(a[4], a[5]);
      v.w = ptx::pack_bf16x2(a[6], a[7]);
      ptx::st_v4(p + 8 * j, v);
    }
  }
};

template <bool Dyn>
__global__ void __launch_bounds__(cta_threads(kCommWarps), 1)
    k_moe_gemm1(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, G1SchedT<Dyn> s,
                G1Epi e, ErrorRecord* err, uint64_t timeout_ns, unsigned long long* next_ctr) {
  if (Dyn && blockIdx.x == 0 && threadIdx.x == 0) *next_ctr = 0;  // the next call's counter
  gemm_core<256>(&tmA, &tmB, s, e, err, timeout_ns, s.r);
}

// ---------------------------------------------------------------------------------------
// 5. grouped GEMM 2: H W2^T, gate-weighted rows pushed to their source
// ---------------------------------------------------------------------------------------
struct G2Sched {
  static constexpr int kCommWarps = 0;
  int El, I, H, num_n;  // K = I, N = H
  const int* mblk_prefix;
  const int* expert_base;
  __device__ int num_tiles() const { return mblk_prefix[El] * num_n; }
  __device__ TileInfo tile(int t) const {
    const int mbq = t / num_n;
    int lo = 0, hi = El - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (mblk_prefix[mid] <= mbq) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    const int rem = t - mblk_prefix[e] * num_n;
    const int mbs = mblk_prefix[e + 1] - mblk_prefix[e];
    const int nb = mbs ? rem / mbs : 0, mb = mbs ? rem - nb * mbs : 0;
    TileInfo ti;
    ti.a_row = expert_base[e] + mb * BM;
    ti.m0 = ti.a_row;
    ti.n0 = nb * 256;
    ti.b_row = e * H + nb * 256;
    ti.kb0 = 0;
    ti.kb1 = I / BK;
    ti.aux = e;
    ti.aux2 = mb;
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

struct G2Epi {
  static constexpr bool kNeedsTileDone = true;
  static constexpr bool kPairHalves = false;
  int n, H;
  const int* expert_rows;
  const int4* meta;       // my [cap] meta
  Ptrs8 comb;             // each rank's combine buffer [T*topk][H]
  Words8 comb_arrivals;   // each rank's [1] arrival word
  // per-thread state
  int valid, src, pair;
  float gate;
  int tcount;
  __device__ static void fence_before_done() { ptx::fence_acq_rel_sys(); }
  __device__ uint32_t* counters() const {
    __shared__ uint32_t cnt[2][kMaxR];
    return &cnt[0][0];
  }
  __device__ void begin_tile(const TileInfo& ti, int row) {
    valid = ti.aux2 * BM + row < expert_rows[ti.aux];
    if (valid) {
      const int4 m = meta[ti.a_row + row];
      src = m.x;
      pair = m.y;
      gate = __int_as_float(m.z);
    }
  }
  __device__ __forceinline__ void store(const TileInfo& ti, int, int c, const uint32_t* acc) {
    if (!valid) return;
    uint16_t* p = reinterpret_cast<uint16_t*>(comb.p[src]) + (size_t)pair * H + ti.n0 + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 v;
      v.x = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 0]), gate * __uint_as_float(acc[8 * j + 1]));
      v.y = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 2]), gate * __uint_as_float(acc[8 * j + 3]));
      v.z = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 4]), gate * __uint_as_float(acc[8 * j + 5]));
      v.w = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 6]), gate * __uint_as_float(acc[8 * j + 7]));
      ptx::st_v4_na(p + 8 * j, v);
    }
  }
  __device__ void end_tile(const TileInfo&, int) {
    uint32_t* cnt = counters() + (tcount & 1) * kMaxR;
    if (valid) atomicAdd(&cnt[src], 1u);
    __threadfence_block();
    ++tcount;
  }
  __device__ void tile_done(const TileInfo&) {
    // runs in the last epilogue warp to finish (lane 0); tcount already advanced
    uint32_t* cnt = counters() + ((tcount - 1) & 1) * kMaxR;
    for (int s = 0; s < n; ++s) {
      const uint32_t c = atomicExch(&cnt[s], 0u);
      if (c) ptx::red_release_sys_add(comb_arrivals.p[s], c);
    }
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    k_moe_gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, G2Sched s, G2Epi e,
                ErrorRecord* err, uint64_t timeout_ns, int rank) {
  if (threadIdx.x < 2 * kMaxR) e.counters()[threadIdx.x] = 0;
  __syncthreads();
  e.tcount = 0;
  e.valid = 0;
  gemm_core<256>(&tmA, &tmB, s, e, err, timeout_ns, rank);
}

// ---------------------------------------------------------------------------------------
// 5b. grouped GEMM 2 with a staged combine (the combine_ctas option): the epilogue stores
// the gate-scaled rows into a local staging buffer and publishes each finished tile in a
// queue; the communication warps of `C` CTAs take tiles from the queue and push their rows
// to the source ranks, so only those SMs issue NVLink stores.  Tiles are taken dynamically,
// so the pushing CTAs do less math.  Counters come in parity pairs (the tile count follows
// the routing): call e uses set e & 1 and zeroes the other set for call e+1.
// ---------------------------------------------------------------------------------------
// A queued tile: expert (9 bits), m-block within the expert (14 bits), n-block (8 bits); the
// top bit stays clear so the value is a non-negative int.
__device__ __forceinline__ uint32_t pack_tile(int e, int mb, int nb) {
  return ((uint32_t)e << 22) | ((uint32_t)mb << 8) | (uint32_t)nb;  // e < 512, mb < 16384, nb < 256
}

struct G2StageSched {
  static constexpr int kCommWarps = moe::kCommWarps;
  static constexpr bool kDynamic = true;
  int n, El, I, H, num_n, C;
  const int* mblk_prefix;
  const int* expert_base;
  const int* expert_rows;
  unsigned long long* ctr;   // this call's set: [0] tiles taken, [1] queue tail, [2] queue head
  uint64_t* queue;           // [max tiles] entries (epoch << 32) | packed tile
  uint64_t epoch;
  const int4* meta;          // my [cap] meta
  const uint16_t* y;         // my staging [cap][H]
  Ptrs8 comb;                // each rank's combine buffer [T*topk][H]
  Words8 comb_arrivals;      // each rank's [1] arrival word

  __device__ int num_tiles() const { return mblk_prefix[El] * num_n; }
  __device__ int next_tile() const {
    const unsigned long long v = atomicAdd(&ctr[0], 1ull);
    return v < (unsigned long long)num_tiles() ? (int)v : num_tiles();
  }
  __device__ TileInfo tile(int t) const {
    const int mbq = t / num_n;
    int lo = 0, hi = El - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (mblk_prefix[mid] <= mbq) lo = mid; else hi = mid - 1;
    }
    const int e = lo;
    const int rem = t - mblk_prefix[e] * num_n;
    const int mbs = mblk_prefix[e + 1] - mblk_prefix[e];
    const int nb = mbs ? rem / mbs : 0, mb = mbs ? rem - nb * mbs : 0;
    TileInfo ti;
    ti.a_row = expert_base[e] + mb * BM;
    ti.m0 = ti.a_row;
    ti.n0 = nb * 256;
    ti.b_row = e * H + nb * 256;
    ti.kb0 = 0;
    ti.kb1 = I / BK;
    ti.aux = e;
    ti.aux2 = mb;
    return ti;
  }
  __device__ bool producer_wait(const TileInfo&, uint64_t, volatile int*, ErrorRecord*) const { return true; }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
    ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
  }
  // Push queued tiles: one warp per row (32 lanes x 16 bytes = the tile's 256 columns).
  __device__ void comm(int cw, int lane, volatile int* abort_flag, ErrorRecord* err, uint64_t timeout_ns) const {
    __shared__ int comm_tile;
    __shared__ uint32_t cnt[kMaxR];
    const int tid = cw * 32 + lane;
    constexpr int kT = kCommWarps * 32;
    if ((int)blockIdx.x >= C) return;
    if (tid < kMaxR) cnt[tid] = 0;
    const int T = num_tiles();
    for (;;) {
      if (tid == 0) {
        int packed = -1;
        const unsigned long long idx = atomicAdd(&ctr[2], 1ull);
        if (idx < (unsigned long long)T && !*abort_flag) {
          const uint64_t* q = queue + idx;
          const uint64_t t0 = ptx::globaltimer();
          for (uint32_t i = 0;; ++i) {
            const uint64_t v = ptx::ld_acquire_sys(q);
            if ((v >> 32) == (epoch & 0xffffffffull)) {
              packed = (int)(v & 0xffffffffull);
              break;
            }
            if ((i & 63) == 63 && (*abort_flag || ptx::globaltimer() - t0 > timeout_ns)) {
              if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_MOE_COUNT, -1, -1, v, epoch);
              *abort_flag = 1;
              break;
            }
          }
        }
        comm_tile = packed;
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      const int packed = comm_tile;
      if (packed < 0) break;
      const int e = packed >> 22, mb = (packed >> 8) & 0x3fff, nb = packed & 0xff;
      const int a_row = expert_base[e] + mb * BM;
      const int valid = min(BM, expert_rows[e] - mb * BM);
      // Each warp loads kRows rows before it stores any, so kRows loads per lane are in
      // flight (one row at a time leaves a single load in flight and bounds the push rate
      // by the load latency).
      constexpr int kRows = 8;
      for (int row0 = cw * kRows; row0 < valid; row0 += kCommWarps * kRows) {
        int4 m[kRows];
        uint4 v[kRows];
#pragma unroll
        for (int k = 0; k < kRows; ++k) {
          const int row = row0 + k;
          if (row < valid) {
            m[k] = meta[a_row + row];
            v[k] = reinterpret_cast<const uint4*>(y + (size_t)(a_row + row) * H + nb * 256)[lane];
          }
        }
#pragma unroll
        for (int k = 0; k < kRows; ++k) {
          if (row0 + k < valid) {
            uint16_t* dst = reinterpret_cast<uint16_t*>(comb.p[m[k].x]) + (size_t)m[k].y * H + nb * 256;
            ptx::st_v4_na(reinterpret_cast<uint4*>(dst) + lane, v[k]);
            if (lane == 0) atomicAdd(&cnt[m[k].x], 1u);
          }
        }
      }
      ptx::fence_acq_rel_sys();
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
      if (tid < n) {
        const uint32_t c = cnt[tid];
        cnt[tid] = 0;
        if (c) ptx::red_release_sys_add(comb_arrivals.p[tid], c);
      }
      asm volatile("bar.sync 2, %0;" ::"n"(kT) : "memory");
    }
  }
};

struct G2StageEpi {
  static constexpr bool kNeedsTileDone = true;
  static constexpr bool kPairHalves = false;
  int H;
  const int* expert_rows;
  const int4* meta;
  uint16_t* y;               // my staging [cap][H]
  unsigned long long* ctr;   // this call's set (queue tail at [1])
  uint64_t* queue;
  uint64_t epoch;
  int valid;
  float gate;
  __device__ static void fence_before_done() { ptx::fence_acq_rel_sys(); }
  __device__ void begin_tile(const TileInfo& ti, int row) {
    valid = ti.aux2 * BM + row < expert_rows[ti.aux];
    if (valid) gate = __int_as_float(meta[ti.a_row + row].z);
  }
  __device__ __forceinline__ void store(const TileInfo& ti, int row, int c, const uint32_t* acc) {
    if (!valid) return;
    uint16_t* p = y + (size_t)(ti.a_row + row) * H + ti.n0 + c;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint4 v;
      v.x = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 0]), gate * __uint_as_float(acc[8 * j + 1]));
      v.y = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 2]), gate * __uint_as_float(acc[8 * j + 3]));
      v.z = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 4]), gate * __uint_as_float(acc[8 * j + 5]));
      v.w = ptx::pack_bf16x2(gate * __uint_as_float(acc[8 * j + 6]), gate * __uint_as_float(acc[8 * j + 7]));
      ptx::st_v4(p + 8 * j, v);
    }
  }
  __device__ void end_tile(const TileInfo&, int) {}
  __device__ void tile_done(const TileInfo& ti) {  // last epilogue warp, after every warp's stores
    const unsigned long long slot = atomicAdd(&ctr[1], 1ull);
    ptx::st_release_sys(queue + slot, (epoch << 32) | pack_tile(ti.aux, ti.aux2, ti.n0 / 256));
  }
};

__global__ void __launch_bounds__(cta_threads(kCommWarps), 1)
    k_moe_gemm2_staged(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       G2StageSched s, G2StageEpi e, ErrorRecord* err, uint64_t timeout_ns, int rank,
                       unsigned long long* next_ctr) {
  if (blockIdx.x == 0 && threadIdx.x < 3) next_ctr[threadIdx.x] = 0;  // the next call's set
  gemm_core<256>(&tmA, &tmB, s, e, err, timeout_ns, rank);
}

// ---------------------------------------------------------------------------------------
// 6. combine: out[t] = sum_j comb[t*topk + j]
// ---------------------------------------------------------------------------------------
// ---------------------------------------------------------------------------------------
// Communication only (MoeArgs::comm_only): the same dispatch and combine with identity
// experts, to time the all-to-all round trip by itself.  k_moe_dispatch runs the first
// grouped GEMM's dispatch warps alone; k_moe_return sends every received row, scaled by its
// gate, back to its source (counting H/256 per row, as the second GEMM's epilogue does), so
// k_combine then sums sum_j w_j * x[t] for every token.
// ---------------------------------------------------------------------------------------
__global__ void __launch_bounds__(kCommWarps * 32) k_moe_dispatch(G1SchedT<false> s, ErrorRecord* err,
                                                                   uint64_t timeout_ns) {
  __shared__ int abort_flag;
  if (threadIdx.x == 0) abort_flag = 0;
  __syncthreads();
  s.comm((int)threadIdx.x / 32, (int)threadIdx.x % 32, &abort_flag, err, timeout_ns);
}

struct ReturnArgs {
  int n, r, El, H;
  const int* mblk_prefix;
  const int* expert_base;
  const int* expert_rows;
  const uint64_t* arrivals;  // my [n][El] row counters
  const uint64_t* cum_rows;  // [n][El] targets
  const uint16_t* recv;      // my [cap][H]
  const int4* meta;          // my [cap]
  Ptrs8 comb;
  Words8 comb_arrivals;
};

__global__ void __launch_bounds__(256) k_moe_return(ReturnArgs a, ErrorRecord* err, uint64_t timeout_ns) {
  __shared__ int ok;
  __shared__ uint32_t cnt[kMaxR];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32, nwarps = blockDim.x / 32;
  if (threadIdx.x < kMaxR) cnt[threadIdx.x] = 0;
  const int blocks = a.mblk_prefix[a.El];
  for (int u = blockIdx.x; u < blocks; u += gridDim.x) {
    int lo = 0, hi = a.El - 1;  // the expert of m-block u
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.mblk_prefix[mid] <= u) lo = mid; else hi = mid - 1;
    }
    const int e = lo, mb = u - a.mblk_prefix[e];
    if (threadIdx.x == 0) {
      ok = 1;
      for (int src = 0; src < a.n && ok; ++src)
        if (!wait_ge(a.arrivals + (size_t)src * a.El + e, a.cum_rows[(size_t)src * a.El + e], timeout_ns, nullptr)) {
          report_error(err, GICC_ETIMEDOUT, W_MOE_COUNT, a.r, src, 0, a.cum_rows[(size_t)src * a.El + e]);
          ok = 0;
        }
    }
    __syncthreads();
    if (!ok) return;
    const int rows = min(BM, a.expert_rows[e] - mb * BM);
    const int row0 = a.expert_base[e] + mb * BM;
    for (int i = warp; i < rows; i += nwarps) {
      const int4 m = a.meta[row0 + i];
      const float gate = __int_as_float(m.z);
      const uint4* src = reinterpret_cast<const uint4*>(a.recv + (size_t)(row0 + i) * a.H);
      uint4* dst = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.comb.p[m.x]) + (size_t)m.y * a.H);
      // kU loads per lane in flight before the stores (one at a time is latency-bound)
      constexpr int kU = 7;
      const int nv = a.H / 8;
      for (int c0 = lane; c0 < nv; c0 += 32 * kU) {
        uint4 v[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u)
          if (c0 + 32 * u < nv) v[u] = src[c0 + 32 * u];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          if (c0 + 32 * u < nv) {
            uint4 o;
            o.x = ptx::pack_bf16x2(gate * ptx::bf16_lo(v[u].x), gate * ptx::bf16_hi(v[u].x));
            o.y = ptx::pack_bf16x2(gate * ptx::bf16_lo(v[u].y), gate * ptx::bf16_hi(v[u].y));
            o.z = ptx::pack_bf16x2(gate * ptx::bf16_lo(v[u].z), gate * ptx::bf16_hi(v[u].z));
            o.w = ptx::pack_bf16x2(gate * ptx::bf16_lo(v[u].w), gate * ptx::bf16_hi(v[u].w));
            ptx::st_v4_na(dst + c0 + 32 * u, o);
          }
        }
      }
      if (lane == 0) atomicAdd(&cnt[m.x], (uint32_t)(a.H / 256));
    }
    ptx::fence_acq_rel_sys();
    __syncthreads();
    if (threadIdx.x < a.n) {
      const uint32_t c = cnt[threadIdx.x];
      cnt[threadIdx.x] = 0;
      if (c) ptx::red_release_sys_add(a.comb_arrivals.p[threadIdx.x], c);
    }
    __syncthreads();
  }
}

__global__ void k_combine(const uint16_t* comb, uint16_t* out, int T, int H, int topk, const uint64_t* arrivals,
                          uint64_t target, ErrorRecord* err, uint64_t timeout_ns, int rank) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    ok = 1;
    if (!wait_ge(arrivals, target, timeout_ns, nullptr)) {
      report_error(err, GICC_ETIMEDOUT, W_MOE_COUNT, rank, -1, ptx::ld_relaxed_sys(arrivals), target);
      ok = 0;
    }
  }
  __syncthreads();
  if (!ok) return;
  const size_t nvec = (size_t)T * (H / 8);
  for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (size_t)gridDim.x * blockDim.x) {
    const size_t t = v / (H / 8), c = v - t * (H / 8);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < topk; ++j) {
      const uint4 x = reinterpret_cast<const uint4*>(comb + ((size_t)t * topk + j) * H)[c];
      const uint32_t w[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] += ptx::bf16_lo(w[q]);
        acc[2 * q + 1] += ptx::bf16_hi(w[q]);
      }
    }
    uint4 o;
    o.x = ptx::pack_bf16x2(acc[0], acc[1]);
    o.y = ptx::pack_bf16x2(acc[2], acc[3]);
    o.z = ptx::pack_bf16x2(acc[4], acc[5]);
    o.w = ptx::pack_bf16x2(acc[6], acc[7]);
    reinterpret_cast<uint4*>(out + (size_t)t * H)[c] = o;
  }
}

}  // namespace
}  // namespace moe

namespace ops {

void moe_route(const float* logits, int T, int E, int topk, int* topk_idx, float* topk_w, int* counts, cudaStream_t s) {
  if (E < topk || E > 1024 || topk < 1 || topk > 8) throw std::runtime_error("gicc::moe_route: topk <= E <= 1024, k <= 8");
  GICC_CUDA(cudaMemsetAsync(counts, 0, sizeof(int) * E, s));
  const int warps_per_block = 8;
  moe::k_route<<<(T + warps_per_block - 1) / warps_per_block, 32 * warps_per_block, 0, s>>>(logits, T, E, topk,
                                                                                           topk_idx, topk_w, counts);
  GICC_CUDA(cudaGetLastError());
}

void moe_forward(const MoeArgs& a, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::moe_forward");
  using namespace gemm;
  const int n = a.n, r = a.r, El = a.E / a.n;
  if (n < 1 || n > moe::kMaxR) throw std::runtime_error("gicc::moe: 1..8 ranks");
  if (a.E % n || El > moe::kMaxLocalExperts || a.E > 1024)
    throw std::runtime_error("gicc::moe: E <= 1024 must split evenly, <= 256 per rank");
  if (a.H % 256 || a.I % 128 || a.H % BK || a.I % BK) throw std::runtime_error("gicc::moe: hidden % 256, inter % 128");
  const int pairs = a.T * a.topk;
  ErrorRecord* err = device_error_record();
  const uint64_t tmo = a.timeout_ns ? a.timeout_ns : default_timeout_ns();
  // optional per-stage timing (profiling only: synchronises at the end)
  cudaEvent_t ev[7] = {};
  auto mark = [&](int i) {
    if (a.stage_ms) GICC_CUDA(cudaEventRecord(ev[i], s));
  };
  if (a.stage_ms)
    for (auto& e : ev) GICC_CUDA(cudaEventCreate(&e));
  mark(0);
  // 1. route
  moe_route(a.logits, a.T, a.E, a.topk, a.topk_idx, a.topk_w, a.counts, s);
  mark(1);
  // 2. plan
  moe::PlanArgs p{};
  p.n = n;
  p.r = r;
  p.E = a.E;
  p.El = El;
  p.counts = a.counts;
  for (int i = 0; i < n; ++i) {
    p.count_tab.p[i] = a.count_tab[i];
    p.flags.p[i] = a.plan_flags[i];
  }
  p.epoch = a.epoch;
  p.dest_row_base = a.ws.dest_row_base;
  p.key_base = a.ws.key_base;
  p.key_cursor = a.ws.key_cursor;
  p.expert_base = a.ws.expert_base;
  p.expert_rows = a.ws.expert_rows;
  p.mblk_prefix = a.ws.mblk_prefix;
  p.cum_rows = a.ws.cum_rows;
  p.cum_pairs = a.ws.cum_pairs;
  p.pairs = pairs;
  p.err = err;
  p.timeout_ns = tmo;
  moe::k_plan<<<1, 256, 0, s>>>(p);
  GICC_CUDA(cudaGetLastError());
  mark(2);
  // 3. sort
  moe::k_sort<<<(pairs + 255) / 256, 256, 0, s>>>(a.topk_idx, pairs, n, r, El, a.ws.key_base, a.ws.key_cursor,
                                                  a.ws.dest_row_base, a.ws.send_pair, a.ws.send_row);
  GICC_CUDA(cudaGetLastError());
  mark(3);
  // 4. GEMM 1 (+ dispatch)
  const int G = num_sms();
  if (a.comm_only) {  // identity experts: dispatch, return, combine
    moe::G1SchedT<false> d{};
    d.n = n;
    d.r = r;
    d.El = El;
    d.H = a.H;
    d.topk = a.topk;
    d.G = G;
    d.C = G;
    d.npairs = pairs;
    d.send_pair = a.ws.send_pair;
    d.send_row = a.ws.send_row;
    d.topk_idx = a.topk_idx;
    d.topk_w = a.topk_w;
    d.x = static_cast<const uint16_t*>(a.x);
    for (int i = 0; i < n; ++i) {
      d.recv.p[i] = a.recv[i];
      d.meta.p[i] = a.meta[i];
      d.arrivals_peer.p[i] = a.arrivals[i];
    }
    moe::k_moe_dispatch<<<G, moe::kCommWarps * 32, 0, s>>>(d, err, tmo);
    GICC_CUDA(cudaGetLastError());
    mark(4);
    moe::ReturnArgs ra{};
    ra.n = n;
    ra.r = r;
    ra.El = El;
    ra.H = a.H;
    ra.mblk_prefix = a.ws.mblk_prefix;
    ra.expert_base = a.ws.expert_base;
    ra.expert_rows = a.ws.expert_rows;
    ra.arrivals = a.arrivals[r];
    ra.cum_rows = a.ws.cum_rows;
    ra.recv = static_cast<const uint16_t*>(a.recv[r]);
    ra.meta = static_cast<const int4*>(a.meta[r]);
    for (int i = 0; i < n; ++i) {
      ra.comb.p[i] = a.comb[i];
      ra.comb_arrivals.p[i] = a.comb_arrivals[i];
    }
    moe::k_moe_return<<<2 * G, 256, 0, s>>>(ra, err, tmo);
    GICC_CUDA(cudaGetLastError());
    mark(5);
    const uint64_t target = a.epoch * (uint64_t)pairs * (uint64_t)(a.H / 256);
    moe::k_combine<<<4 * G, 256, 0, s>>>(static_cast<const uint16_t*>(a.comb[r]), static_cast<uint16_t*>(a.out), a.T,
                                          a.H, a.topk, a.comb_arrivals[r], target, err, tmo, r);
    GICC_CUDA(cudaGetLastError());
    mark(6);
    if (a.stage_ms) {
      GICC_CUDA(cudaEventSynchronize(ev[6]));
      for (int i = 0; i < 6; ++i) GICC_CUDA(cudaEventElapsedTime(&a.stage_ms[i], ev[i], ev[i + 1]));
      for (auto& e : ev) cudaEventDestroy(e);
    }
    return;
  }
  const CUtensorMap tA1 = make_tmap_2d(a.recv[r], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.cap_rows, a.H, a.H, BM, BK,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB1 = make_tmap_2d(a.w1, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)El * 2 * a.I, a.H, a.H, 256,
                                       BK, CU_TENSOR_MAP_SWIZZLE_128B);
  const bool dyn = a.dispatch_ctas > 0 && a.dispatch_ctas < G;
  if (dyn && !a.ws.g1_tile_ctr) throw std::runtime_error("gicc::moe_forward: dispatch_ctas needs ws.g1_tile_ctr");
  moe::G1SchedT<false> g1{};
  g1.n = n;
  g1.r = r;
  g1.El = El;
  g1.H = a.H;
  g1.I2 = 2 * a.I;
  g1.num_n = 2 * a.I / 256;
  g1.topk = a.topk;
  g1.G = G;
  g1.C = dyn ? a.dispatch_ctas : G;
  g1.tile_ctr = dyn ? reinterpret_cast<unsigned long long*>(a.ws.g1_tile_ctr) + (a.epoch & 1) : nullptr;
  unsigned long long* next_ctr =
      dyn ? reinterpret_cast<unsigned long long*>(a.ws.g1_tile_ctr) + ((a.epoch + 1) & 1) : nullptr;
  g1.mblk_prefix = a.ws.mblk_prefix;
  g1.expert_base = a.ws.expert_base;
  g1.arrivals = a.arrivals[r];
  g1.cum_rows = a.ws.cum_rows;
  g1.npairs = pairs;
  g1.send_pair = a.ws.send_pair;
  g1.send_row = a.ws.send_row;
  g1.topk_idx = a.topk_idx;
  g1.topk_w = a.topk_w;
  g1.x = static_cast<const uint16_t*>(a.x);
  for (int i = 0; i < n; ++i) {
    g1.recv.p[i] = a.recv[i];
    g1.meta.p[i] = a.meta[i];
    g1.arrivals_peer.p[i] = a.arrivals[i];
  }
  moe::G1Epi e1{static_cast<uint16_t*>(a.h), a.I, a.ws.expert_rows, a.ws.expert_base};
  constexpr uint32_t smem = Cfg<256>::kSmemBytes;
  static bool attr[64] = {false};
  int dev = 0;
  GICC_CUDA(cudaGetDevice(&dev));
  if (!attr[dev]) {
    GICC_CUDA(cudaFuncSetAttribute(moe::k_moe_gemm1<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    GICC_CUDA(cudaFuncSetAttribute(moe::k_moe_gemm1<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    GICC_CUDA(cudaFuncSetAttribute(moe::k_moe_gemm2, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    attr[dev] = true;
  }
  if (dyn) {
    moe::G1SchedT<true> g1d;
    static_assert(sizeof(g1d) == sizeof(g1), "the two schedules share one layout");
    std::memcpy(&g1d, &g1, sizeof(g1));
    moe::k_moe_gemm1<true><<<G, cta_threads(moe::kCommWarps), smem, s>>>(tA1, tB1, g1d, e1, err, tmo, next_ctr);
  } else {
    moe::k_moe_gemm1<false><<<G, cta_threads(moe::kCommWarps), smem, s>>>(tA1, tB1, g1, e1, err, tmo, nullptr);
  }
  GICC_CUDA(cudaGetLastError());
  mark(4);
  // 5. GEMM 2 (+ combine push)
  const CUtensorMap tA2 = make_tmap_2d(a.h, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.cap_rows, a.I, a.I, BM, BK,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  const CUtensorMap tB2 = make_tmap_2d(a.w2, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)El * a.H, a.I, a.I, 256, BK,
                                       CU_TENSOR_MAP_SWIZZLE_128B);
  moe::G2Sched g2{El, a.I, a.H, a.H / 256, a.ws.mblk_prefix, a.ws.expert_base};
  moe::G2Epi e2{};
  e2.n = n;
  e2.H = a.H;
  e2.expert_rows = a.ws.expert_rows;
  e2.meta = static_cast<const int4*>(a.meta[r]);
  for (int i = 0; i < n; ++i) {
    e2.comb.p[i] = a.comb[i];
    e2.comb_arrivals.p[i] = a.comb_arrivals[i];
  }
  if (a.combine_ctas > 0 && a.combine_ctas < G) {
    if (!a.ws.g2_ctr || !a.ws.g2_queue || !a.y_stage)
      throw std::runtime_error("gicc::moe_forward: combine_ctas needs ws.g2_ctr, ws.g2_queue and y_stage");
    if (El > 512 || a.cap_rows / BM > 16384 || a.H / 256 > 255)  // a queue entry packs (e, mb, nb) in 31 bits
      throw std::runtime_error("gicc::moe_forward: combine_ctas supports El <= 512, cap/128 <= 16384, H/256 < 256");
    unsigned long long* cur = reinterpret_cast<unsigned long long*>(a.ws.g2_ctr) + 3 * (a.epoch & 1);
    unsigned long long* nxt = reinterpret_cast<unsigned long long*>(a.ws.g2_ctr) + 3 * ((a.epoch + 1) & 1);
    moe::G2StageSched gs{};
    gs.n = n;
    gs.El = El;
    gs.I = a.I;
    gs.H = a.H;
    gs.num_n = a.H / 256;
    gs.C = a.combine_ctas;
    gs.mblk_prefix = a.ws.mblk_prefix;
    gs.expert_base = a.ws.expert_base;
    gs.expert_rows = a.ws.expert_rows;
    gs.ctr = cur;
    gs.queue = a.ws.g2_queue;
    gs.epoch = a.epoch;
    gs.meta = static_cast<const int4*>(a.meta[r]);
    gs.y = static_cast<const uint16_t*>(a.y_stage);
    for (int i = 0; i < n; ++i) {
      gs.comb.p[i] = a.comb[i];
      gs.comb_arrivals.p[i] = a.comb_arrivals[i];
    }
    moe::G2StageEpi es{};
    es.H = a.H;
    es.expert_rows = a.ws.expert_rows;
    es.meta = static_cast<const int4*>(a.meta[r]);
    es.y = static_cast<uint16_t*>(a.y_stage);
    es.ctr = cur;
    es.queue = a.ws.g2_queue;
    es.epoch = a.epoch;
    static bool attr2[64] = {false};
    if (!attr2[dev]) {
      GICC_CUDA(cudaFuncSetAttribute(moe::k_moe_gemm2_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      attr2[dev] = true;
    }
    moe::k_moe_gemm2_staged<<<G, cta_threads(moe::kCommWarps), smem, s>>>(tA2, tB2, gs, es, err, tmo, r, nxt);
  } else {
    moe::k_moe_gemm2<<<G, kThreads, smem, s>>>(tA2, tB2, g2, e2, err, tmo, r);
  }
  GICC_CUDA(cudaGetLastError());
  mark(5);
  // 6. combine
  const uint64_t target = a.epoch * (uint64_t)pairs * (uint64_t)(a.H / 256);
  moe::k_combine<<<4 * G, 256, 0, s>>>(static_cast<const uint16_t*>(a.comb[r]), static_cast<uint16_t*>(a.out), a.T, a.H,
                                        a.topk, a.comb_arrivals[r], target, err, tmo, r);
  GICC_CUDA(cudaGetLastError());
  mark(6);
  if (a.stage_ms) {
    GICC_CUDA(cudaEventSynchronize(ev[6]));
    for (int i = 0; i < 6; ++i) GICC_CUDA(cudaEventElapsedTime(&a.stage_ms[i], ev[i], ev[i + 1]));
    for (auto& e : ev) cudaEventDestroy(e);
  }
}

}  // namespace ops
}  // namespace gicc
