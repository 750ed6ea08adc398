// gemm_core.cuh -- persistent, warp-specialised tcgen05 GEMM core for sm_100a.
//
//   C[M,N] = A[M,K] * B[N,K]^T      (bf16 in, f32 accumulate in TMEM)
//
// One CTA per SM (grid = #SMs), 6 warps:
//   warp 0        TMA producer: per k-block one A tile (128x64) and one B tile (BNx64),
//                 128-byte swizzle, into a STAGES-deep smem ring guarded by mbarriers.
//   warp 1        TMEM owner + MMA issuer: one elected thread issues tcgen05.mma
//                 (M=128, N=BN, K=16) x4 per k-block and tcgen05.commit's the smem slot
//                 back to the producer; the accumulator is double-buffered in TMEM
//                 (2 x BN columns) so the epilogue of tile i overlaps the MMAs of tile i+1.
//   warps 2..5    epilogue: tcgen05.ld (32 lanes x 32 columns per warp step), convert,
//                 and hand the values to the Epi policy (plain store, peer store, ...).
//
// The tile order and operand coordinates come from a Sched policy, the output side from
// an Epi policy, so the same core runs the plain GEMM, all-gather->GEMM (the producer
// waits on per-chunk arrival flags), GEMM->reduce-scatter (the epilogue stores into the
// owner GPU) and the MoE grouped GEMM.  This replaces the reference's SIMT stripe kernel
// (examples/gicc/mm.cu:47-62), which accumulates with per-element atomicAdd.
//
// Tile order: static (CTA b takes tiles b, b + grid, ...) or, for schedules that set
// kDynamic, dynamic: the producer thread takes the next tile index from a global counter
// (Sched::next_tile) and hands it to the MMA and epilogue warps through a 4-entry smem
// queue.  Dynamic order lets CTAs that also move data (communication warps) take fewer
// tiles, and keeps the whole grid on the tiles in index order.
//
// Every wait is bounded (timeout_ns via %globaltimer); on timeout the CTA records the
// error, lets its in-flight TMA loads and MMAs drain (again bounded), frees TMEM and
// returns.
#pragma once
#include <cstdint>
#include <type_traits>

#include "gicc/device/ptx.cuh"
#include "gicc/error.hpp"

namespace gicc {
namespace gemm {

constexpr int BM = 128;
constexpr int BK = 64;  // one 128-byte swizzle row of bf16
constexpr int kThreads = 192;   // without communication warps
constexpr int kEpiThreads = 128;

// Threads of a CTA for a schedule with `comm_warps` extra communication warps.
__host__ __device__ constexpr int cta_threads(int comm_warps) { return kThreads + 32 * comm_warps; }

// Schedules opt into dynamic tile order with `static constexpr bool kDynamic = true` and
// `__device__ int next_tile() const` (an index >= num_tiles() ends the CTA's work).
template <class S, class = void>
struct sched_dynamic : std::false_type {};
template <class S>
struct sched_dynamic<S, std::void_t<decltype(S::kDynamic)>> : std::bool_constant<S::kDynamic> {};

constexpr int kTileQ = 4;  // entries of the producer -> MMA/epilogue tile queue

template <int BN>
struct Cfg {
  static_assert(BN % 32 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 32 in [64, 256]");
  static constexpr int kStages = BN == 256 ? 4 : (BN >= 192 ? 5 : 6);
  static constexpr uint32_t kABytes = BM * BK * 2;
  static constexpr uint32_t kBBytes = BN * BK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr uint32_t kTmemCols = 2 * BN <= 32 ? 32 : (2 * BN <= 64 ? 64 : (2 * BN <= 128 ? 128 : (2 * BN <= 256 ? 256 : 512)));
  static constexpr uint32_t kBarBytes = 256;
  static constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + kBarBytes;
  // mbarriers (full/empty per stage, 2+2 accumulator, drain, 2 x tile queue) + 8 words
  static_assert((2 * kStages + 5 + 2 * 4) * 8 + 8 * 4 <= kBarBytes, "barrier area too small");
};

struct TileInfo {
  int m0;     // first output row of the tile
  int n0;     // first output column of the tile
  int a_row;  // row coordinate of the tile in A's tensor map
  int b_row;  // row coordinate of the tile in B's tensor map (B is [N, K])
  int kb0;    // first k-block
  int kb1;    // one past the last k-block
  int aux;    // policy-defined (source rank, owner rank, expert, ...)
  int aux2;
};

// Grouped (super-row) rasterisation so concurrently running CTAs share A and B bands in L2.
__device__ __forceinline__ void raster(int t, int num_m, int num_n, int group_m, int& mb, int& nb) {
  const int per_group = group_m * num_n;
  const int g = t / per_group;
  const int first = g * group_m;
  const int gsz = min(num_m - first, group_m);
  const int r = t - g * per_group;
  mb = first + r % gsz;
  nb = r / gsz;
}

// Plain schedule over an M x N output with K-major A and B.
struct PlainSched {
  int M, N, K;
  int bn;
  int num_m, num_n, group_m;
  // L2 eviction priority of the operand loads: 0 = none (default), 1 = A kept / B streamed
  // (A's m-blocks are reused by every column tile of a raster group), 2 = the reverse.
  int l2hint = 0;
  __device__ int num_tiles() const { return num_m * num_n; }
  __device__ TileInfo tile(int t) const {
    int mb, nb;
    raster(t, num_m, num_n, group_m, mb, nb);
    TileInfo ti;
    ti.m0 = mb * BM;
    ti.n0 = nb * bn;
    ti.a_row = mb * BM;
    ti.b_row = nb * bn;
    ti.kb0 = 0;
    ti.kb1 = (K + BK - 1) / BK;
    ti.aux = 0;
    ti.aux2 = 0;
    return ti;
  }
  static constexpr int kCommWarps = 0;
  __device__ bool producer_wait(const TileInfo&, uint64_t, volatile int*, ErrorRecord*) const { return true; }
  __device__ void issue_loads(const TileInfo& ti, int kb, void* sA, void* sB, uint64_t* bar, const CUtensorMap* tmA,
                              const CUtensorMap* tmB) const {
    if (l2hint == 0) {
      ptx::tma_load_2d(sA, tmA, bar, kb * BK, ti.a_row);
      ptx::tma_load_2d(sB, tmB, bar, kb * BK, ti.b_row);
    } else {
      const uint64_t keep = ptx::l2_policy_evict_last(), stream = ptx::l2_policy_evict_first();
      ptx::tma_load_2d_hint(sA, tmA, bar, kb * BK, ti.a_row, l2hint == 1 ? keep : stream);
      ptx::tma_load_2d_hint(sB, tmB, bar, kb * BK, ti.b_row, l2hint == 1 ? stream : keep);
    }
  }
  __device__ void comm(int, int, volatile int*, ErrorRecord*, uint64_t) const {}
};

// Schedules with `static constexpr bool kTf32 = true` feed fp32 operands (128-byte swizzle
// rows of 32 elements; their issue_loads use x = kb * 32) to kind::tf32 MMAs.
template <class S, class = void>
struct sched_tf32 : std::false_type {};
template <class S>
struct sched_tf32<S, std::void_t<decltype(S::kTf32)>> : std::integral_constant<bool, S::kTf32> {};

template <int BN, class Sched, class Epi>
__device__ __forceinline__ void gemm_core(const CUtensorMap* tmA, const CUtensorMap* tmB, const Sched& sched,
                                          Epi& epi, ErrorRecord* err, uint64_t timeout_ns, int rank) {
  using C = Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * C::kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * C::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tq_full = drain + 1;        // dynamic order: tile index published
  uint64_t* tq_empty = tq_full + kTileQ;  // ... and read by the MMA thread and 4 epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tq_empty + kTileQ);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  // Per accumulator: how many epilogue warps have finished a tile held in it (monotonic).
  // One counter per accumulator, because a fast warp can finish the tile in the other
  // accumulator before a slow warp finishes this one.
  uint32_t* epi_cnt = tmem_slot + 2;
  volatile int* tq = reinterpret_cast<volatile int*>(tmem_slot + 4);  // [kTileQ] tile indices
  constexpr bool kDyn = sched_dynamic<Sched>::value;

  const uint32_t warp = ptx::warp_id();
  const uint32_t lane = ptx::lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], kEpiThreads);
    }
    ptx::mbar_init(drain, 1);
    for (int q = 0; q < kTileQ; ++q) {
      ptx::mbar_init(&tq_full[q], 1);
      ptx::mbar_init(&tq_empty[q], 1 + kEpiThreads / 32);
    }
    *abort_flag = 0;
    epi_cnt[0] = 0;
    epi_cnt[1] = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(tmA);
    ptx::prefetch_tmap(tmB);
  }
  if (warp == 1) {
    ptx::tmem_alloc(tmem_slot, C::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before();
  __syncthreads();
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = sched.num_tiles();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed[S];
#pragma unroll
      for (int s = 0; s < S; ++s) armed[s] = 0;
      int tq_slot = 0;
      uint32_t tq_phase = 0;
      for (int t = blockIdx.x; !*abort_flag; t += gridDim.x) {
        if constexpr (kDyn) {
          if (!ptx::mbar_wait(&tq_empty[tq_slot], tq_phase ^ 1, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 4, 0);
            *abort_flag = 1;
            break;
          }
          t = sched.next_tile();
          tq[tq_slot] = t < ntiles ? t : -1;
          ptx::mbar_arrive(&tq_full[tq_slot]);
          if (++tq_slot == kTileQ) {
            tq_slot = 0;
            tq_phase ^= 1;
          }
        }
        if (t >= ntiles) break;
        TileInfo ti = sched.tile(t);
        if (!sched.producer_wait(ti, timeout_ns, abort_flag, err)) {
          *abort_flag = 1;
          break;
        }
        bool ok = true;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          ptx::mbar_arrive_expect_tx(&full[stage], C::kStageBytes);
          sched.issue_loads(ti, kb, sA + stage * C::kABytes, sB + stage * C::kBBytes, &full[stage], tmA, tmB);
          armed[stage]++;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 0, 0);
          *abort_flag = 1;
          break;
        }
      }
      if (*abort_flag) {
        // Let the TMA loads already issued land before the CTA's smem goes away.
        for (int s = 0; s < S; ++s)
          if (armed[s]) ptx::mbar_wait(&full[s], (armed[s] - 1) & 1, 20000000ull, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr bool kTf32 = sched_tf32<Sched>::value;
      constexpr uint32_t idesc = kTf32 ? ptx::idesc_tf32_f32(BM, BN) : ptx::idesc_bf16_f32(BM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      int tq_slot = 0;
      uint32_t tq_phase = 0;
      for (int t = blockIdx.x; !*abort_flag; t += gridDim.x) {
        if constexpr (kDyn) {
          if (!ptx::mbar_wait(&tq_full[tq_slot], tq_phase, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 5, 0);
            *abort_flag = 1;
            break;
          }
          t = tq[tq_slot];
          ptx::mbar_arrive(&tq_empty[tq_slot]);
          if (++tq_slot == kTileQ) {
            tq_slot = 0;
            tq_phase ^= 1;
          }
          if (t < 0) break;
        }
        if (t >= ntiles) break;
        TileInfo ti = sched.tile(t);
        if (!ptx::mbar_wait(&tempty[acc], acc_phase ^ 1, timeout_ns, abort_flag)) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 1, 0);
          *abort_flag = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        bool ok = true;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = ptx::smem_u32(sA + stage * C::kABytes);
          const uint32_t b0 = ptx::smem_u32(sB + stage * C::kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = ptx::sdesc_kmajor_sw128(a0 + k * 32);
            const uint64_t bd = ptx::sdesc_kmajor_sw128(b0 + k * 32);
            if constexpr (kTf32) ptx::mma_tf32_ss(d, ad, bd, idesc, (kb > ti.kb0 || k > 0) ? 1u : 0u);
            else ptx::mma_f16_ss(d, ad, bd, idesc, (kb > ti.kb0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          ptx::mma_commit(&empty[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 2, 0);
          *abort_flag = 1;
          break;
        }
        ptx::mma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (*abort_flag && issued) {
        // Wait for the MMAs in flight before TMEM is released.
        ptx::mma_commit(drain);
        ptx::mbar_wait(drain, 0, 20000000ull, nullptr);
      }
    }
  } else if (warp >= 6) {
    // ---------------- communication warps (schedules that move data) ----------------
    if constexpr (Sched::kCommWarps > 0) sched.comm((int)warp - 6, (int)lane, abort_flag, err, timeout_ns);
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row = q * 32 + lane;
    // TMEM columns read per tcgen05.wait::ld (each wait is a round trip): as many as the
    // launch's registers allow (65536 per SM over cta_threads(kCommWarps), 1 CTA per SM)
    constexpr int kRegs = 65536 / cta_threads(Sched::kCommWarps);
    constexpr int kW0 = kRegs >= 240 ? 128 : (kRegs >= 160 ? 64 : 32);
    constexpr int kW = kW0 < BN ? kW0 : BN;  // plain epilogues
    constexpr int kWh0 = kW0 >= 64 ? kW0 / 2 : 32;
    constexpr int kWh = kWh0 < BN / 2 ? kWh0 : BN / 2;  // per half, epilogues of column pairs
    static_assert(BN % kW == 0 && (BN / 2) % kWh == 0 && kWh % 32 == 0, "TMEM read batches must tile the accumulator");
    int acc = 0;
    uint32_t acc_phase = 0;
    int tq_slot = 0;
    uint32_t tq_phase = 0;
    for (int t = blockIdx.x;; t += gridDim.x) {
      if constexpr (kDyn) {
        if (!ptx::mbar_wait(&tq_full[tq_slot], tq_phase, timeout_ns, abort_flag)) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 6, 0);
          *abort_flag = 1;
          break;
        }
        t = tq[tq_slot];
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(&tq_empty[tq_slot]);
        if (++tq_slot == kTileQ) {
          tq_slot = 0;
          tq_phase ^= 1;
        }
        if (t < 0) break;
      }
      if (t >= ntiles) break;
      TileInfo ti = sched.tile(t);
      if (!ptx::mbar_wait_long(&tfull[acc], acc_phase, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, -1, 3, 0);
        *abort_flag = 1;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      epi.begin_tile(ti, row);
      if constexpr (Epi::kPairHalves) {
        // columns c and c + BN/2 together (e.g. gate | up halves of a SwiGLU tile)
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += kWh) {
          uint32_t lo[kWh], hi[kWh];
#pragma unroll
          for (int i = 0; i < kWh / 32; ++i) {
            ptx::tmem_ld32(tbase + c + 32 * i, lo + 32 * i);
            ptx::tmem_ld32(tbase + c + BN / 2 + 32 * i, hi + 32 * i);
          }
          ptx::tmem_ld_wait();
          if constexpr (!Epi::kNeedsTileDone) {
            if (c + kWh >= BN / 2) {
              ptx::tc_fence_before();
              ptx::mbar_arrive(&tempty[acc]);
            }
          }
#pragma unroll
          for (int i = 0; i < kWh / 32; ++i) epi.store_pair(ti, row, c + 32 * i, lo + 32 * i, hi + 32 * i);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += kW) {
          uint32_t r[kW];
#pragma unroll
          for (int i = 0; i < kW / 32; ++i) ptx::tmem_ld32(tbase + c + 32 * i, r + 32 * i);
          ptx::tmem_ld_wait();
          if constexpr (!Epi::kNeedsTileDone) {
            if (c + kW >= BN) {
              // all TMEM reads of this accumulator are done: hand it back to the MMA warp
              ptx::tc_fence_before();
              ptx::mbar_arrive(&tempty[acc]);
            }
          }
#pragma unroll
          for (int i = 0; i < kW / 32; ++i) epi.store(ti, row, c + 32 * i, r + 32 * i);
        }
      }
      epi.end_tile(ti, row);
      if constexpr (Epi::kNeedsTileDone) {
        // The last of the 4 epilogue warps to finish publishes the tile (e.g. releases a
        // flag on the owner GPU).  The accumulator is handed back only afterwards, so the
        // next tile in this accumulator cannot start counting before this one is complete;
        // the tile in the other accumulator counts on its own counter.
        Epi::fence_before_done();  // every thread: its own (possibly remote) stores first
        __syncwarp();
        if (lane == 0) {
          const uint32_t old = atomicAdd(&epi_cnt[acc], 1u);
          if ((old & 3u) == 3u) {
            Epi::fence_before_done();
            epi.tile_done(ti);
          }
        }
        __syncwarp();
        ptx::tc_fence_before();
        ptx::mbar_arrive(&tempty[acc]);
      }
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace gemm
}  // namespace gicc
