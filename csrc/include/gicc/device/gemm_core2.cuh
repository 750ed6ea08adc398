// gemm_core2.cuh -- persistent tcgen05 GEMM core on CTA pairs (cta_group::2).
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x (NH*256) output tile:
//   * each CTA TMA-loads its own 128 rows of A and, for each of the NH column halves, its
//     own 128 rows of B (no multicast: every load reads this GPU's memory); both CTAs'
//     loads complete on the leader CTA's "full" mbarrier (cta_group::2 form of
//     cp.async.bulk.tensor);
//   * one thread of the leader issues tcgen05.mma.cta_group::2 (M=256, N=256, K=16 of
//     bf16, or K=8 of tf32 for schedules with kTf32: the same 32 bytes of a 128-byte row) NH
//     times per k-step (the A tile is shared by the NH halves), which reads both CTAs'
//     shared memory and accumulates into both CTAs' TMEM (each CTA holds its 128 rows x
//     NH*256 columns);
//   * NH = 1: the accumulator is double-buffered (2 x 256 of the 512 TMEM columns), so the
//     epilogue of tile i overlaps the MMAs of tile i+1;
//     NH = 2: one 512-column accumulator (all of TMEM), drained by 8 epilogue warps (two
//     per TMEM lane quarter, each 128 columns of each half) column half 0 first; the MMA
//     thread starts the next tile on half 0 as soon as that half is free, for up to
//     kStages - 1 k-steps, and issues the lagging half-1 MMAs of those k-steps once the
//     epilogue has drained half 1 (the stages are released only then), so most of the
//     drain overlaps tensor work;
//   * the epilogue reads TMEM in batches of up to 128 columns per tcgen05.wait::ld (as the
//     launch's registers allow) and, for epilogues with kStagedStore, writes bf16 C through
//     two 2 KB shared-memory boxes per warp to TMA stores (whole lines to L2);
//   * the leader's tcgen05.commit arrives on the barrier of each CTA (two commits, no
//     multicast form), and the peer CTA's epilogue warps arrive on the leader's
//     "accumulator free" barrier remotely.
// Shared-memory traffic per SM and k-step (64 deep), per 128 x 256 block of output:
//   single-CTA 128 x 256 tile: 16 KB of A + 32 KB of B = 48 KB;
//   pair, NH = 1:             16 KB of A + 16 KB of B = 32 KB;
//   pair, NH = 2:            (16 KB of A + 32 KB of B) / 2 = 24 KB,
// and the shared-memory ring (192 KB) covers 2, 3 and 4 k-steps of MMA time respectively,
// so the wider tile both halves the L2 -> SMEM bytes per FLOP of the single-CTA kernel and
// doubles the load latency it tolerates.
//
// Warp roles per CTA: 0 producer, 1 TMEM + MMA (leader only issues), 2.. epilogue.  Every
// wait is bounded; both CTAs always reach the final cluster barrier, after which TMEM is
// released.
#pragma once
#include <cstdint>
#include <type_traits>

#include "gicc/device/gemm_core.cuh"

namespace gicc {
namespace gemm {
namespace pair {

constexpr int BN2 = 256;  // columns per MMA (each CTA loads BN2/2 rows of B per column half)
constexpr uint32_t kABytes = BM * BK * 2;          // 16 KB
constexpr uint32_t kBBytes = (BN2 / 2) * BK * 2;   // 16 KB per column half

template <int NH>
struct PairCfg {
  static_assert(NH == 1 || NH == 2, "a pair tile has 1 or 2 column halves of 256");
  static constexpr int kCols = NH * BN2;                  // output columns of a pair tile
  static constexpr int kAccs = NH == 1 ? 2 : 1;           // TMEM accumulators (2 x 256 or 1 x 512)
  static constexpr uint32_t kStageBytes = kABytes + NH * kBBytes;
  static constexpr int kStages = NH == 1 ? 6 : 4;
  static constexpr int kEpiWarps = 4 * NH;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;  // without communication warps
  // threads of a CTA for a schedule with `comm_warps` communication warps after the epilogue
  __host__ __device__ static constexpr int threads(int comm_warps) { return kThreads + 32 * comm_warps; }
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + 256;
  // Epilogues that stage C through shared memory (Epi::kStagedStore): two 32 x 32 bf16
  // boxes per epilogue warp after the barrier area.
  static constexpr uint32_t kBoxBytes = 32 * 32 * 2;
  static constexpr uint32_t kSmemBytesStaged = kSmemBytes + kEpiWarps * 2 * kBoxBytes;
  static_assert(kSmemBytesStaged <= 227 * 1024, "shared memory");
};
// The 256 x 256 configuration's constants, kept under their original names.
constexpr int kStages = PairCfg<1>::kStages;
constexpr uint32_t kStageBytes = PairCfg<1>::kStageBytes;
constexpr uint32_t kTmemCols = PairCfg<1>::kTmemCols;
constexpr uint32_t kSmemBytes = PairCfg<1>::kSmemBytes;

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t map_to(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          ptx::smem_u32(dst)),
      "l"(m), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_2d_pair_hint(void* dst, const CUtensorMap* m, uint32_t bar_cluster_addr, int x,
                                                      int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(
          ptx::smem_u32(dst)),
      "l"(m), "r"(bar_cluster_addr), "r"(x), "r"(y), "l"(policy)
      : "memory");
}
// Prefetch of one tile of a tensor map into L2 (no shared memory, no completion).
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* m, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(m), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_pair_tf32(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}
__device__ __forceinline__ void arrive_cluster(uint32_t bar_cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster_addr) : "memory");
}
// Bounded wait on an mbarrier phase with cluster-scope acquire semantics: for barriers
// that another CTA of the cluster arrives on after writing this CTA's shared memory.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(ptx::smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint64_t timeout_ns,
                                                  volatile int* abort_flag) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    if ((i & 15) == 0) {
      if (abort_flag != nullptr && *abort_flag) return false;
      if (ptx::globaltimer() - t0 > timeout_ns) return false;
    }
  }
}
// 32-bit store into another CTA's shared memory (address from map_to).
__device__ __forceinline__ void st_cluster_u32(uint32_t addr, int v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ptx::smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Epilogues with `static constexpr bool kStagedStore = true` may store C through shared
// memory and TMA (Epi::staged(), Epi::pack(), Epi::tmap(), Epi::chunk_in_bounds()).
template <class E, class = void>
struct epi_staged : std::false_type {};
template <class E>
struct epi_staged<E, std::void_t<decltype(E::kStagedStore)>> : std::integral_constant<bool, E::kStagedStore> {};

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }

// Options of the operand loads (the plain GEMM's tuning; the fused kernels use none):
// l2hint 1 = A kept in L2 / B streamed, 2 = the reverse; prefetch = k-steps ahead at which
// each CTA's producer prefetches its A and B boxes into L2 while loading the current one.
struct PairLoadOpts {
  int l2hint = 0;
  int prefetch = 0;
};

// Sched for pairs: tile(t) gives the pair tile (m0 = first of 256 rows, n0 = first of
// NH*256 columns, kb range); the core derives each CTA's A row (m0 + 128*rank) and B rows
// (n0 + h*256 + 128*rank for column half h).  Epi::store gets the CTA-local row (0..127)
// and the column offset within the pair tile.
//
// Schedules with kDynamic take tiles from Sched::next_tile(), called by the leader's
// producer only; the index goes to both CTAs through a 4-entry queue in shared memory (the
// leader writes its own and the peer's entry, st.shared::cluster, then arrives on both
// CTAs' "queue full" barriers with cluster-scope release).  Readers -- the leader's MMA
// thread, the peer's producer and every epilogue warp of both CTAs -- arrive on the
// leader's "queue empty" barrier.  Sched::producer_wait(ti, crank, ...) runs in each CTA's
// producer before that CTA loads its half of a tile.  Schedules with kCommWarps > 0 get
// that many warps after the epilogue warps, running Sched::comm.  Epilogues with
// kNeedsTileDone get tile_done(ti) once per CTA and tile (ti.m0 = that CTA's first row),
// after all of that CTA's epilogue warps stored their part.
template <int NH = 1, class Sched, class Epi>
__device__ __forceinline__ void gemm_core_pair(const CUtensorMap* tmA, const CUtensorMap* tmB, const Sched& sched,
                                               Epi& epi, ErrorRecord* err, uint64_t timeout_ns, int rank,
                                               PairLoadOpts lopt = PairLoadOpts()) {
  using Cf = PairCfg<NH>;
  constexpr int S = Cf::kStages;
  constexpr int kAccs = Cf::kAccs;
  constexpr bool kDyn = sched_dynamic<Sched>::value;
  // kind::tf32 schedules (Sched::kTf32): fp32 operands, 32 elements per 128-byte k-block
  constexpr bool kTf32 = sched_tf32<Sched>::value;
  constexpr int kKE = kTf32 ? 32 : BK;  // elements per k-block (the TMA x step)
  constexpr int kFirstComm = 2 + Cf::kEpiWarps;  // first communication warp
  extern __shared__ uint8_t gemm2_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm2_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kABytes;  // per stage: NH consecutive 16 KB boxes (one per column half)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * Cf::kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint64_t* tq_full = drain + 1;
  uint64_t* tq_empty = tq_full + kTileQ;  // only the leader's is used
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tq_empty + kTileQ);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* tq = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [kTileQ] tile indices
  // Per accumulator: epilogue warps of this CTA that finished a tile held in it (monotonic;
  // epilogues that publish finished tiles).
  uint32_t* epi_cnt = tmem_slot + 2 + kTileQ;

  const uint32_t warp = ptx::warp_id();
  const uint32_t lane = ptx::lane_id();
  const uint32_t crank = cta_rank();
  const bool leader = crank == 0;
  const int pair_id = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      ptx::mbar_init(&tfull[a], 1);
      ptx::mbar_init(&tempty[a], 2 * Cf::kEpiWarps);  // every epilogue warp of both CTAs
    }
    ptx::mbar_init(drain, 1);
    for (int q = 0; q < kTileQ; ++q) {
      ptx::mbar_init(&tq_full[q], 1);
      ptx::mbar_init(&tq_empty[q], 2 + 2 * Cf::kEpiWarps);  // MMA + peer producer + all epilogue warps
    }
    *abort_flag = 0;
    epi_cnt[0] = 0;
    epi_cnt[1] = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(tmA);
    ptx::prefetch_tmap(tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, Cf::kTmemCols);
    tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // peer barriers initialised before any remote arrive / TMA completion
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = sched.num_tiles();
  // the leader's queue-empty barriers and the peer's queue (leader writes it)
  const uint32_t tq_empty_leader = map_to(ptx::smem_u32(&tq_empty[0]), 0);
  const uint32_t tq_peer = map_to(ptx::smem_u32(const_cast<int*>(&tq[0])), 1);
  const uint32_t tq_full_peer = map_to(ptx::smem_u32(&tq_full[0]), 1);

  // Next tile index of the dynamic order for a reader (not the leader's producer); -1 ends.
  // Returns false on timeout (abort).
  auto take = [&](int& slot, uint32_t& qphase, int& t, bool epi_warp) -> bool {
    if (!mbar_wait_cluster(&tq_full[slot], qphase, timeout_ns, abort_flag)) return false;
    t = tq[slot];
    if (epi_warp) __syncwarp();
    if (!epi_warp || lane == 0) arrive_cluster(tq_empty_leader + slot * 8);
    if (++slot == kTileQ) {
      slot = 0;
      qphase ^= 1;
    }
    return true;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed[S];
#pragma unroll
      for (int s = 0; s < S; ++s) armed[s] = 0;
      int qslot = 0;
      uint32_t qphase = 0;
      uint64_t pol_a = 0, pol_b = 0;
      if (lopt.l2hint != 0) {
        const uint64_t keep = ptx::l2_policy_evict_last(), stream = ptx::l2_policy_evict_first();
        pol_a = lopt.l2hint == 1 ? keep : stream;
        pol_b = lopt.l2hint == 1 ? stream : keep;
      }
      for (int t = pair_id; !*abort_flag; t += npairs) {
        if constexpr (kDyn) {
          if (leader) {
            if (!mbar_wait_cluster(&tq_empty[qslot], qphase ^ 1, timeout_ns, abort_flag)) {
              if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 4, 0);
              *abort_flag = 1;
              break;
            }
            t = sched.next_tile();
            const int v = t < ntiles ? t : -1;
            tq[qslot] = v;
            st_cluster_u32(tq_peer + qslot * 4, v);
            ptx::mbar_arrive(&tq_full[qslot]);
            arrive_cluster(tq_full_peer + qslot * 8);
            if (++qslot == kTileQ) {
              qslot = 0;
              qphase ^= 1;
            }
          } else if (!take(qslot, qphase, t, false)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 1, 5, 0);
            *abort_flag = 1;
            break;
          }
          if (t < 0) break;
        }
        if (t >= ntiles) break;
        TileInfo ti = sched.tile(t);
        if (!sched.producer_wait(ti, (int)crank, timeout_ns, abort_flag, err)) {
          *abort_flag = 1;
          break;
        }
        bool ok = true;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!ptx::mbar_wait(&empty[stage], phase ^ 1, timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t bar = map_to(ptx::smem_u32(&full[stage]), 0);
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], 2 * Cf::kStageBytes);
          const int a_y = ti.a_row + (int)crank * BM;
          if (lopt.l2hint == 0) {
            tma_load_2d_pair(sA + stage * kABytes, tmA, bar, kb * kKE, a_y);
#pragma unroll
            for (int h = 0; h < NH; ++h)
              tma_load_2d_pair(sB + (stage * NH + h) * kBBytes, tmB, bar, kb * kKE,
                               ti.b_row + h * BN2 + (int)crank * (BN2 / 2));
          } else {
            tma_load_2d_pair_hint(sA + stage * kABytes, tmA, bar, kb * kKE, a_y, pol_a);
#pragma unroll
            for (int h = 0; h < NH; ++h)
              tma_load_2d_pair_hint(sB + (stage * NH + h) * kBBytes, tmB, bar, kb * kKE,
                                    ti.b_row + h * BN2 + (int)crank * (BN2 / 2), pol_b);
          }
          if (lopt.prefetch > 0 && kb + lopt.prefetch < ti.kb1) {
            const int px = (kb + lopt.prefetch) * kKE;
            tma_prefetch_2d(tmA, px, a_y);
#pragma unroll
            for (int h = 0; h < NH; ++h) tma_prefetch_2d(tmB, px, ti.b_row + h * BN2 + (int)crank * (BN2 / 2));
          }
          armed[stage]++;
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, (int)crank, 0, 0);
          *abort_flag = 1;
          break;
        }
      }
      if (*abort_flag && leader) {
        for (int s = 0; s < S; ++s)
          if (armed[s]) ptx::mbar_wait(&full[s], (armed[s] - 1) & 1, 20000000ull, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // ---------------- MMA issuer (leader CTA) ----------------
      constexpr uint32_t idesc = kTf32 ? ptx::idesc_tf32_f32(2 * BM, BN2) : ptx::idesc_bf16_f32(2 * BM, BN2);
      const uint32_t peer = 1;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      int qslot = 0;
      uint32_t qphase = 0;
      for (int t = pair_id; !*abort_flag; t += npairs) {
        if constexpr (kDyn) {
          if (!take(qslot, qphase, t, false)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 6, 0);
            *abort_flag = 1;
            break;
          }
          if (t < 0) break;
        }
        if (t >= ntiles) break;
        TileInfo ti = sched.tile(t);
        // NH = 1: tempty[acc] frees the whole accumulator; NH = 2: tempty[h] frees column half h.
        if (!ptx::mbar_wait(&tempty[acc], acc_phase ^ 1, timeout_ns, abort_flag)) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 1, 0);
          *abort_flag = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem + acc * NH * BN2;
        // k-step kb's MMAs for column halves [h0, h1) from the stage that holds it
        auto issue = [&](int st, int kb, int h0, int h1) {
          const uint32_t a0 = ptx::smem_u32(sA + st * kABytes);
          const uint32_t b0 = ptx::smem_u32(sB + st * NH * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = ptx::sdesc_kmajor_sw128(a0 + k * 32);
#pragma unroll
            for (int h = 0; h < NH; ++h) {
              if (h < h0 || h >= h1) continue;
              const uint64_t bd = ptx::sdesc_kmajor_sw128(b0 + h * kBBytes + k * 32);
              if constexpr (kTf32) mma_pair_tf32(d + h * BN2, ad, bd, idesc, (kb > ti.kb0 || k > 0) ? 1u : 0u);
              else mma_pair(d + h * BN2, ad, bd, idesc, (kb > ti.kb0 || k > 0) ? 1u : 0u);
            }
          }
        };
        auto release = [&](int st) {
          const uint32_t e_own = ptx::smem_u32(&empty[st]);
          commit_pair(e_own);
          commit_pair(map_to(e_own, peer));
        };
        bool ok = true;
        // NH = 2: the first `lag` k-steps run on half 0 only (their stages stay held), then
        // half 1 catches up once the epilogue has drained it.  One stage is left to the
        // producer so the k-step after the catch-up is already loaded.
        const int nk = ti.kb1 - ti.kb0;
        const int lag = NH == 2 ? (nk < S - 1 ? nk : S - 1) : 0;
        if (lag > 0) {
          int st = stage;
          for (int i = 0; i < lag; ++i) {
            if (!ptx::mbar_wait(&full[st], phase ^ (stage + i >= S ? 1u : 0u), timeout_ns, abort_flag)) {
              ok = false;
              break;
            }
            ptx::tc_fence_after();
            issue(st, ti.kb0 + i, 0, 1);
            issued = true;
            if (++st == S) st = 0;
          }
          if (ok && !ptx::mbar_wait(&tempty[1], acc_phase ^ 1, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 8, 0);
            *abort_flag = 1;
            break;
          }
          if (ok) {
            ptx::tc_fence_after();
            for (int i = 0; i < lag; ++i) {
              issue(stage, ti.kb0 + i, 1, NH);
              release(stage);
              if (++stage == S) {
                stage = 0;
                phase ^= 1;
              }
            }
          }
        } else if (NH == 2) {
          if (!ptx::mbar_wait(&tempty[1], acc_phase ^ 1, timeout_ns, abort_flag)) {
            if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 8, 0);
            *abort_flag = 1;
            break;
          }
          ptx::tc_fence_after();
        }
        for (int kb = ti.kb0 + lag; ok && kb < ti.kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          issue(stage, kb, 0, NH);
          issued = true;
          release(stage);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 2, 0);
          *abort_flag = 1;
          break;
        }
        const uint32_t f_own = ptx::smem_u32(&tfull[acc]);
        commit_pair(f_own);
        commit_pair(map_to(f_own, peer));
        if (++acc == kAccs) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (*abort_flag && issued) {
        commit_pair(ptx::smem_u32(drain));
        ptx::mbar_wait(drain, 0, 20000000ull, nullptr);
      }
    }
  } else if ((int)warp >= kFirstComm) {
    // ---------------- communication warps (schedules that move data) ----------------
    if constexpr (Sched::kCommWarps > 0) sched.comm((int)warp - kFirstComm, (int)lane, abort_flag, err, timeout_ns);
  } else {
    // ---------------- epilogue (warps 2.., both CTAs) ----------------
    // Warp w may read TMEM lanes 32*(w%4)..+31; with NH = 2 warps 2..5 take columns
    // 0..127 and warps 6..9 columns 128..255 of each column half of the same rows, half 0
    // first, and free each half (tempty[h]) as soon as they have read it.
    constexpr int kSeg = NH == 1 ? BN2 : BN2 / 2;  // columns of one half that a warp drains
    // TMEM columns read per wait: as many as the registers of this launch allow (65536 per
    // SM over Cf::threads(kCommWarps) threads, 1 CTA per SM)
    constexpr int kRegs = 65536 / Cf::threads(Sched::kCommWarps);
    constexpr int kW0 = kRegs >= 200 ? 128 : (kRegs >= 136 ? 64 : 32);
    constexpr int kW = kW0 < kSeg ? kW0 : kSeg;
    const int q = warp & 3;
    const int part = NH == 1 ? 0 : ((int)warp - 2) / 4;
    const int row = q * 32 + lane;
    // Staged stores: this warp's two 32 x 32 bf16 boxes, used in turn; the TMA store that
    // read a box must have finished reading it before the box is written again.
    constexpr bool kStaged = epi_staged<Epi>::value;
    uint8_t* my_boxes = smem + S * Cf::kStageBytes + 256 + ((int)warp - 2) * 2 * Cf::kBoxBytes;
    uint32_t box_turn = 0;
    const uint32_t tempty_leader0 = map_to(ptx::smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = map_to(ptx::smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    int qslot = 0;
    uint32_t qphase = 0;
    for (int t = pair_id;; t += npairs) {
      if constexpr (kDyn) {
        if (!take(qslot, qphase, t, true)) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, (int)crank, 7, 0);
          *abort_flag = 1;
          break;
        }
        if (t < 0) break;
      }
      if (t >= ntiles) break;
      TileInfo ti = sched.tile(t);
      ti.m0 += (int)crank * BM;  // this CTA's 128 rows of the pair tile
      if (!ptx::mbar_wait_long(&tfull[acc], acc_phase, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, (int)crank, 3, 0);
        *abort_flag = 1;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * NH * BN2;
      epi.begin_tile(ti, row);
#pragma unroll 1
      for (int h = 0; h < NH; ++h) {
        // the barrier that frees what this warp has read: the accumulator (NH = 1) or half h
        const uint32_t free_bar = (NH == 1 ? acc : h) ? tempty_leader1 : tempty_leader0;
#pragma unroll 1
        for (int c = 0; c < kSeg; c += kW) {
          // kW columns: every TMEM load issued before one wait (each wait is a round trip)
          const int col0 = h * BN2 + part * kSeg + c;
          uint32_t r[kW];
#pragma unroll
          for (int i = 0; i < kW / 32; ++i) ptx::tmem_ld32(tbase + col0 + 32 * i, r + 32 * i);
          ptx::tmem_ld_wait();
          // Epilogues that publish finished tiles free the last half only after tile_done
          // (below); half 0 of a 512-column accumulator can go back at once, because the
          // next tile's epilogue cannot start before half 1 is free.
          if (!Epi::kNeedsTileDone || h + 1 < NH) {
            if (c + kW >= kSeg) {
              ptx::tc_fence_before();
              __syncwarp();
              if (lane == 0) arrive_cluster(free_bar);
            }
          }
#pragma unroll
          for (int i = 0; i < kW / 32; ++i) {
            const int col = col0 + 32 * i;
            const uint32_t* ri = r + 32 * i;
            bool done = false;
            if constexpr (kStaged) {
              if (epi.staged()) {
                uint8_t* box = my_boxes + (box_turn & 1) * Cf::kBoxBytes;
                ++box_turn;
                if (lane == 0) bulk_wait_read_1();  // the store issued from this box two chunks ago
                __syncwarp();
                uint4 v[4];
                epi.pack(ri, v);
                // row `lane` of the box (64 bytes); the 16-byte pieces are written in an
                // order rotated by lane/2, so each group of 8 lanes covers all 32 banks
                const uint32_t rowaddr = ptx::smem_u32(box) + lane * 64;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const int cj = (j + (int)(lane >> 1)) & 3;
                  const uint4 w = cj == 0 ? v[0] : cj == 1 ? v[1] : cj == 2 ? v[2] : v[3];
                  st_shared_v4(rowaddr + cj * 16, w);
                }
                ptx::fence_proxy_async_smem();
                __syncwarp();
                if (lane == 0) {
                  if (epi.chunk_in_bounds(ti, q * 32, col))
                    ptx::tma_store_2d(epi.tmap(), box, ti.n0 + col, ti.m0 + q * 32);
                  ptx::bulk_commit();  // a group per box, empty when out of bounds, so the wait counts boxes
                }
                done = true;
              }
            }
            if (!done) epi.store(ti, row, col, ri);
          }
        }
      }
      epi.end_tile(ti, row);
      if constexpr (Epi::kNeedsTileDone) {
        // The last of this CTA's epilogue warps to finish publishes this CTA's 128 rows of
        // the tile (ti.m0 is this CTA's first row); the accumulator (its last half, with
        // NH = 2) goes back to the MMA warp only afterwards, so the next tile in it cannot
        // start counting first.
        Epi::fence_before_done();
        __syncwarp();
        if (lane == 0) {
          const uint32_t old = atomicAdd(&epi_cnt[acc], 1u);
          if (old % Cf::kEpiWarps == Cf::kEpiWarps - 1) {
            Epi::fence_before_done();
            epi.tile_done(ti);
          }
        }
        __syncwarp();
        ptx::tc_fence_before();
        if (lane == 0) arrive_cluster(NH == 1 ? (acc ? tempty_leader1 : tempty_leader0) : tempty_leader1);
      }
      if (++acc == kAccs) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    if constexpr (kStaged) {
      if (lane == 0) ptx::bulk_wait_all();  // staged stores complete before the CTA's memory goes
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer may still arrive on our barriers / the leader's MMAs write our TMEM
  if (warp == 1) {
    ptx::tc_fence_after();
    tmem_dealloc_pair(tmem, Cf::kTmemCols);
  }
}

}  // namespace pair
}  // namespace gemm
}  // namespace gicc
