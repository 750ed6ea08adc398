// gemm_core2.cuh -- persistent tcgen05 GEMM core on CTA pairs (cta_group::2).
//
// A cluster of two CTAs on neighbouring SMs computes one 256 x BN2 output tile:
//   * each CTA TMA-loads its own 128 rows of A and its own BN2/2 rows of B (no multicast:
//     every load reads this GPU's memory); both CTAs' loads complete on the leader CTA's
//     "full" mbarrier (cta_group::2 form of cp.async.bulk.tensor);
//   * one thread of the leader issues tcgen05.mma.cta_group::2 (M=256, N=BN2, K=16), which
//     reads both CTAs' shared memory and accumulates into both CTAs' TMEM (each CTA holds
//     its 128 rows x BN2 columns, double-buffered: 2 x BN2 columns);
//   * the leader's tcgen05.commit arrives on the barrier of each CTA (two commits, no
//     multicast form), and the peer CTA's epilogue warps arrive on the leader's
//     "accumulator free" barrier remotely.
// Per SM and k-step this moves 16 KB of A and 16 KB of B instead of 16 KB + 32 KB for a
// 128 x 256 single-CTA tile with the same tensor work, i.e. a third less L2 -> SMEM traffic.
//
// Warp roles per CTA as in gemm_core.cuh (192 threads): 0 producer, 1 TMEM + MMA (leader
// only issues), 2..5 epilogue.  Every wait is bounded; both CTAs always reach the final
// cluster barrier, after which TMEM is released.
#pragma once
#include <cstdint>

#include "gicc/device/gemm_core.cuh"

namespace gicc {
namespace gemm {
namespace pair {

constexpr int BN2 = 256;  // pair tile width (each CTA loads BN2/2 rows of B)
constexpr int kStages = 6;
constexpr uint32_t kABytes = BM * BK * 2;          // 16 KB
constexpr uint32_t kBBytes = (BN2 / 2) * BK * 2;   // 16 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kTmemCols = 2 * BN2;            // 512
constexpr uint32_t kSmemBytes = 1024 + kStages * kStageBytes + 256;

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
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
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

// Sched for pairs: tile(t) gives the pair tile (m0 = first of 256 rows, n0 = first of BN2
// columns, kb range); the core derives each CTA's A row (m0 + 128*rank) and B row
// (n0 + 64*... BN2/2*rank).  Epi::store gets the CTA-local row (0..127) and column chunk.
template <class Sched, class Epi>
__device__ __forceinline__ void gemm_core_pair(const CUtensorMap* tmA, const CUtensorMap* tmB, const Sched& sched,
                                               Epi& epi, ErrorRecord* err, uint64_t timeout_ns, int rank) {
  constexpr int S = kStages;
  extern __shared__ uint8_t gemm2_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm2_smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + S * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S * kStageBytes);
  uint64_t* empty = full + S;
  uint64_t* tfull = empty + S;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

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
      ptx::mbar_init(&tempty[a], 8);  // 4 epilogue warps x 2 CTAs
    }
    ptx::mbar_init(drain, 1);
    *abort_flag = 0;
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(tmA);
    ptx::prefetch_tmap(tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(tmem_slot, kTmemCols);
    tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // peer barriers initialised before any remote arrive / TMA completion
  ptx::tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int ntiles = sched.num_tiles();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- producer (both CTAs) ----------------
      int stage = 0;
      uint32_t phase = 0;
      uint32_t armed[S];
#pragma unroll
      for (int s = 0; s < S; ++s) armed[s] = 0;
      for (int t = pair_id; t < ntiles && !*abort_flag; t += npairs) {
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
          const uint32_t bar = map_to(ptx::smem_u32(&full[stage]), 0);
          if (leader) ptx::mbar_arrive_expect_tx(&full[stage], 2 * kStageBytes);
          tma_load_2d_pair(sA + stage * kABytes, tmA, bar, kb * BK, ti.a_row + (int)crank * BM);
          tma_load_2d_pair(sB + stage * kBBytes, tmB, bar, kb * BK, ti.b_row + (int)crank * (BN2 / 2));
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
      constexpr uint32_t idesc = ptx::idesc_bf16_f32(2 * BM, BN2);
      const uint32_t peer = 1;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool issued = false;
      for (int t = pair_id; t < ntiles && !*abort_flag; t += npairs) {
        TileInfo ti = sched.tile(t);
        if (!ptx::mbar_wait(&tempty[acc], acc_phase ^ 1, timeout_ns, abort_flag)) {
          if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, 0, 1, 0);
          *abort_flag = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem + acc * BN2;
        bool ok = true;
        for (int kb = ti.kb0; kb < ti.kb1; ++kb) {
          if (!ptx::mbar_wait(&full[stage], phase, timeout_ns, abort_flag)) {
            ok = false;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a0 = ptx::smem_u32(sA + stage * kABytes);
          const uint32_t b0 = ptx::smem_u32(sB + stage * kBBytes);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = ptx::sdesc_kmajor_sw128(a0 + k * 32);
            const uint64_t bd = ptx::sdesc_kmajor_sw128(b0 + k * 32);
            mma_pair(d, ad, bd, idesc, (kb > ti.kb0 || k > 0) ? 1u : 0u);
          }
          issued = true;
          const uint32_t e_own = ptx::smem_u32(&empty[stage]);
          commit_pair(e_own);
          commit_pair(map_to(e_own, peer));
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
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (*abort_flag && issued) {
        commit_pair(ptx::smem_u32(drain));
        ptx::mbar_wait(drain, 0, 20000000ull, nullptr);
      }
    }
  } else {
    // ---------------- epilogue (warps 2..5, both CTAs) ----------------
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t tempty_leader0 = map_to(ptx::smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = map_to(ptx::smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = pair_id; t < ntiles; t += npairs) {
      TileInfo ti = sched.tile(t);
      ti.m0 += (int)crank * BM;  // this CTA's 128 rows of the pair tile
      if (!ptx::mbar_wait(&tfull[acc], acc_phase, timeout_ns, abort_flag)) {
        if (!*abort_flag) report_error(err, GICC_ETIMEDOUT, W_GEMM_PIPE, rank, (int)crank, 3, 0);
        *abort_flag = 1;
        break;
      }
      ptx::tc_fence_after();
      const uint32_t tbase = tmem + (static_cast<uint32_t>(q * 32) << 16) + acc * BN2;
      epi.begin_tile(ti, row);
#pragma unroll 1
      for (int c = 0; c < BN2; c += 32) {
        uint32_t r[32];
        ptx::tmem_ld32(tbase + c, r);
        ptx::tmem_ld_wait();
        if (c + 32 >= BN2) {
          ptx::tc_fence_before();
          __syncwarp();
          if (lane == 0) arrive_cluster(acc ? tempty_leader1 : tempty_leader0);
        }
        epi.store(ti, row, c, r);
      }
      epi.end_tile(ti, row);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }
  ptx::tc_fence_before();
  __syncthreads();
  cluster_sync();  // the peer may still arrive on our barriers / the leader's MMAs write our TMEM
  if (warp == 1) {
    ptx::tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
}

}  // namespace pair
}  // namespace gemm
}  // namespace gicc
