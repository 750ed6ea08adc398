// collectives.cu -- allreduce (one-shot, two-shot, NVLS) fused with scale/cast, standalone
// reduce-scatter and all-gather (NVLS or direct NVLink), and a multi-source reduction used
// by GEMM->reduce-scatter.  Every call's epoch is either a kernel argument or, for CUDA-graph
// capture, a device word that the call reads and its last CTA advances.
//
// None of these exists in the reference (its only reduction is the host scalar
// coll::allreduce_sum over MPI, src/gicc/coll.hpp:15-21).  Design:
//   * inputs live in symmetric memory, so every rank reads its peers' data directly;
//   * no separate barrier kernel: every CTA does an entry and an exit handshake with
//     the CTA of the same index on every peer (epoch-valued flags in the signal heap,
//     release stores / acquire polls, bounded by %globaltimer).  CTA b of every rank
//     touches the same element range, so the pairwise handshake is all that is needed;
//   * bf16 data is summed in f32 registers (fixed source order, so every rank gets the
//     same bits), scaled, and written as bf16 or f32;
//   * every thread keeps kU 16-byte vectors (x up to 8 sources) in flight per step, so
//     NVLink latency is covered by memory-level parallelism;
//   * NVLS: multimem.ld_reduce sums all ranks' copies inside the NVSwitch, multimem.st
//     broadcasts the result -- each GPU moves 1/n of the bytes once in each direction.
#include <cuda_runtime.h>

#include "gicc/device/comm.cuh"
#include "gicc/config.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"

namespace gicc {
namespace {

constexpr int kMaxRanks = 8;  // one NVSwitch node
constexpr int kU = 4;         // vectors per thread per step

struct PeerPtrs {
  const void* p[kMaxRanks];
};
struct PeerOut {
  void* p[kMaxRanks];
};
struct FlagPtrs {
  uint64_t* p[kMaxRanks];  // each rank's flag area base (this rank's view)
};
// Where a call's epoch comes from.  dev == null: the host passes it (value).  Otherwise the
// epoch is *dev + 1, read by every CTA at its start, and the last CTA to finish stores it
// back (and re-arms the ticket): a captured CUDA graph then uses a new epoch on every replay.
struct EpochRef {
  uint64_t value;
  uint64_t* dev;
  unsigned int* ticket;
};

__device__ __forceinline__ uint64_t call_epoch(const EpochRef& e) {
  __shared__ uint64_t ep;
  if (threadIdx.x == 0) ep = e.dev ? *reinterpret_cast<volatile uint64_t*>(e.dev) + 1 : e.value;
  __syncthreads();
  return ep;
}
__device__ __forceinline__ void finish_epoch(const EpochRef& e, uint64_t ep) {
  if (!e.dev) return;
  __syncthreads();
  if (threadIdx.x == 0 && atomicAdd(e.ticket, 1u) + 1 == gridDim.x) {
    *e.ticket = 0;  // every CTA of this call has counted; the next call starts after this kernel
    *reinterpret_cast<volatile uint64_t*>(e.dev) = ep;
  }
}

__device__ __forceinline__ void add_bf16x8(float* acc, const uint4& v) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] += ptx::bf16_lo(w[j]);
    acc[2 * j + 1] += ptx::bf16_hi(w[j]);
  }
}

__device__ __forceinline__ void store8(void* out, size_t vec, const float* acc, float scale, int out_f32) {
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(out) + 2 * vec;
    o[0] = make_float4(acc[0] * scale, acc[1] * scale, acc[2] * scale, acc[3] * scale);
    o[1] = make_float4(acc[4] * scale, acc[5] * scale, acc[6] * scale, acc[7] * scale);
  } else {
    uint4 r;
    r.x = ptx::pack_bf16x2(acc[0] * scale, acc[1] * scale);
    r.y = ptx::pack_bf16x2(acc[2] * scale, acc[3] * scale);
    r.z = ptx::pack_bf16x2(acc[4] * scale, acc[5] * scale);
    r.w = ptx::pack_bf16x2(acc[6] * scale, acc[7] * scale);
    reinterpret_cast<uint4*>(out)[vec] = r;
  }
}

// Pairwise handshake of CTA `blockIdx.x` with the same CTA on every peer.
// flags layout (per rank): [phase][block][src] words.
__device__ __forceinline__ int cta_handshake(const FlagPtrs& flags, int n, int me, int phase, int max_blocks,
                                             uint64_t epoch, uint64_t timeout_ns, ErrorRecord* err) {
  __shared__ int st;
  ptx::fence_acq_rel_sys();
  __syncthreads();
  if (threadIdx.x == 0) st = GICC_OK;
  __syncthreads();
  const size_t slot = ((size_t)phase * max_blocks + blockIdx.x) * n;
  const int t = threadIdx.x;
  if (t < n && t != me) {
    ptx::st_release_sys(flags.p[t] + slot + me, epoch);
    uint64_t seen = 0;
    if (!proto::wait_until<proto::DevMem>(flags.p[me] + slot + t, proto::CMP_GE, epoch, timeout_ns, &seen)) {
      report_error(err, GICC_ETIMEDOUT, W_ALLREDUCE, me, t, seen, epoch);
      st = GICC_ETIMEDOUT;
    }
  }
  __syncthreads();
  return st;
}

// Reduce vectors [lo, hi) of the n inputs; hand each finished vector to `emit(vec, acc)`.
template <class Emit>
__device__ __forceinline__ void reduce_range(const PeerPtrs& in, int n, size_t lo, size_t hi, Emit emit) {
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  size_t v = lo + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; v + (kU - 1) * stride < hi; v += kU * stride) {
    uint4 x[kU][kMaxRanks];
#pragma unroll
    for (int u = 0; u < kU; ++u)
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < n) x[u][p] = reinterpret_cast<const uint4*>(in.p[p])[v + u * stride];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < n) add_bf16x8(acc, x[u][p]);
      emit(v + u * stride, acc);
    }
  }
  for (; v < hi; v += stride) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int p = 0; p < kMaxRanks; ++p)
      if (p < n) add_bf16x8(acc, reinterpret_cast<const uint4*>(in.p[p])[v]);
    emit(v, acc);
  }
}

// One-shot: every rank reads all inputs and writes the whole result locally.
__global__ void __launch_bounds__(256) k_allreduce_oneshot(PeerPtrs in, void* out, size_t nvec, int n, int me,
                                                           float scale, int out_f32, FlagPtrs flags, int max_blocks,
                                                           EpochRef er, uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    reduce_range(in, n, 0, nvec, [&](size_t v, const float* acc) { store8(out, v, acc, scale, out_f32); });
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);
  }
  finish_epoch(er, epoch);
}

// Two-shot: rank r reduces chunk r from all inputs and pushes it into every rank's output.
__global__ void __launch_bounds__(256) k_allreduce_twoshot(PeerPtrs in, PeerOut out, size_t nvec, int n, int me,
                                                           float scale, int out_f32, FlagPtrs flags, int max_blocks,
                                                           EpochRef er, uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    const size_t per = (nvec + n - 1) / n;
    const size_t lo = per * me, hi = lo + per < nvec ? lo + per : nvec;
    reduce_range(in, n, lo, hi, [&](size_t v, const float* acc) {
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < n) store8(out.p[(me + p) % n], v, acc, scale, out_f32);
    });
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);
  }
  finish_epoch(er, epoch);
}

__device__ __forceinline__ void nvls_emit(void* mc_out, size_t v, uint4 s, float scale, int out_f32) {
  if (out_f32) {
    float acc[8];
    const uint32_t w[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      acc[2 * j] = ptx::bf16_lo(w[j]) * scale;
      acc[2 * j + 1] = ptx::bf16_hi(w[j]) * scale;
    }
    uint4* o = reinterpret_cast<uint4*>(mc_out) + 2 * v;
    ptx::multimem_st_v4(o, make_uint4(__float_as_uint(acc[0]), __float_as_uint(acc[1]), __float_as_uint(acc[2]),
                                      __float_as_uint(acc[3])));
    ptx::multimem_st_v4(o + 1, make_uint4(__float_as_uint(acc[4]), __float_as_uint(acc[5]), __float_as_uint(acc[6]),
                                          __float_as_uint(acc[7])));
  } else {
    uint4 r = s;
    if (scale != 1.0f) {
      const uint32_t w[4] = {s.x, s.y, s.z, s.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) o[j] = ptx::pack_bf16x2(ptx::bf16_lo(w[j]) * scale, ptx::bf16_hi(w[j]) * scale);
      r = make_uint4(o[0], o[1], o[2], o[3]);
    }
    ptx::multimem_st_v4(reinterpret_cast<uint4*>(mc_out) + v, r);
  }
}

// NVLS: rank r reduces chunk r inside the switch and multicasts the result.
__global__ void __launch_bounds__(512) k_allreduce_nvls(const void* mc_in, void* mc_out, size_t nvec, int n, int me,
                                                        float scale, int out_f32, FlagPtrs flags, int max_blocks,
                                                        EpochRef er, uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) != GICC_OK) {
    finish_epoch(er, epoch);
    return;
  }
  const size_t per = (nvec + n - 1) / n;
  const size_t lo = per * me, hi = lo + per < nvec ? lo + per : nvec;
  const size_t stride = (size_t)gridDim.x * blockDim.x;
  const uint4* src = reinterpret_cast<const uint4*>(mc_in);
  size_t v = lo + (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  constexpr int U = 2 * kU;
  for (; v + (U - 1) * stride < hi; v += U * stride) {
    uint4 s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) s[u] = ptx::multimem_ld_reduce_bf16x8(src + v + u * stride);
#pragma unroll
    for (int u = 0; u < U; ++u) nvls_emit(mc_out, v + u * stride, s[u], scale, out_f32);
  }
  for (; v < hi; v += stride) nvls_emit(mc_out, v, ptx::multimem_ld_reduce_bf16x8(src + v), scale, out_f32);
  cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);
  finish_epoch(er, epoch);
}

// Reduce-scatter: rank r ends with chunk r of the sum, out[v - lo] for v in [lo, hi).
// Direct: CTAs read every rank's input over NVLink; NVLS: the switch adds the copies.
__global__ void __launch_bounds__(256) k_reduce_scatter(PeerPtrs in, void* out, size_t nvec, int n, int me,
                                                        float scale, int out_f32, FlagPtrs flags, int max_blocks,
                                                        EpochRef er, uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    const size_t per = nvec / n, lo = per * me;
    reduce_range(in, n, lo, lo + per, [&](size_t v, const float* acc) { store8(out, v - lo, acc, scale, out_f32); });
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);  // inputs may be rewritten after this
  }
  finish_epoch(er, epoch);
}

__global__ void __launch_bounds__(512) k_reduce_scatter_nvls(const void* mc_in, void* out, size_t nvec, int n, int me,
                                                             float scale, int out_f32, FlagPtrs flags, int max_blocks,
                                                             EpochRef er, uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    const size_t per = nvec / n, lo = per * me;
    const uint4* src = reinterpret_cast<const uint4*>(mc_in);
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    constexpr int U = 2 * kU;
    for (; v + (U - 1) * stride < per; v += U * stride) {
      uint4 t[U];
#pragma unroll
      for (int u = 0; u < U; ++u) t[u] = ptx::multimem_ld_reduce_bf16x8(src + lo + v + u * stride);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        add_bf16x8(acc, t[u]);
        store8(out, v + u * stride, acc, scale, out_f32);
      }
    }
    for (; v < per; v += stride) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      add_bf16x8(acc, ptx::multimem_ld_reduce_bf16x8(src + lo + v));
      store8(out, v, acc, scale, out_f32);
    }
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);
  }
  finish_epoch(er, epoch);
}

// All-gather of 16-byte vectors: rank r's shard goes to [r*per, (r+1)*per) of every rank's
// output.  Direct: one store per peer; NVLS: one multimem store reaches every GPU.
__global__ void __launch_bounds__(256) k_all_gather(const uint4* shard, PeerOut out, size_t per, int n, int me,
                                                    FlagPtrs flags, int max_blocks, EpochRef er, uint64_t timeout_ns,
                                                    ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < per; v += stride) {
      const uint4 x = shard[v];
#pragma unroll
      for (int p = 0; p < kMaxRanks; ++p)
        if (p < n) reinterpret_cast<uint4*>(out.p[(me + p) % n])[(size_t)me * per + v] = x;
    }
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);  // every shard has landed here
  }
  finish_epoch(er, epoch);
}

__global__ void __launch_bounds__(512) k_all_gather_nvls(const uint4* shard, void* mc_out, size_t per, int n, int me,
                                                         FlagPtrs flags, int max_blocks, EpochRef er,
                                                         uint64_t timeout_ns, ErrorRecord* err) {
  const uint64_t epoch = call_epoch(er);
  if (cta_handshake(flags, n, me, 0, max_blocks, epoch, timeout_ns, err) == GICC_OK) {
    const size_t stride = (size_t)gridDim.x * blockDim.x;
    uint4* dst = reinterpret_cast<uint4*>(mc_out) + (size_t)me * per;
    for (size_t v = (size_t)blockIdx.x * blockDim.x + threadIdx.x; v < per; v += stride)
      ptx::multimem_st_v4(dst + v, shard[v]);
    cta_handshake(flags, n, me, 1, max_blocks, epoch, timeout_ns, err);
  }
  finish_epoch(er, epoch);
}

// Plain multi-source reduction (callers order it with barriers): out = scale * sum(src).
__global__ void __launch_bounds__(256) k_reduce(PeerPtrs src, int nsrc, void* out, size_t nvec, float scale,
                                                int out_f32) {
  reduce_range(src, nsrc, 0, nvec, [&](size_t v, const float* acc) { store8(out, v, acc, scale, out_f32); });
}

}  // namespace

namespace ops {

void reduce_bf16(const void* const* srcs, int nsrc, void* out, size_t count, float scale, bool out_f32,
                 cudaStream_t s) {
  if (nsrc < 1 || nsrc > kMaxRanks) throw std::runtime_error("gicc::reduce_bf16: 1..8 sources");
  if (count % 8) throw std::runtime_error("gicc::reduce_bf16: count must be a multiple of 8");
  PeerPtrs p{};
  for (int i = 0; i < nsrc; ++i) {
    if (reinterpret_cast<uintptr_t>(srcs[i]) & 15) throw std::runtime_error("gicc::reduce_bf16: unaligned source");
    p.p[i] = srcs[i];
  }
  const size_t nvec = count / 8;
  int blocks = (int)std::min<size_t>(std::max<size_t>((nvec + 256 * kU - 1) / (256 * kU), 1), 4 * (size_t)num_sms());
  k_reduce<<<blocks, 256, 0, s>>>(p, nsrc, out, nvec, scale, out_f32 ? 1 : 0);
  GICC_CUDA(cudaGetLastError());
}

void allreduce_bf16(int algo, const void* const* in, void* const* out, const void* mc_in, void* mc_out, int n, int me,
                    size_t count, float scale, bool out_f32, uint64_t* const* flag_bases, int max_blocks,
                    uint64_t epoch, uint64_t timeout_ns, int blocks, cudaStream_t s, uint64_t* epoch_dev,
                    unsigned int* ticket) {
  if (epoch_dev && !ticket) throw std::runtime_error("gicc::allreduce: a device epoch needs a ticket word");
  NvtxRange nvtx("gicc::ops::allreduce_bf16");
  if (n < 1 || n > kMaxRanks) throw std::runtime_error("gicc::allreduce: 1..8 ranks (one NVSwitch node)");
  if (count % 8) throw std::runtime_error("gicc::allreduce: element count must be a multiple of 8");
  const size_t nvec = count / 8;
  PeerPtrs ip{};
  PeerOut op{};
  FlagPtrs fp{};
  for (int i = 0; i < n; ++i) {
    ip.p[i] = in ? in[i] : nullptr;
    op.p[i] = out ? out[i] : nullptr;
    fp.p[i] = flag_bases[i];
  }
  const size_t work = algo == ALLREDUCE_ONESHOT ? nvec : (nvec + n - 1) / n;
  if (blocks <= 0) {
    // Never more CTAs than can be resident at once: every CTA handshakes with its peers'
    // CTA of the same index, so a second wave would run in lock-step across GPUs.
    int per_sm = 1;
    const void* fn = algo == ALLREDUCE_ONESHOT   ? (const void*)k_allreduce_oneshot
                     : algo == ALLREDUCE_TWOSHOT ? (const void*)k_allreduce_twoshot
                                                 : (const void*)k_allreduce_nvls;
    const int threads = algo == ALLREDUCE_NVLS ? 512 : 256;
    GICC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0));
    const size_t resident = (size_t)std::max(per_sm, 1) * num_sms();
    blocks = (int)std::min<size_t>(std::max<size_t>((work + threads * kU - 1) / (threads * kU), 1), resident);
  }
  if (blocks > max_blocks) blocks = max_blocks;
  ErrorRecord* err = device_error_record();
  const EpochRef er{epoch, epoch_dev, ticket};
  switch (algo) {
    case ALLREDUCE_ONESHOT:
      k_allreduce_oneshot<<<blocks, 256, 0, s>>>(ip, op.p[me], nvec, n, me, scale, out_f32, fp, max_blocks, er,
                                                 timeout_ns, err);
      break;
    case ALLREDUCE_TWOSHOT:
      k_allreduce_twoshot<<<blocks, 256, 0, s>>>(ip, op, nvec, n, me, scale, out_f32, fp, max_blocks, er,
                                                 timeout_ns, err);
      break;
    case ALLREDUCE_NVLS:
      if (!mc_in || !mc_out) throw std::runtime_error("gicc::allreduce: NVLS needs multicast-bound buffers");
      k_allreduce_nvls<<<blocks, 512, 0, s>>>(mc_in, mc_out, nvec, n, me, scale, out_f32, fp, max_blocks, er,
                                              timeout_ns, err);
      break;
    default:
      throw std::runtime_error("gicc::allreduce: unknown algorithm");
  }
  GICC_CUDA(cudaGetLastError());
}

namespace {
int resident_blocks(const void* fn, int threads, size_t work) {
  int per_sm = 1;
  GICC_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, 0));
  const size_t resident = (size_t)std::max(per_sm, 1) * num_sms();
  return (int)std::min<size_t>(std::max<size_t>((work + threads * kU - 1) / (threads * kU), 1), resident);
}
}  // namespace

void reduce_scatter_bf16(bool nvls, const void* const* in, const void* mc_in, void* out, int n, int me, size_t count,
                         float scale, bool out_f32, uint64_t* const* flag_bases, int max_blocks, uint64_t epoch,
                         uint64_t timeout_ns, int blocks, cudaStream_t s, uint64_t* epoch_dev, unsigned int* ticket) {
  NvtxRange nvtx("gicc::ops::reduce_scatter_bf16");
  if (n < 1 || n > kMaxRanks) throw std::runtime_error("gicc::reduce_scatter: 1..8 ranks");
  if (count % (8 * (size_t)n)) throw std::runtime_error("gicc::reduce_scatter: count must be a multiple of 8 * ranks");
  if (epoch_dev && !ticket) throw std::runtime_error("gicc::reduce_scatter: a device epoch needs a ticket word");
  const size_t nvec = count / 8;
  PeerPtrs ip{};
  FlagPtrs fp{};
  for (int i = 0; i < n; ++i) {
    ip.p[i] = in ? in[i] : nullptr;
    fp.p[i] = flag_bases[i];
  }
  const EpochRef er{epoch, epoch_dev, ticket};
  ErrorRecord* err = device_error_record();
  if (nvls) {
    if (!mc_in) throw std::runtime_error("gicc::reduce_scatter: NVLS needs a multicast-bound input");
    if (blocks <= 0) blocks = resident_blocks((const void*)k_reduce_scatter_nvls, 512, nvec / n);
    blocks = std::min(blocks, max_blocks);
    k_reduce_scatter_nvls<<<blocks, 512, 0, s>>>(mc_in, out, nvec, n, me, scale, out_f32, fp, max_blocks, er,
                                                 timeout_ns, err);
  } else {
    if (blocks <= 0) blocks = resident_blocks((const void*)k_reduce_scatter, 256, nvec / n);
    blocks = std::min(blocks, max_blocks);
    k_reduce_scatter<<<blocks, 256, 0, s>>>(ip, out, nvec, n, me, scale, out_f32, fp, max_blocks, er, timeout_ns,
                                            err);
  }
  GICC_CUDA(cudaGetLastError());
}

void all_gather(bool nvls, const void* shard, void* const* out, void* mc_out, int n, int me, size_t shard_bytes,
                uint64_t* const* flag_bases, int max_blocks, uint64_t epoch, uint64_t timeout_ns, int blocks,
                cudaStream_t s, uint64_t* epoch_dev, unsigned int* ticket) {
  NvtxRange nvtx("gicc::ops::all_gather");
  if (n < 1 || n > kMaxRanks) throw std::runtime_error("gicc::all_gather: 1..8 ranks");
  if (shard_bytes % 16 || (reinterpret_cast<uintptr_t>(shard) & 15))
    throw std::runtime_error("gicc::all_gather: 16-byte aligned shard of a multiple of 16 bytes");
  if (epoch_dev && !ticket) throw std::runtime_error("gicc::all_gather: a device epoch needs a ticket word");
  const size_t per = shard_bytes / 16;
  PeerOut op{};
  FlagPtrs fp{};
  for (int i = 0; i < n; ++i) {
    op.p[i] = out ? out[i] : nullptr;
    fp.p[i] = flag_bases[i];
  }
  const EpochRef er{epoch, epoch_dev, ticket};
  ErrorRecord* err = device_error_record();
  const uint4* src = static_cast<const uint4*>(shard);
  if (nvls) {
    if (!mc_out) throw std::runtime_error("gicc::all_gather: NVLS needs a multicast-bound output");
    if (blocks <= 0) blocks = resident_blocks((const void*)k_all_gather_nvls, 512, per);
    blocks = std::min(blocks, max_blocks);
    k_all_gather_nvls<<<blocks, 512, 0, s>>>(src, mc_out, per, n, me, fp, max_blocks, er, timeout_ns, err);
  } else {
    if (blocks <= 0) blocks = resident_blocks((const void*)k_all_gather, 256, per * n);
    blocks = std::min(blocks, max_blocks);
    k_all_gather<<<blocks, 256, 0, s>>>(src, op, per, n, me, fp, max_blocks, er, timeout_ns, err);
  }
  GICC_CUDA(cudaGetLastError());
}

}  // namespace ops
}  // namespace gicc
