/* gda.h -- the OpenGDA C API (gda_*) over the NVLink runtime.
 *
 * The reference ships examples written against an OpenGDA C API whose header is not in
 * its tree (examples/put_example.cpp, test_example.cpp, mr_example.cpp, gda_get_bw.cpp,
 * barrier_test.cpp, mm_hip_gda.cpp, mm_hip_gda_proxy*.cpp).  This header provides that API
 * surface, as gathered from those call sites, for one NVLink/NVSwitch node:
 *
 *   process   gda_init / gda_finalize / gda_rank / gda_size / gda_get_version / gda_barrier
 *   memory    gda_gpu_buf / gda_gpu_buf_size (a symmetric buffer allocated by gda_init),
 *             gda_register_memory / gda_mr_get_key / gda_mr_get_desc / gda_deregister_memory
 *   one-sided gda_put / gda_get create a deferred transfer whose device half
 *             (handle->gpu) is triggered from a kernel: gda_gpu_trigger (one thread),
 *             gda_gpu_trigger_all (the whole block) and gda_gpu_wait; the host tracks it
 *             with gda_wait / gda_test / gda_test_any / gda_test_all, gda_flush, gda_free
 *   barriers  gda_gpu_barrier_alloc / _reset / _free + device gda_gpu_barrier_wait;
 *             gda_proxy_barrier_* + device gda_gpu_proxy_barrier_wait
 *
 * Semantics on NVLink.  A transfer is performed by the triggering thread(s) with loads and
 * stores through the peer mapping of the target buffer (remote_offset is an offset into
 * the peer's gda_gpu_buf); completion is a release store of the handle's sequence number
 * into pinned host memory, so the host can test it.  No proxy thread is needed for the
 * "proxy" barrier -- NVLink signals carry epochs and never need re-arming -- so
 * gda_proxy_start / gda_proxy_stop are accepted and do nothing, and the proxy barrier is
 * the device barrier; its statistics report zero re-arms, polls and CQ events plus the
 * number of barriers completed.
 *
 * Every device wait is bounded (GICC_TIMEOUT_MS, default 5 s) and returns nonzero on
 * timeout instead of hanging.  Functions returning int return 0 on success, nonzero on
 * failure (and print the reason to stderr), except the gda_test* family (1 = complete).
 *
 * Environment: GDA_GPU_BUF_SIZE (bytes of the symmetric buffer, default 64 MiB), plus the
 * runtime's bootstrap variables (GICC_RANK / GICC_SIZE / GICC_BOOTSTRAP_ADDR or torchrun's).
 */
#ifndef GDA_H
#define GDA_H

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "gicc/types.hpp"

#ifdef __CUDACC__
#include "gicc/device/comm.cuh"
#endif

#define GDA_API extern "C" __attribute__((visibility("default")))

/* ---- types ---------------------------------------------------------------------------- */

/* Device half of a transfer: plain data, copied to device memory by the caller. */
typedef struct gda_gpu_handle {
  const void* src;        /* device-addressable source (local, or the peer mapping for a get) */
  void* dst;              /* device-addressable destination */
  uint64_t size;          /* bytes */
  uint64_t* completion;   /* pinned host word: last completed sequence number */
  uint64_t seq;           /* this transfer's sequence number */
  uint64_t timeout_ns;    /* bound of gda_gpu_wait */
} gda_gpu_handle_t;

typedef struct gda_handle {
  gda_gpu_handle_t gpu;   /* copy this to the device and trigger it from a kernel */
  int peer;
  int is_get;
  size_t remote_offset;
  int slot;               /* completion slot (internal) */
} gda_handle_t;

typedef struct gda_mr {
  void* addr;
  size_t size;
  int is_gpu;
  int index;              /* runtime buffer index */
  uint64_t key;           /* lkey == rkey == index on NVLink */
} gda_mr_t;

/* The device barrier: the runtime's BarrierCtx (copy it to device memory to use it). */
typedef struct gda_gpu_barrier {
  gicc::BarrierCtx ctx;
} gda_gpu_barrier_t;

typedef gda_gpu_barrier_t gda_proxy_barrier_dev_t;
typedef struct gda_proxy_barrier gda_proxy_barrier_t;

typedef struct gda_proxy_stats {
  uint64_t total_rearms;       /* always 0: NVLink signals never need re-arming */
  uint64_t queue_polls;        /* always 0: there is no proxy queue */
  uint64_t cq_events_drained;  /* always 0: there is no completion queue */
  uint64_t barriers_completed; /* barriers this rank completed */
} gda_proxy_stats_t;

/* ---- host API ------------------------------------------------------------------------- */

GDA_API int gda_init(void);
GDA_API void gda_finalize(void);
GDA_API int gda_rank(void);
GDA_API int gda_size(void);
GDA_API const char* gda_get_version(void);
GDA_API int gda_barrier(void);

GDA_API void* gda_gpu_buf(void);
GDA_API size_t gda_gpu_buf_size(void);

GDA_API gda_mr_t* gda_register_memory(void* buf, size_t size, int is_gpu);
GDA_API uint64_t gda_mr_get_key(gda_mr_t* mr);
GDA_API void* gda_mr_get_desc(gda_mr_t* mr);
GDA_API int gda_deregister_memory(gda_mr_t* mr);

GDA_API gda_handle_t* gda_put(const void* local, size_t size, int peer, size_t remote_offset);
GDA_API gda_handle_t* gda_get(void* local, size_t size, int peer, size_t remote_offset);
GDA_API int gda_wait(gda_handle_t* h);
GDA_API int gda_test(gda_handle_t* h);
GDA_API int gda_test_any(gda_handle_t** hs, int n, int* idx);
GDA_API int gda_test_all(gda_handle_t** hs, int n);
GDA_API int gda_flush(void);
GDA_API void gda_free(gda_handle_t* h);

GDA_API gda_gpu_barrier_t* gda_gpu_barrier_alloc(int max_iters);
GDA_API int gda_gpu_barrier_reset(gda_gpu_barrier_t* b);
GDA_API void gda_gpu_barrier_free(gda_gpu_barrier_t* b);

GDA_API gda_proxy_barrier_t* gda_proxy_barrier_alloc(int window_size);
GDA_API gda_proxy_barrier_dev_t* gda_proxy_barrier_get_dev(gda_proxy_barrier_t* b);
GDA_API int gda_proxy_start(gda_proxy_barrier_t* b);
GDA_API void gda_proxy_stop(gda_proxy_barrier_t* b);
GDA_API int gda_proxy_barrier_get_stats(gda_proxy_barrier_t* b, gda_proxy_stats_t* out);
GDA_API void gda_proxy_barrier_free(gda_proxy_barrier_t* b);

/* ---- device API ----------------------------------------------------------------------- */
#ifdef __CUDACC__

namespace gda_detail {
__device__ __forceinline__ void copy_range(const gda_gpu_handle_t& h, uint64_t first, uint64_t stride) {
  const uintptr_t s = reinterpret_cast<uintptr_t>(h.src), d = reinterpret_cast<uintptr_t>(h.dst);
  if (((s | d | h.size) & 15) == 0) {
    const uint4* src = reinterpret_cast<const uint4*>(h.src);
    uint4* dst = reinterpret_cast<uint4*>(h.dst);
    const uint64_t nv = h.size / 16;
    for (uint64_t i = first; i < nv; i += stride) gicc::ptx::st_v4(dst + i, gicc::ptx::ld_v4(src + i));
  } else {
    const uint8_t* src = static_cast<const uint8_t*>(h.src);
    uint8_t* dst = static_cast<uint8_t*>(h.dst);
    for (uint64_t i = first; i < h.size; i += stride) dst[i] = src[i];
  }
}
__device__ __forceinline__ void complete(const gda_gpu_handle_t& h) {
  gicc::ptx::fence_acq_rel_sys();
  gicc::ptx::st_release_sys(h.completion, h.seq);
}
}  // namespace gda_detail

/* Perform the transfer with the calling thread, then publish its completion. */
__device__ __forceinline__ void gda_gpu_trigger(gda_gpu_handle_t h) {
  gda_detail::copy_range(h, 0, 1);
  gda_detail::complete(h);
}

/* Perform the transfer with every thread of the block (all must call it). */
__device__ __forceinline__ void gda_gpu_trigger_all(gda_gpu_handle_t h) {
  const uint64_t nthreads = (uint64_t)blockDim.x * blockDim.y * blockDim.z;
  const uint64_t tid = threadIdx.x + (uint64_t)blockDim.x * (threadIdx.y + (uint64_t)blockDim.y * threadIdx.z);
  gda_detail::copy_range(h, tid, nthreads);
  gicc::ptx::fence_acq_rel_sys();
  __syncthreads();
  if (tid == 0) gda_detail::complete(h);
}

/* Bounded wait until the transfer completed; 0 or GICC_ETIMEDOUT. */
__device__ __forceinline__ int gda_gpu_wait(gda_gpu_handle_t h) {
  uint64_t seen = 0;
  return gicc::proto::wait_until<gicc::proto::DevMem>(h.completion, gicc::proto::CMP_GE, h.seq, h.timeout_ns, &seen)
             ? 0
             : (int)gicc::GICC_ETIMEDOUT;
}

/* One barrier across all ranks (one thread; the epoch advances in the caller's copy). */
__device__ __forceinline__ int gda_gpu_barrier_wait(gda_gpu_barrier_t* b) {
  const int st = gicc::barrier(&b->ctx);
  b->ctx.expected_signal += 1;
  return st;
}

__device__ __forceinline__ int gda_gpu_proxy_barrier_wait(gda_proxy_barrier_dev_t* b) { return gda_gpu_barrier_wait(b); }

#endif /* __CUDACC__ */
#endif /* GDA_H */
