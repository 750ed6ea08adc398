// mem.hpp -- memory-ordering policies shared by the device kernels and the CPU test path.
//
// The flag protocols (signal wait, dissemination barrier, active-message rings) are
// written once as templates over a Mem policy:
//   * DevMem  -- PTX acquire/release at .sys scope and %globaltimer (GPU, NVLink peers);
//   * HostMem -- C++ __atomic builtins and CLOCK_MONOTONIC (CPU ranks over shared memory,
//                the "fake device" used by the CPU test-suite).
// So the CPU tests exercise exactly the protocol code that runs on the GPU.
#pragma once
#include <cstdint>

#if defined(__CUDACC__)
#define GICC_HD __host__ __device__ __forceinline__
// Before a protocol template: each instantiation runs on one side only (DevMem on the GPU,
// HostMem on the CPU), so nvcc's check that a host-device function calls host-device code
// does not apply.
#define GICC_PROTO_TEMPLATE _Pragma("nv_exec_check_disable") template <class Mem>
#else
#define GICC_HD inline
#define GICC_PROTO_TEMPLATE template <class Mem>
#endif

#if !defined(__CUDA_ARCH__)
#include <sched.h>
#include <time.h>
#endif

namespace gicc {
namespace proto {

enum Cmp : int { CMP_EQ = 0, CMP_NE = 1, CMP_GE = 2, CMP_GT = 3, CMP_LT = 4, CMP_LE = 5 };

GICC_HD bool cmp_ok(uint64_t v, int cmp, uint64_t x) {
  switch (cmp) {
    case CMP_EQ: return v == x;
    case CMP_NE: return v != x;
    case CMP_GE: return v >= x;
    case CMP_GT: return v > x;
    case CMP_LT: return v < x;
    default: return v <= x;
  }
}

#if defined(__CUDACC__)
struct DevMem {
  static __device__ __forceinline__ uint64_t load_acquire(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
  }
  static __device__ __forceinline__ uint64_t load_relaxed(const uint64_t* p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
  }
  static __device__ __forceinline__ void store_release(uint64_t* p, uint64_t v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
  }
  static __device__ __forceinline__ void add_release(uint64_t* p, uint64_t v) {
    asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
  }
  static __device__ __forceinline__ void store_relaxed(uint64_t* p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
  }
  static __device__ __forceinline__ void fence() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
  static __device__ __forceinline__ void fence_sc() { asm volatile("fence.sc.sys;" ::: "memory"); }
  static __device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
  }
  static __device__ __forceinline__ void relax() {}
};
#endif

struct HostMem {
  static inline uint64_t load_acquire(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_ACQUIRE); }
  static inline uint64_t load_relaxed(const uint64_t* p) { return __atomic_load_n(p, __ATOMIC_RELAXED); }
  static inline void store_release(uint64_t* p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELEASE); }
  static inline void add_release(uint64_t* p, uint64_t v) { __atomic_fetch_add(p, v, __ATOMIC_RELEASE); }
  static inline void store_relaxed(uint64_t* p, uint64_t v) { __atomic_store_n(p, v, __ATOMIC_RELAXED); }
  static inline void fence() { __atomic_thread_fence(__ATOMIC_SEQ_CST); }
  static inline void fence_sc() { __atomic_thread_fence(__ATOMIC_SEQ_CST); }
#if !defined(__CUDA_ARCH__)
  static inline uint64_t now_ns() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (uint64_t)ts.tv_sec * 1000000000ull + (uint64_t)ts.tv_nsec;
  }
  static inline void relax() { sched_yield(); }
#else
  static inline uint64_t now_ns() { return 0; }
  static inline void relax() {}
#endif
};

// Wait until cmp(*p, x) holds (acquire), at most timeout_ns.  Returns the last value seen
// through *seen and true on success.
GICC_PROTO_TEMPLATE
GICC_HD bool wait_until(const uint64_t* p, int cmp, uint64_t x, uint64_t timeout_ns, uint64_t* seen) {
  uint64_t v = Mem::load_acquire(p);
  if (cmp_ok(v, cmp, x)) {
    if (seen) *seen = v;
    return true;
  }
  const uint64_t t0 = Mem::now_ns();
  for (uint32_t i = 1;; ++i) {
    v = Mem::load_acquire(p);
    if (cmp_ok(v, cmp, x)) {
      if (seen) *seen = v;
      return true;
    }
    if ((i & 31) == 0) {
      if (Mem::now_ns() - t0 > timeout_ns) {
        if (seen) *seen = v;
        return false;
      }
      Mem::relax();
    }
  }
}

}  // namespace proto
}  // namespace gicc
