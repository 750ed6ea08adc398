// error.hpp -- status codes and the device-visible error record.
//
// Every bounded device wait in this library (flag waits, barriers, mbarrier pipelines,
// MoE arrival counters, AG-GEMM chunk flags) ends with a status instead of a trap: the
// first failing thread writes an ErrorRecord (one per device, in device memory) and the
// kernel returns.  The host copies the record back after a synchronize and raises.
// The reference's device waits either spin forever (platform/mlx5/device_opt.cuh:505-519)
// or return -2/-1 codes (device_opt.cuh:476-481; examples/barrier_test.cpp:53-60);
// this is the same idea made uniform.
#pragma once
#include <cstdint>

namespace gicc {

enum Status : int {
  GICC_OK = 0,
  GICC_ETIMEDOUT = 1,   // a bounded wait ran out of time
  GICC_EINVAL = 2,      // bad argument (size, alignment, peer index)
  GICC_ERANGE = 3,      // access outside a registered region (GICC_CHECKS builds)
  GICC_EPEER = 4,       // a peer reported failure / left
  GICC_ECUDA = 5,       // a CUDA runtime/driver call failed
  GICC_EBOOT = 6,       // bootstrap (socket KVS) failure
  GICC_EMISMATCH = 7,   // collective metadata differs across ranks
  GICC_ENOMEM = 8,
  GICC_EUNSUPPORTED = 9,
};

// Where a device-side error was raised (ErrorRecord::where).
enum Where : int {
  W_NONE = 0,
  W_SIGNAL_WAIT = 1,
  W_BARRIER = 2,
  W_GEMM_PIPE = 3,
  W_AG_FLAG = 4,
  W_RS_FLAG = 5,
  W_MOE_COUNT = 6,
  W_AM_WAIT = 7,
  W_ALLREDUCE = 8,
  W_JACOBI_HALO = 9,
  W_QUIET = 10,
  W_BOUNDS = 11,
  W_PINGPONG = 12,
  W_RING_MM = 13,
};

struct ErrorRecord {
  int code;       // first error's Status (0 = none)
  int where;      // Where
  int rank;
  int peer;
  unsigned long long value;     // observed value at the failing wait
  unsigned long long expected;  // value waited for
  unsigned long long count;     // number of errors raised since the last clear
};

#if defined(__CUDACC__)
__device__ __forceinline__ void report_error(ErrorRecord* e, int code, int where, int rank, int peer,
                                             unsigned long long value, unsigned long long expected) {
  if (e == nullptr) return;
  if (atomicCAS(&e->code, 0, code) == 0) {
    e->where = where;
    e->rank = rank;
    e->peer = peer;
    e->value = value;
    e->expected = expected;
    __threadfence_system();
  }
  atomicAdd(&e->count, 1ull);
}
#endif

// Host side (errors.cpp): one record per device, allocated on first use.
#define GICC_VIS __attribute__((visibility("default")))
GICC_VIS ErrorRecord* device_error_record();  // device-usable pointer (allocated on first use)
GICC_VIS ErrorRecord read_error_record(bool clear);
GICC_VIS const char* status_name(int code);
GICC_VIS const char* where_name(int where);

// Default bound for device waits, from GICC_TIMEOUT_MS (default 5000 ms).
GICC_VIS uint64_t default_timeout_ns();

}  // namespace gicc
