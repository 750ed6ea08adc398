// errors.cpp -- the per-device error record shared by every kernel of the library.
//
// The record lives in device memory (device atomics pick the first error); the host
// copies it back after a synchronize.  One record per device, allocated on first use.
#include "gicc/config.hpp"
#include "gicc/error.hpp"

#include <cuda_runtime.h>

#include <cstdlib>
#include <cstring>
#include <mutex>
#include <stdexcept>
#include <string>

namespace gicc {

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
ErrorRecord* g_dev[kMaxDevices] = {};

int current_device() {
  int d = 0;
  cudaError_t e = cudaGetDevice(&d);
  if (e != cudaSuccess) throw std::runtime_error(std::string("gicc: cudaGetDevice: ") + cudaGetErrorString(e));
  if (d < 0 || d >= kMaxDevices) throw std::runtime_error("gicc: device index out of range");
  return d;
}
}  // namespace

ErrorRecord* device_error_record() {
  const int d = current_device();
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_dev[d]) return g_dev[d];
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, sizeof(ErrorRecord));
  if (e != cudaSuccess) throw std::runtime_error(std::string("gicc: cudaMalloc(error record): ") + cudaGetErrorString(e));
  e = cudaMemset(p, 0, sizeof(ErrorRecord));
  if (e != cudaSuccess) throw std::runtime_error(std::string("gicc: cudaMemset(error record): ") + cudaGetErrorString(e));
  g_dev[d] = static_cast<ErrorRecord*>(p);
  return g_dev[d];
}

ErrorRecord read_error_record(bool clear) {
  ErrorRecord r{};
  const int d = current_device();
  ErrorRecord* p = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    p = g_dev[d];
  }
  if (!p) return r;
  cudaError_t e = cudaMemcpy(&r, p, sizeof(r), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) throw std::runtime_error(std::string("gicc: reading error record: ") + cudaGetErrorString(e));
  if (clear && r.count != 0) {
    e = cudaMemset(p, 0, sizeof(ErrorRecord));
    if (e != cudaSuccess) throw std::runtime_error(std::string("gicc: clearing error record: ") + cudaGetErrorString(e));
  }
  return r;
}

const char* status_name(int code) {
  switch (code) {
    case GICC_OK: return "OK";
    case GICC_ETIMEDOUT: return "ETIMEDOUT";
    case GICC_EINVAL: return "EINVAL";
    case GICC_ERANGE: return "ERANGE";
    case GICC_EPEER: return "EPEER";
    case GICC_ECUDA: return "ECUDA";
    case GICC_EBOOT: return "EBOOT";
    case GICC_EMISMATCH: return "EMISMATCH";
    case GICC_ENOMEM: return "ENOMEM";
    case GICC_EUNSUPPORTED: return "EUNSUPPORTED";
  }
  return "UNKNOWN";
}

const char* where_name(int w) {
  switch (w) {
    case W_NONE: return "none";
    case W_SIGNAL_WAIT: return "signal_wait";
    case W_BARRIER: return "barrier";
    case W_GEMM_PIPE: return "gemm_pipeline";
    case W_AG_FLAG: return "ag_gemm_chunk_flag";
    case W_RS_FLAG: return "gemm_rs_flag";
    case W_MOE_COUNT: return "moe_arrival";
    case W_AM_WAIT: return "am_wait";
    case W_ALLREDUCE: return "allreduce";
    case W_JACOBI_HALO: return "jacobi_halo";
    case W_QUIET: return "quiet";
    case W_BOUNDS: return "bounds";
    case W_PINGPONG: return "pingpong";
    case W_RING_MM: return "ring matmul";
  }
  return "?";
}

uint64_t default_timeout_ns() { return config().timeout_ms * 1000000ull; }

}  // namespace gicc
