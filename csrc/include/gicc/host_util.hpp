// host_util.hpp -- small host helpers shared by the native library: CUDA error checks,
// device properties and TMA tensor-map construction.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <stdexcept>
#include <string>

#include "gicc/driver.hpp"
#include "gicc/visibility.hpp"

namespace gicc {

[[noreturn]] inline void throw_cuda(const char* what, cudaError_t e, const char* file, int line) {
  throw std::runtime_error(std::string("gicc: ") + what + " failed: " + cudaGetErrorString(e) + " (" + file + ":" +
                           std::to_string(line) + ")");
}

#define GICC_CUDA(x)                                                   \
  do {                                                                 \
    cudaError_t _e = (x);                                              \
    if (_e != cudaSuccess) ::gicc::throw_cuda(#x, _e, __FILE__, __LINE__); \
  } while (0)

inline int num_sms(int dev = -1) {
  static int cache[64] = {0};
  if (dev < 0) GICC_CUDA(cudaGetDevice(&dev));
  if (dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  GICC_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev < 64) cache[dev] = n;
  return n;
}

// 2-D bf16/f16 (2-byte) tensor map: rows x cols row-major with leading dimension `ld`
// (elements), box = box_rows x box_cols, 128-byte swizzle when box_cols*2 == 128.
inline CUtensorMap make_tmap_2d(const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t rows, uint64_t cols,
                                uint64_t ld, uint32_t box_rows, uint32_t box_cols, CUtensorMapSwizzle swz) {
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * (uint64_t)elem_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("gicc: TMA base must be 16-byte aligned");
  if ((strides[0] & 15) != 0) throw std::runtime_error("gicc: TMA row stride must be a multiple of 16 bytes");
  GICC_DRV(driver().TensorMapEncodeTiled(&m, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  return m;
}

// 3-D tensor map: [depth][rows][cols] with row stride ld and depth stride `dstride` (elements).
inline CUtensorMap make_tmap_3d(const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t depth,
                                uint64_t rows, uint64_t cols, uint64_t ld, uint64_t dstride, uint32_t box_rows,
                                uint32_t box_cols, CUtensorMapSwizzle swz) {
  CUtensorMap m;
  cuuint64_t dims[3] = {cols, rows, depth};
  cuuint64_t strides[2] = {ld * (uint64_t)elem_bytes, dstride * (uint64_t)elem_bytes};
  cuuint32_t box[3] = {box_cols, box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) throw std::runtime_error("gicc: TMA base must be 16-byte aligned");
  GICC_DRV(driver().TensorMapEncodeTiled(&m, dt, 3, const_cast<void*>(base), dims, strides, box, estr,
                                 CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                 CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE));
  return m;
}

// Convert a C++ exception into a status for the extern "C" entry points.
template <class F>
inline int guarded(F&& f) {
  try {
    f();
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "%s\n", e.what());
    return -1;
  }
}

}  // namespace gicc
