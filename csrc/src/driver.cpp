// driver.cpp -- lazy resolution of the CUDA driver entry points used by the library.
#include "gicc/driver.hpp"

#include <mutex>

namespace gicc {

namespace {
template <class F>
void resolve(const char* name, F*& fn, bool required = true) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q{};
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr) {
    if (required)
      throw std::runtime_error(std::string("gicc: CUDA driver entry point '") + name +
                               "' is unavailable (no GPU driver on this host?)");
    fn = nullptr;
    return;
  }
  fn = reinterpret_cast<F*>(p);
}
}  // namespace

const DriverApi& driver() {
  static DriverApi api;
  static std::once_flag once;
  static std::string err;
  std::call_once(once, [] {
    try {
      resolve("cuGetErrorString", api.GetErrorString);
      resolve("cuTensorMapEncodeTiled", api.TensorMapEncodeTiled);
      resolve("cuMemCreate", api.MemCreate);
      resolve("cuMemRelease", api.MemRelease);
      resolve("cuMemAddressReserve", api.MemAddressReserve);
      resolve("cuMemAddressFree", api.MemAddressFree);
      resolve("cuMemMap", api.MemMap);
      resolve("cuMemUnmap", api.MemUnmap);
      resolve("cuMemSetAccess", api.MemSetAccess);
      resolve("cuMemGetAllocationGranularity", api.MemGetAllocationGranularity);
      resolve("cuMemExportToShareableHandle", api.MemExportToShareableHandle);
      resolve("cuMemImportFromShareableHandle", api.MemImportFromShareableHandle);
      resolve("cuMemGetAddressRange", api.MemGetAddressRange);
      resolve("cuMulticastCreate", api.MulticastCreate, false);
      resolve("cuMulticastAddDevice", api.MulticastAddDevice, false);
      resolve("cuMulticastBindMem", api.MulticastBindMem, false);
      resolve("cuMulticastUnbind", api.MulticastUnbind, false);
      resolve("cuMulticastGetGranularity", api.MulticastGetGranularity, false);
      resolve("cuDeviceGetAttribute", api.DeviceGetAttribute);
      resolve("cuDeviceGet", api.DeviceGet);
      resolve("cuStreamWriteValue64", api.StreamWriteValue64, false);
    } catch (const std::exception& e) {
      err = e.what();
    }
  });
  if (!err.empty()) throw std::runtime_error(err);
  return api;
}

}  // namespace gicc
