// topology.cpp -- the peer matrix of the visible GPUs, read with cudaDeviceGetP2PAttribute:
// for every ordered pair, whether this process can map the peer's memory, whether atomics
// on it are native, CUDA-array access, and the driver's relative performance rank.  On an
// NVSwitch node every pair reports the same values; the runtime only uses this as a sanity
// check (a pair without access means the peer mappings of exchange() will fail).
#include <cuda_runtime.h>

#include <vector>

#include "gicc/host_util.hpp"
#include "gicc/runtime.hpp"

namespace gicc {

std::vector<P2PLink> p2p_links() {
  int n = 0;
  GICC_CUDA(cudaGetDeviceCount(&n));
  std::vector<P2PLink> out;
  for (int s = 0; s < n; ++s)
    for (int d = 0; d < n; ++d) {
      if (s == d) continue;
      P2PLink l;
      l.src = s;
      l.dst = d;
      GICC_CUDA(cudaDeviceGetP2PAttribute(&l.access, cudaDevP2PAttrAccessSupported, s, d));
      GICC_CUDA(cudaDeviceGetP2PAttribute(&l.native_atomics, cudaDevP2PAttrNativeAtomicSupported, s, d));
      GICC_CUDA(cudaDeviceGetP2PAttribute(&l.array_access, cudaDevP2PAttrCudaArrayAccessSupported, s, d));
      GICC_CUDA(cudaDeviceGetP2PAttribute(&l.perf_rank, cudaDevP2PAttrPerformanceRank, s, d));
      out.push_back(l);
    }
  return out;
}

}  // namespace gicc
