// api.hpp -- the NVSHMEM-style convenience API over one process-wide gicc::Runtime
// (the reference's platform/mlx5/gicc_api.hpp:42-129 names: init, malloc, free, context,
// remote_ptr, barrier, my_pe, n_pes, runtime, finalize).
//
//   gicc::init();                                   // bootstrap from the environment
//   float* x = (float*)gicc::malloc(n * 4);         // collective, symmetric, zeroed
//   GiccContext* ctx = gicc::context();             // device memory; pass to kernels
//   kernel<<<..>>>(ctx, x);  // device: gicc::put(ctx, remote_dst, src, bytes, peer)
//   gicc::barrier();
//   gicc::finalize();
//
// malloc and free are collective (every rank calls them in the same order).  free() only
// retires the address: the runtime's buffer table is append-only, so the memory returns
// at finalize().  context() rebuilds the device context after allocations.
#pragma once
#include <cstddef>

#include "gicc/runtime.hpp"

namespace gicc {

GICC_EXPORT void init();
GICC_EXPORT void* malloc(size_t size);
GICC_EXPORT void free(void* ptr);
GICC_EXPORT GiccContext* context();
GICC_EXPORT void* remote_ptr(void* local_ptr, int peer);
GICC_EXPORT void barrier();
GICC_EXPORT int my_pe();
GICC_EXPORT int n_pes();
GICC_EXPORT Runtime& runtime();
GICC_EXPORT void finalize();

}  // namespace gicc
