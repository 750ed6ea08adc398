/* noalloc.h -- an entry point that allocates no memory.
 *
 * This entry point has no counterpart in the reference.  It exists for callers that
 * cannot allocate device memory at the moment they call: code running inside a custom
 * allocator or an out-of-memory handler, embedders whose own memory manager owns every
 * device allocation, and runtimes that must not call cudaMalloc/cudaFree once they are
 * set up (both can synchronise the device and can fail).  Everything else in this
 * library asks the caller (or cudaMalloc) for its working memory; this one keeps its
 * working memory in a fixed array that lives inside the library itself.
 *
 * gicc_jacobi_step_norm_noalloc -- one Jacobi sweep (the 5-point stencil of
 * gicc::ops::jacobi_step, one GPU, no halo peers) that also returns the squared L2 norm of
 * the update, new - old, summed over the owned rows.
 *
 *   a        [rows+2][nx] fp32 input field (row 0 and row rows+1 are the fixed edges)
 *   b        [rows+2][nx] fp32 output field (interior rows written; keep the edges set)
 *   norm_sq  one double on the device, output: sum of (new - old)^2
 *
 * Working memory: one partial sum per thread block in a static device array of
 * GICC_NOALLOC_MAX_BLOCKS doubles (512 KiB).  The sweep uses ceil(nx/1024) * ceil(rows/16)
 * blocks; larger grids (beyond 32768 x 32768 cells) are rejected with
 * cudaErrorInvalidValue and a message on stderr.  Every block overwrites its own slot, so
 * nothing has to start at zero.  The array is loaded on every GPU that loads the library
 * and stays there until the process exits.
 *
 * Set-up: the first call on a device looks up the array's device address with
 * cudaGetSymbolAddress (with that device current) and caches it.  Make that first call
 * before capturing a stream into a CUDA graph.  The cached address is not refreshed
 * after cudaDeviceReset (or any other teardown of the device's primary context): do not
 * call this entry point on a device after resetting it in the same process.
 *
 * Aliasing: a and b must be two separate fields (the sweep reads the neighbours of cells
 * it writes); overlapping fields are rejected with cudaErrorInvalidValue.
 *
 * Concurrency: all calls share the one array.  Calls that overlap on the GPU (different
 * streams, or different host threads) race on it and may return wrong norms; serialise
 * them (same stream, or events).
 *
 * Returns cudaSuccess or the first CUDA error; never allocates (no cudaMalloc, no
 * cudaFree, no allocating library routine).
 */
#ifndef GICC_NOALLOC_H
#define GICC_NOALLOC_H

#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define GICC_NOALLOC_MAX_BLOCKS 65536

cudaError_t gicc_jacobi_step_norm_noalloc(const float* a, float* b, int nx, int rows, double* norm_sq,
                                          cudaStream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GICC_NOALLOC_H */
