// ops.hpp -- C++ entry points of the sm_100a kernels (throw std::runtime_error on misuse).
// Every function enqueues on `stream` and returns without synchronising.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>

#include "gicc/host_util.hpp"

namespace gicc {
namespace ops {

// C[M,N] = alpha * A[M,K] * B[N,K]^T  (bf16 in, f32 accumulate; bf16 or f32 out).
// bn selects the tile width (0 = default 256).
GICC_EXPORT void gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, long long lda, long long ldb,
                           long long ldc, bool out_f32, float alpha, int bn, cudaStream_t stream);

}  // namespace ops
}  // namespace gicc
