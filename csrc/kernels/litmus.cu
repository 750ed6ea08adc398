// litmus.cu -- the MP / SB litmus tests of gicc/proto/litmus.hpp on GPUs: one thread per
// role, either two GPUs (one role each, peer-mapped words) or two CTAs of one GPU (both
// roles in one launch of two blocks, so they always run concurrently).
#include <cuda_runtime.h>

#include "gicc/config.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"
#include "gicc/proto/litmus.hpp"

namespace gicc {
namespace {

__global__ void k_litmus(ops::LitmusArgs a) {
  if (threadIdx.x != 0) return;
  const int role = a.role_base + (int)blockIdx.x;
  const ops::LitmusRole& R = a.role[role];
  uint64_t violations = 0;
  int st = GICC_OK;
  if (a.test == 0) {
    if (role == 0) {
      proto::litmus_mp_writer<proto::DevMem>(R.data, R.flag, a.k, a.iters, a.seed + 17u * role, a.max_delay);
    } else {
      st = proto::litmus_mp_reader<proto::DevMem>(R.data, R.flag, a.k, a.iters, a.seed + 17u * role, a.max_delay,
                                                  a.timeout_ns, &violations);
    }
  } else {
    st = proto::litmus_sb_side<proto::DevMem>(R.ready_remote, R.ready_local, R.mine_remote, R.theirs_local, a.iters,
                                              a.use_fence, a.seed + 17u * role, a.max_delay, a.timeout_ns, R.out);
  }
  R.result[0] = (uint64_t)st;
  R.result[1] = violations;
}

}  // namespace

namespace ops {
void litmus(const LitmusArgs& a, int nroles_here, cudaStream_t s) {
  NvtxRange nvtx("gicc::ops::litmus");
  if (nroles_here < 1 || nroles_here > 2 || a.role_base < 0 || a.role_base + nroles_here > 2)
    throw std::runtime_error("gicc::litmus: roles 0 and 1, one or both on this GPU");
  if (a.iters < 1 || (a.test == 0 && a.k < 1)) throw std::runtime_error("gicc::litmus: bad sizes");
  k_litmus<<<nroles_here, 32, 0, s>>>(a);
  GICC_CUDA(cudaGetLastError());
}
}  // namespace ops
}  // namespace gicc
