// litmus.hpp -- memory-model litmus tests for the flag protocols, written once over the
// Mem policies (DevMem: two GPUs over NVLink, or two CTAs of one GPU; HostMem: two CPU
// ranks over shared memory), with pseudo-random delays between the operations.
//
//   MP (message passing): the writer stores data (relaxed) then the flag (release); the
//      reader waits for the flag (acquire) then loads the data.  Seeing the new flag with
//      old data is forbidden -- every signal/put protocol here relies on it.
//   SB (store buffering): side A stores x, side B stores y, then each loads the other's
//      word.  With a sequentially consistent fence between store and load, both loads
//      returning the old value is forbidden; without it, that outcome is allowed (and is
//      what a store buffer produces), which is why protocols that store-then-poll across
//      ranks put fence.sc between the two.
//
// The reference relies on these orderings in comments only (relaxed data + release
// doorbell, device_opt.cuh:70-95; acquire seq loads, am_device.cuh:101-110); it has no
// litmus tests.
#pragma once
#include <cstdint>

#include "gicc/error.hpp"
#include "gicc/proto/mem.hpp"

namespace gicc {
namespace proto {

GICC_HD uint32_t litmus_rng(uint32_t& s) {
  s ^= s << 13;
  s ^= s >> 17;
  s ^= s << 5;
  return s;
}

// Busy delay of about n cycles (GPU: the SM clock; CPU: loop iterations).
GICC_HD void litmus_delay(uint32_t n) {
#if defined(__CUDA_ARCH__)
  const long long t0 = clock64();
  while (clock64() - t0 < (long long)n) {
  }
#else
  for (volatile uint32_t i = 0; i < n; i = i + 1) {
  }
#endif
}

// MP writer: data is a ring of k words in the reader's memory, flag one word there.
GICC_PROTO_TEMPLATE
GICC_HD void litmus_mp_writer(uint64_t* data, uint64_t* flag, int k, int iters, uint32_t seed, uint32_t max_delay) {
  uint32_t s = seed | 1u;
  for (int i = 0; i < iters; ++i) {
    litmus_delay(litmus_rng(s) % (max_delay + 1));
    Mem::store_relaxed(&data[i % k], (uint64_t)i + 1);
    Mem::store_release(flag, (uint64_t)i + 1);
  }
}

// MP reader (local memory): counts iterations where the flag said >= i+1 but the data
// word of iteration i still held less.  Returns GICC_OK or GICC_ETIMEDOUT.
GICC_PROTO_TEMPLATE
GICC_HD int litmus_mp_reader(const uint64_t* data, const uint64_t* flag, int k, int iters, uint32_t seed,
                             uint32_t max_delay, uint64_t timeout_ns, uint64_t* violations) {
  uint32_t s = seed | 1u;
  uint64_t bad = 0;
  for (int i = 0; i < iters; ++i) {
    uint64_t seen = 0;
    if (!wait_until<Mem>(flag, CMP_GE, (uint64_t)i + 1, timeout_ns, &seen)) {
      *violations = bad;
      return GICC_ETIMEDOUT;
    }
    litmus_delay(litmus_rng(s) % (max_delay + 1));
    if (Mem::load_relaxed(&data[i % k]) < (uint64_t)i + 1) ++bad;
  }
  *violations = bad;
  return GICC_OK;
}

// SB side.  Iteration i: a two-party handshake (ready words, so both sides start together),
// a random delay, then  store 1 -> mine_remote[i];  [fence.sc];  out[i] = theirs_local[i].
// mine_remote is the other side's copy of "my" word array, theirs_local this side's copy of
// the other side's word array; both start zeroed.
GICC_PROTO_TEMPLATE
GICC_HD int litmus_sb_side(uint64_t* ready_remote, const uint64_t* ready_local, uint64_t* mine_remote,
                           const uint64_t* theirs_local, int iters, int use_fence, uint32_t seed, uint32_t max_delay,
                           uint64_t timeout_ns, uint64_t* out) {
  uint32_t s = seed | 1u;
  for (int i = 0; i < iters; ++i) {
    Mem::store_release(ready_remote, (uint64_t)i + 1);
    uint64_t seen = 0;
    if (!wait_until<Mem>(ready_local, CMP_GE, (uint64_t)i + 1, timeout_ns, &seen)) return GICC_ETIMEDOUT;
    litmus_delay(litmus_rng(s) % (max_delay + 1));
    Mem::store_relaxed(&mine_remote[i], 1);
    if (use_fence) Mem::fence_sc();
    out[i] = Mem::load_relaxed(&theirs_local[i]);
  }
  return GICC_OK;
}

}  // namespace proto
}  // namespace gicc
