// am.cuh -- device-side active-message API under the reference's names
// (platform/mlx5/am_device.cuh:90-475: am_poll_peer / am_poll_all, am_wait_one,
// am_send_short / am_send_payload / am_send_request, am_send_reply_fast, am_wait_reply,
// am_recv_and_reply_fast).  Each is one thread's call on an AmView in device memory
// (gicc::am::Am::device_view()); the protocol itself (slot layout, release/acquire
// sequence words, credits, request/reply words) is gicc/proto/am.hpp with device memory
// semantics.  Every wait is bounded by the view's timeout_ns.
#pragma once
#include "gicc/proto/am.hpp"
#include "gicc/proto/mem.hpp"

namespace gicc {
namespace am {

using DevMem = proto::DevMem;

// Dispatch up to max_msgs arrived messages from src with the built-in handlers.
__device__ __forceinline__ int am_poll_peer(AmView* v, int src, int max_msgs = 1 << 30) {
  return poll_peer_builtin<DevMem>(*v, src, max_msgs);
}
__device__ __forceinline__ int am_poll_all(AmView* v, int max_per_peer = 64) {
  return poll_all_builtin<DevMem>(*v, max_per_peer);
}
// Wait (bounded) for the next message from src and dispatch it: 1, or 0 on timeout.
__device__ __forceinline__ int am_wait_one(AmView* v, int src) { return wait_one<DevMem>(*v, src); }

// Sends return the message's sequence number, or 0 when no credit arrived in time.
__device__ __forceinline__ uint64_t am_send_short(AmView* v, int dst, uint16_t handler, const am_args_t& args) {
  return send<DevMem>(*v, dst, handler, args, nullptr, 0, 0);
}
__device__ __forceinline__ uint64_t am_send_payload(AmView* v, int dst, uint16_t handler, const am_args_t& args,
                                                    const void* payload, uint32_t len) {
  return send<DevMem>(*v, dst, handler, args, payload, len, 0);
}
__device__ __forceinline__ uint64_t am_send_request(AmView* v, int dst, uint16_t handler, const am_args_t& args) {
  return send<DevMem>(*v, dst, handler, args, nullptr, 0, AM_FLAG_REQUEST);
}
// Answer request `seq` from src with an 8-byte value.
__device__ __forceinline__ void am_send_reply_fast(AmView* v, int src, uint64_t seq, uint64_t value) {
  reply<DevMem>(*v, src, seq, value);
}
// Wait (bounded) for the reply to request `seq` sent to dst.
__device__ __forceinline__ bool am_wait_reply(AmView* v, int dst, uint64_t seq, uint64_t* value) {
  return wait_reply<DevMem>(*v, dst, seq, value);
}
// Receive the next request from src, run its handler and send the reply: 1, or 0 on timeout.
__device__ __forceinline__ int am_recv_and_reply_fast(AmView* v, int src) { return wait_one<DevMem>(*v, src); }

}  // namespace am
}  // namespace gicc
