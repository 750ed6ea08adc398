// am.hpp -- active messages over NVLink: host class + device entry points.
//
// Reference: platform/ofi/internal/am.hpp:70-373 (host Am: send_handle, send_payload,
// trigger_and_wait, poll_once, reply, check_can_send) and platform/mlx5/am_device.cuh:
// 90-475 (device poll / send_short / send_payload / request / reply).  The ring protocol
// itself (proto/am.hpp) is shared with the CPU-rank tests.
//
// One symmetric region per rank holds: inbox rings [src][nslots][slot] | head[n] | tail[n]
// | credit[n] | ack[n] | ack_val[n] | counter | checksum.  Device code drives the rings
// through the AmView returned by device_view(); the host can also send (copy-engine writes
// of the slot, then of its sequence word) and drain (poll kernel).  A given direction
// (src -> dst) must be driven by either the host or device code, not both at once.
#pragma once
#include <cstdint>

#include "gicc/proto/am.hpp"
#include "gicc/runtime.hpp"

namespace gicc {
namespace am {

class GICC_EXPORT Am {
 public:
  Am(Runtime& rt, int nslots = AM_DEFAULT_RING_SLOTS, uint32_t max_payload = AM_MAX_PAYLOAD_SIZE);
  ~Am();
  Am(const Am&) = delete;
  Am& operator=(const Am&) = delete;

  AmView* device_view() const { return dview_; }  // device memory
  int nslots() const { return nslots_; }
  uint32_t slot_bytes() const { return slot_bytes_; }

  // Host-initiated sends (two copies: slot body, then its seq).  Return the sequence
  // number, or 0 when the receiver has no free slot (check_can_send was false).  Host and
  // device sends share one send cursor per direction, so they may be mixed in stream order.
  uint64_t send_handle(int dst, uint16_t handler, const am_args_t& args, bool request = false);
  uint64_t send_payload(int dst, uint16_t handler, const am_args_t& args, const void* payload, uint32_t len);
  bool check_can_send(int dst);
  // Drain every inbox once with the built-in handlers (kernel); returns messages handled.
  int poll_once(int max_per_peer = 64);
  // Host reply to request `seq` received from `src`.
  void reply(int src, uint64_t seq, uint64_t value);
  // Wait (bounded) until request `seq` to dst was answered; returns the reply value.
  uint64_t wait_reply(int dst, uint64_t seq);
  uint64_t counter();   // COUNTER_ADD accumulator of this rank
  uint64_t checksum();  // CHECKSUM accumulator of this rank
  void trigger_and_wait() { cudaDeviceSynchronize(); }

 private:
  uint64_t head(int dst);  // messages sent to dst so far (device-resident cursor)
  uint64_t host_send(int dst, uint16_t handler, const am_args_t& args, const void* payload, uint32_t len,
                     uint8_t flags);
  Runtime& rt_;
  int n_, me_, nslots_;
  uint32_t slot_bytes_;
  int buf_;
  AmView view_{};           // host copy (device pointers)
  AmView* dview_ = nullptr;
  int* dcount_ = nullptr;
};

}  // namespace am

namespace ops {
// AM ping-pong between this rank and `peer` (device-driven both ways).  mode 0: request/
// reply (64-B request, 8-B reply); mode 1: request/request (64-B both ways).
GICC_EXPORT void am_pingpong(am::AmView* view, int peer, int iters, int mode, bool initiator,
                             unsigned long long* out_ns, cudaStream_t s);
}  // namespace ops
}  // namespace gicc
