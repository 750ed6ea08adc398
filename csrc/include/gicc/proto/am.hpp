// am.hpp -- active messages over one-sided stores, shared by GPU and CPU-rank code.
//
// Wire format (kept identical to the reference so messages mean the same thing;
// platform/mlx5/am_types.hpp:24-91): a slot is seq(8) | hdr(8) | args(6 x 8) | payload
// (<= 8192 B).  The sender writes hdr/args/payload into the receiver's ring slot for this
// (src, dst) pair and then stores `seq` with release semantics -- so delivery order does
// not rely on in-order NIC byte delivery as the reference's single-write short AM does
// (am_device.cuh:182-236).  The receiver polls `seq` with acquire, dispatches, advances its
// tail and publishes the tail into the sender's credit word (credit-based flow control,
// reference OFI tail_seq: am_types.hpp:155-190).  Requests carry AM_FLAG_REQUEST; the
// receiver answers with an 8-byte value + sequence written into the requester's ack words.
#pragma once
#include <cstdint>

#include "gicc/error.hpp"
#include "gicc/proto/mem.hpp"

namespace gicc {
namespace am {

constexpr int AM_MAX_PEERS = 64;
constexpr int AM_DEFAULT_RING_SLOTS = 128;
constexpr uint32_t AM_SHORT_SIZE = 64;
constexpr uint32_t AM_MAX_PAYLOAD_SIZE = 8192;
constexpr uint32_t AM_SLOT_SIZE = AM_SHORT_SIZE + AM_MAX_PAYLOAD_SIZE;

constexpr uint8_t AM_FLAG_HANDLE_ONLY = 0x01;
constexpr uint8_t AM_FLAG_HAS_PAYLOAD = 0x02;
constexpr uint8_t AM_FLAG_REQUEST = 0x04;

enum AmHandlerId : uint16_t {
  AM_HANDLER_NOOP = 0,
  AM_HANDLER_COUNTER_ADD = 1,  // *counter += args[0]
  AM_HANDLER_CHECKSUM = 2,     // *checksum += sum of payload bytes
  AM_HANDLER_ECHO = 3,         // request: reply with args[0]
  AM_HANDLER_USER_BASE = 100,
};

struct am_args_t {
  uint64_t data[6];
};
struct am_hdr_t {
  uint16_t handler_id;
  uint16_t src_rank;
  uint16_t payload_len;
  uint8_t flags;
  uint8_t reserved;
};
static_assert(sizeof(am_args_t) == 48, "am_args_t is 48 bytes");
static_assert(sizeof(am_hdr_t) == 8, "am_hdr_t is 8 bytes");

struct am_slot_t {
  uint64_t seq;
  am_hdr_t hdr;
  am_args_t args;
  uint8_t payload[AM_MAX_PAYLOAD_SIZE];
};
static_assert(sizeof(am_slot_t) == AM_SLOT_SIZE, "slot layout");

// Per-rank view of the AM state (device memory for the GPU path; shared memory for the
// CPU path).  Arrays indexed by peer rank.
struct AmView {
  int rank;
  int size;
  int nslots;
  uint32_t slot_bytes;                    // AM_SHORT_SIZE or AM_SLOT_SIZE
  uint8_t* inbox;                         // local rings: [src][nslots][slot_bytes]
  uint8_t* peer_inbox[AM_MAX_PEERS];      // each peer's inbox base, mapped here
  uint64_t* head;                         // [dst] messages sent (sender-owned, local)
  uint64_t* tail;                         // [src] messages consumed (receiver-owned, local)
  uint64_t* credit;                       // [dst] receiver-published tails (written by peers)
  uint64_t* peer_credit[AM_MAX_PEERS];    // peer's credit array mapped here
  uint64_t* ack;                          // [dst] reply sequence (written by peers)
  uint64_t* ack_val;                      // [dst] reply value
  uint64_t* peer_ack[AM_MAX_PEERS];
  uint64_t* peer_ack_val[AM_MAX_PEERS];
  uint64_t* counter;                      // COUNTER_ADD target
  uint64_t* checksum;                     // CHECKSUM accumulator
  uint64_t timeout_ns;
  ErrorRecord* err;
};

GICC_HD am_slot_t* slot_at(uint8_t* ring_base, int src, int nslots, uint32_t slot_bytes, uint64_t idx) {
  return reinterpret_cast<am_slot_t*>(ring_base + ((uint64_t)src * nslots + idx % (uint64_t)nslots) * slot_bytes);
}

GICC_PROTO_TEMPLATE
GICC_HD bool can_send(const AmView& v, int dst) {
  return v.head[dst] - Mem::load_acquire(&v.credit[dst]) < (uint64_t)v.nslots;
}

// Send one message; returns its sequence number (>0) or 0 on timeout (no credit).
GICC_PROTO_TEMPLATE
GICC_HD uint64_t send(AmView& v, int dst, uint16_t handler, const am_args_t& args, const void* payload,
                      uint32_t len, uint8_t flags) {
  if (len > AM_MAX_PAYLOAD_SIZE || (len > 0 && v.slot_bytes < AM_SHORT_SIZE + len)) return 0;
  if (!can_send<Mem>(v, dst)) {
    uint64_t seen = 0;
    const uint64_t need = v.head[dst] + 1 - (uint64_t)v.nslots;
    if (!proto::wait_until<Mem>(&v.credit[dst], proto::CMP_GE, need, v.timeout_ns, &seen)) return 0;
  }
  const uint64_t seq = v.head[dst] + 1;
  am_slot_t* s = slot_at(v.peer_inbox[dst], v.rank, v.nslots, v.slot_bytes, v.head[dst]);
  if (len) {
    const uint8_t* p = static_cast<const uint8_t*>(payload);
    for (uint32_t i = 0; i < len; ++i) s->payload[i] = p[i];
  }
  for (int i = 0; i < 6; ++i) s->args.data[i] = args.data[i];
  am_hdr_t h;
  h.handler_id = handler;
  h.src_rank = (uint16_t)v.rank;
  h.payload_len = (uint16_t)len;
  h.flags = (uint8_t)(flags | (len ? AM_FLAG_HAS_PAYLOAD : AM_FLAG_HANDLE_ONLY));
  h.reserved = 0;
  s->hdr = h;
  Mem::fence();
  Mem::store_release(&s->seq, seq);
  v.head[dst] = seq;
  return seq;
}

// Write the reply for request `seq` from `src` into the requester's ack words.
GICC_PROTO_TEMPLATE
GICC_HD void reply(AmView& v, int src, uint64_t seq, uint64_t value) {
  Mem::store_release(&v.peer_ack_val[src][v.rank], value);
  Mem::store_release(&v.peer_ack[src][v.rank], seq);
}

// Built-in handlers.  Returns the reply value for requests.
GICC_PROTO_TEMPLATE
GICC_HD uint64_t builtin_handler(AmView& v, const am_slot_t* s) {
  switch (s->hdr.handler_id) {
    case AM_HANDLER_COUNTER_ADD:
      Mem::store_release(v.counter, Mem::load_relaxed(v.counter) + s->args.data[0]);
      return s->args.data[0];
    case AM_HANDLER_CHECKSUM: {
      uint64_t acc = 0;
      for (uint32_t i = 0; i < s->hdr.payload_len; ++i) acc += s->payload[i];
      Mem::store_release(v.checksum, Mem::load_relaxed(v.checksum) + acc);
      return acc;
    }
    case AM_HANDLER_ECHO:
      return s->args.data[0];
    default:
      return 0;
  }
}

// Poll the ring of `src`: dispatch up to max_msgs messages that have arrived.
// Handler(AmView&, const am_slot_t*) -> uint64_t reply value.  Returns messages handled.
template <class Mem, class Handler>
GICC_HD int poll_peer(AmView& v, int src, int max_msgs, Handler&& handler) {
  int n = 0;
  while (n < max_msgs) {
    const uint64_t idx = v.tail[src];
    am_slot_t* s = slot_at(v.inbox, src, v.nslots, v.slot_bytes, idx);
    if (Mem::load_acquire(&s->seq) != idx + 1) break;
    const uint64_t rv = handler(v, s);
    if (s->hdr.flags & AM_FLAG_REQUEST) reply<Mem>(v, src, idx + 1, rv);
    v.tail[src] = idx + 1;
    Mem::store_release(&v.peer_credit[src][v.rank], idx + 1);
    ++n;
  }
  return n;
}

GICC_PROTO_TEMPLATE
GICC_HD int poll_peer_builtin(AmView& v, int src, int max_msgs) {
  return poll_peer<Mem>(v, src, max_msgs, [](AmView& vv, const am_slot_t* s) { return builtin_handler<Mem>(vv, s); });
}

GICC_PROTO_TEMPLATE
GICC_HD int poll_all_builtin(AmView& v, int max_per_peer) {
  int n = 0;
  for (int p = 0; p < v.size; ++p) n += poll_peer_builtin<Mem>(v, p, max_per_peer);  // self included
  return n;
}

// Wait (bounded) for one message from src and dispatch it.  Returns 1, or 0 on timeout.
GICC_PROTO_TEMPLATE
GICC_HD int wait_one(AmView& v, int src) {
  const uint64_t idx = v.tail[src];
  am_slot_t* s = slot_at(v.inbox, src, v.nslots, v.slot_bytes, idx);
  uint64_t seen = 0;
  if (!proto::wait_until<Mem>(&s->seq, proto::CMP_EQ, idx + 1, v.timeout_ns, &seen)) return 0;
  return poll_peer_builtin<Mem>(v, src, 1);
}

// Wait (bounded) for the reply to request `seq` sent to dst; returns true and the value.
GICC_PROTO_TEMPLATE
GICC_HD bool wait_reply(AmView& v, int dst, uint64_t seq, uint64_t* value) {
  uint64_t seen = 0;
  if (!proto::wait_until<Mem>(&v.ack[dst], proto::CMP_GE, seq, v.timeout_ns, &seen)) return false;
  if (value) *value = Mem::load_acquire(&v.ack_val[dst]);
  return true;
}

}  // namespace am
}  // namespace gicc
