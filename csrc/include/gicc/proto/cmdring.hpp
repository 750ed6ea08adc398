// cmdring.hpp -- a host -> device command ring executed by a persistent kernel, written
// over the Mem policies so the CPU test-suite runs the same producer/consumer code.
//
// The reference keeps an (unused) CPU->GPU ring that a persistent kernel drains to post NIC
// work requests (platform/mlx5/persistent.cuh:27-47, 239-311: head/tail words, 64-byte
// commands, CMD_EXIT).  Here a slot carries its own sequence number (the producer fills
// the body, then stores seq with release; the consumer acquires it), so there is no shared
// head word; the consumer publishes how many commands it finished (`done`), which is both
// the completion signal and the producer's credit.  The consumer's waits are bounded: with
// no command for idle_timeout_ns it exits with GICC_ETIMEDOUT instead of spinning forever.
#pragma once
#include <cstdint>

#include "gicc/error.hpp"
#include "gicc/proto/mem.hpp"

namespace gicc {
namespace proto {

enum CmdOp : uint32_t { CMD_NOP = 0, CMD_PUT = 1, CMD_GET = 2, CMD_SIGNAL = 3, CMD_ADD = 4, CMD_FENCE = 5,
                        CMD_EXIT = 0xFF };

struct alignas(64) Command {
  uint64_t seq;    // i + 1 once slot i % nslots holds command i (written last, release)
  uint32_t op;     // CmdOp
  uint32_t flags;
  uint64_t src;    // PUT/GET: source address (device-addressable)
  uint64_t dst;    // PUT/GET: destination; SIGNAL/ADD: the 64-bit word
  uint64_t size;   // PUT/GET bytes
  uint64_t value;  // SIGNAL/ADD operand
  uint64_t user;   // caller's tag
  uint64_t pad;
};
static_assert(sizeof(Command) == 64, "one command per 64-byte line");

struct CmdRingView {
  Command* cmds;     // [nslots]
  int nslots;
  uint64_t* done;    // commands finished (consumer -> producer)
  uint64_t* status;  // consumer exit status (GICC_OK / GICC_ETIMEDOUT)
  uint64_t idle_timeout_ns;
};

// Producer: enqueue command number `next` (0-based); waits (bounded) for a free slot.
// Returns the command's sequence number (next + 1), or 0 when no slot freed in time.
GICC_PROTO_TEMPLATE
GICC_HD uint64_t cmdring_push(const CmdRingView& v, uint64_t next, const Command& c, uint64_t timeout_ns) {
  if (next >= (uint64_t)v.nslots) {
    uint64_t seen = 0;
    if (!wait_until<Mem>(v.done, CMP_GE, next + 1 - (uint64_t)v.nslots, timeout_ns, &seen)) return 0;
  }
  Command* s = &v.cmds[next % (uint64_t)v.nslots];
  s->op = c.op;
  s->flags = c.flags;
  s->src = c.src;
  s->dst = c.dst;
  s->size = c.size;
  s->value = c.value;
  s->user = c.user;
  Mem::store_release(&s->seq, next + 1);
  return next + 1;
}

// Consumer (one thread): wait for command `i`; returns false on idle timeout.
GICC_PROTO_TEMPLATE
GICC_HD bool cmdring_next(const CmdRingView& v, uint64_t i, Command* out) {
  Command* s = &v.cmds[i % (uint64_t)v.nslots];
  uint64_t seen = 0;
  if (!wait_until<Mem>(&s->seq, CMP_GE, i + 1, v.idle_timeout_ns, &seen)) return false;
  out->seq = i + 1;
  out->op = *reinterpret_cast<volatile uint32_t*>(&s->op);
  out->flags = *reinterpret_cast<volatile uint32_t*>(&s->flags);
  out->src = *reinterpret_cast<volatile uint64_t*>(&s->src);
  out->dst = *reinterpret_cast<volatile uint64_t*>(&s->dst);
  out->size = *reinterpret_cast<volatile uint64_t*>(&s->size);
  out->value = *reinterpret_cast<volatile uint64_t*>(&s->value);
  out->user = *reinterpret_cast<volatile uint64_t*>(&s->user);
  return true;
}

// Consumer: command `i` and everything before it are complete (their stores visible).
GICC_PROTO_TEMPLATE
GICC_HD void cmdring_complete(const CmdRingView& v, uint64_t i) {
  Mem::fence();
  Mem::store_release(v.done, i + 1);
}

}  // namespace proto
}  // namespace gicc
