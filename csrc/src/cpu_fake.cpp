// cpu_fake.cpp -- CPU ranks over shared memory ("fake device") running the exact flag
// protocols the kernels use (proto/barrier.hpp, proto/am.hpp) with the HostMem policy.
// Used by the CPU test-suite: forked processes map one shared file and call these.
#include <cstdint>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "gicc/proto/am.hpp"
#include "gicc/proto/barrier.hpp"
#include "gicc/proto/cmdring.hpp"
#include "gicc/proto/litmus.hpp"
#include "gicc/types.hpp"
#include "gicc/visibility.hpp"

namespace gicc {
namespace fake {

using proto::HostMem;

// Shared layout for the barrier test: per rank [GICC_MAX_ROUNDS] signal words, one shared
// counter (NVLS emulation) and a [size] progress array.
struct BarrierLayout {
  static size_t words(int size) { return (size_t)size * 16 + 8 + (size_t)size; }
};

// Runs `iters` barriers.  Before each barrier a rank publishes its progress; after it, every
// rank checks that nobody's progress is behind its own (the cross-rank counter check of the
// reference's barrier verifier, legacy/ofi/prototype/barrier-verify.cpp:347-400).
// mode 0 = dissemination, 1 = shared-counter.  skip_at >= 0: this rank stops participating
// at that barrier (to test timeouts).  Returns 0 ok, 1 timeout, 2 ordering violation.
GICC_EXPORT int barrier_run_inject(uint64_t* shm, int rank, int size, int iters, int mode, uint64_t timeout_ns,
                                   int skip_at, int* fail_iter, int inject_mode, int inject_at);
GICC_EXPORT int barrier_run(uint64_t* shm, int rank, int size, int iters, int mode, uint64_t timeout_ns, int skip_at,
                            int* fail_iter) {
  return barrier_run_inject(shm, rank, size, iters, mode, timeout_ns, skip_at, fail_iter, 0, -1);
}

// inject_mode (proto::Inject) is applied by this rank to its own signal at iteration inject_at.
GICC_EXPORT int barrier_run_inject(uint64_t* shm, int rank, int size, int iters, int mode, uint64_t timeout_ns,
                                   int skip_at, int* fail_iter, int inject_mode, int inject_at) {
  uint64_t* sig = shm;                       // [size][16]
  uint64_t* counter = shm + (size_t)size * 16;
  uint64_t* progress = counter + 8;          // [size]
  const int rounds = proto::n_rounds_for(size);
  uint64_t* trig[GICC_MAX_ROUNDS];
  for (int k = 0; k < rounds; ++k) trig[k] = sig + (size_t)((rank + (1 << k)) % size) * 16 + k;
  for (int it = 0; it < iters; ++it) {
    if (it == skip_at) return 0;
    const uint64_t epoch = (uint64_t)it + 1;
    HostMem::store_release(&progress[rank], epoch);
    int st;
    uint64_t seen = 0;
    const int inj = it == inject_at ? inject_mode : proto::INJECT_NONE;
    if (mode == 0) {
      int round = -1;
      st = proto::dissemination_barrier<HostMem>(rounds, trig, sig + (size_t)rank * 16, epoch, timeout_ns, &round, &seen,
                                                 inj);
    } else {
      st = proto::counter_barrier<HostMem>([counter] { HostMem::add_release(counter, 1); }, counter, size, epoch,
                                           timeout_ns, &seen, inj);
    }
    if (st != GICC_OK) {
      if (fail_iter) *fail_iter = it;
      return 1;
    }
    for (int p = 0; p < size; ++p)
      if (HostMem::load_acquire(&progress[p]) < epoch) {
        if (fail_iter) *fail_iter = it;
        return 2;
      }
  }
  return 0;
}

// ---- active messages over shared memory ------------------------------------------------------
// Per-rank region: inbox [size][nslots][slot] | head[size] | tail[size] | credit[size] |
// ack[size] | ack_val[size] | counter | checksum.
GICC_EXPORT size_t am_region_bytes(int size, int nslots, uint32_t slot_bytes) {
  return (size_t)size * nslots * slot_bytes + (size_t)5 * size * 8 + 16;
}

static am::AmView make_view(uint8_t* shm, int rank, int size, int nslots, uint32_t slot_bytes, uint64_t timeout_ns) {
  const size_t region = am_region_bytes(size, nslots, slot_bytes);
  auto base = [&](int r) { return shm + (size_t)r * region; };
  auto words = [&](int r, int which) {
    return reinterpret_cast<uint64_t*>(base(r) + (size_t)size * nslots * slot_bytes) + (size_t)which * size;
  };
  am::AmView v;
  std::memset(&v, 0, sizeof(v));
  v.rank = rank;
  v.size = size;
  v.nslots = nslots;
  v.slot_bytes = slot_bytes;
  v.inbox = base(rank);
  for (int p = 0; p < size; ++p) {
    v.peer_inbox[p] = base(p);
    v.peer_credit[p] = words(p, 2);
    v.peer_ack[p] = words(p, 3);
    v.peer_ack_val[p] = words(p, 4);
  }
  v.head = words(rank, 0);
  v.tail = words(rank, 1);
  v.credit = words(rank, 2);
  v.ack = words(rank, 3);
  v.ack_val = words(rank, 4);
  v.counter = words(rank, 5);
  v.checksum = v.counter + 1;
  v.timeout_ns = timeout_ns;
  return v;
}

// Every rank sends `nmsg` COUNTER_ADD(src+1) and `nmsg` CHECKSUM payloads to every peer
// while draining its own inboxes (tiny rings force credit waits and wrap-around), then
// runs `nreq` ECHO request/reply round trips with its right neighbour.
// Returns 0 ok, 1 send timeout, 2 wrong counter, 3 wrong checksum, 4 reply timeout, 5 bad echo.
GICC_EXPORT int am_run(uint8_t* shm, int rank, int size, int nslots, int nmsg, int nreq, uint64_t timeout_ns,
                       uint64_t* out_counter, uint64_t* out_checksum) {
  am::AmView v = make_view(shm, rank, size, nslots, am::AM_SHORT_SIZE + 256, timeout_ns);
  uint8_t payload[256];
  for (int i = 0; i < 256; ++i) payload[i] = (uint8_t)(i * 7 + rank);
  int sent = 0;
  const int total = 2 * nmsg * (size - 1);
  const uint64_t t_send = HostMem::now_ns();
  while (sent < total) {
    const int idx = sent / (size - 1);
    const int dst = (rank + 1 + sent % (size - 1)) % size;
    am::am_args_t a;
    std::memset(&a, 0, sizeof(a));
    a.data[0] = (uint64_t)rank + 1;
    uint64_t seq;
    if (!am::can_send<HostMem>(v, dst)) {
      am::poll_all_builtin<HostMem>(v, 64);  // drain while we wait for credit
      if (HostMem::now_ns() - t_send > timeout_ns) return 1;
      continue;
    }
    if (idx < nmsg)
      seq = am::send<HostMem>(v, dst, am::AM_HANDLER_COUNTER_ADD, a, nullptr, 0, 0);
    else
      seq = am::send<HostMem>(v, dst, am::AM_HANDLER_CHECKSUM, a, payload, 256, 0);
    if (seq == 0) return 1;
    ++sent;
    am::poll_all_builtin<HostMem>(v, 4);
  }
  // drain until every peer's messages arrived
  uint64_t want_counter = 0;
  for (int p = 0; p < size; ++p)
    if (p != rank) want_counter += (uint64_t)nmsg * (uint64_t)(p + 1);
  // payload bytes are (i*7 + p) mod 256
  uint64_t want_checksum = 0;
  for (int p = 0; p < size; ++p) {
    if (p == rank) continue;
    uint64_t s = 0;
    for (int i = 0; i < 256; ++i) s += (uint8_t)(i * 7 + p);
    want_checksum += (uint64_t)nmsg * s;
  }
  const uint64_t t0 = HostMem::now_ns();
  while (HostMem::load_acquire(v.counter) < want_counter || HostMem::load_acquire(v.checksum) < want_checksum) {
    am::poll_all_builtin<HostMem>(v, 64);
    if (HostMem::now_ns() - t0 > timeout_ns) break;
  }
  if (out_counter) *out_counter = HostMem::load_acquire(v.counter);
  if (out_checksum) *out_checksum = HostMem::load_acquire(v.checksum);
  if (HostMem::load_acquire(v.counter) != want_counter) return 2;
  if (HostMem::load_acquire(v.checksum) != want_checksum) return 3;
  // request/reply with the right neighbour; serve the left neighbour's requests meanwhile
  const int right = (rank + 1) % size;
  for (int i = 0; i < nreq && size > 1; ++i) {
    am::am_args_t a;
    std::memset(&a, 0, sizeof(a));
    a.data[0] = 1000u * (uint64_t)rank + (uint64_t)i;
    const uint64_t seq = am::send<HostMem>(v, right, am::AM_HANDLER_ECHO, a, nullptr, 0, am::AM_FLAG_REQUEST);
    if (seq == 0) return 4;
    uint64_t val = 0;
    const uint64_t t1 = HostMem::now_ns();
    while (HostMem::load_acquire(&v.ack[right]) < seq) {
      am::poll_all_builtin<HostMem>(v, 8);
      if (HostMem::now_ns() - t1 > timeout_ns) return 4;
    }
    val = HostMem::load_acquire(&v.ack_val[right]);
    if (val != a.data[0]) return 5;
  }
  // keep serving until the left neighbour finished its requests
  const int left = (rank - 1 + size) % size;
  const uint64_t t2 = HostMem::now_ns();
  while (size > 1 && HostMem::load_acquire(&v.tail[left]) < (uint64_t)(2 * nmsg + nreq)) {
    am::poll_all_builtin<HostMem>(v, 8);
    if (HostMem::now_ns() - t2 > timeout_ns) return 4;
  }
  return 0;
}

// A receiver waiting for a message that is never sent must time out (returns 0 on timeout).
GICC_EXPORT int am_wait_one(uint8_t* shm, int rank, int size, int nslots, int src, uint64_t timeout_ns) {
  am::AmView v = make_view(shm, rank, size, nslots, am::AM_SHORT_SIZE + 256, timeout_ns);
  return am::wait_one<HostMem>(v, src);
}

// Litmus tests (proto/litmus.hpp) between CPU ranks 0 and 1.  shm holds two regions of
// 2 + k + 2*iters + 2 words: ready, flag, data[k], W[iters], out[iters], result[2].
GICC_EXPORT int litmus_run(uint64_t* shm, int rank, int test, int iters, int k, int use_fence, uint32_t seed,
                           uint32_t max_delay, uint64_t timeout_ns, uint64_t* violations) {
  if (rank < 0 || rank > 1) return GICC_OK;
  const size_t words = 2 + (size_t)k + 2 * (size_t)iters + 2;
  uint64_t* mine = shm + (size_t)rank * words;
  uint64_t* other = shm + (size_t)(1 - rank) * words;
  uint64_t* result = mine + 2 + k + 2 * (size_t)iters;
  uint64_t v = 0;
  int st = GICC_OK;
  if (test == 0) {
    if (rank == 0) {
      proto::litmus_mp_writer<HostMem>(other + 2, other + 1, k, iters, seed, max_delay);
    } else {
      st = proto::litmus_mp_reader<HostMem>(mine + 2, mine + 1, k, iters, seed + 17u, max_delay, timeout_ns, &v);
    }
  } else {
    st = proto::litmus_sb_side<HostMem>(other + 0, mine + 0, other + 2 + k, mine + 2 + k, iters, use_fence,
                                        seed + 17u * rank, max_delay, timeout_ns, mine + 2 + k + iters);
  }
  result[0] = (uint64_t)st;
  result[1] = v;
  if (violations) *violations = v;
  return st;
}

// Command ring (proto/cmdring.hpp) with a CPU consumer thread: the producer queues
// ncmds puts of varying size and offset into dst plus a signal after every 8th, through a
// ring of nslots; the consumer thread executes them.  Returns 0 ok, 1 consumer timeout,
// 2 data mismatch, 3 producer could not get a slot.
GICC_EXPORT int cmdring_selftest(int ncmds, int nslots, uint64_t idle_timeout_ns) {
  std::vector<proto::Command> cmds(nslots);
  uint64_t done = 0, status = ~0ull, sig = 0;
  proto::CmdRingView v{cmds.data(), nslots, &done, &status, idle_timeout_ns};
  std::vector<uint8_t> src(1 << 16), dst(1 << 16, 0);
  for (size_t i = 0; i < src.size(); ++i) src[i] = (uint8_t)(i * 13 + 7);
  std::thread consumer([&] {
    for (uint64_t i = 0;; ++i) {
      proto::Command c;
      if (!proto::cmdring_next<HostMem>(v, i, &c)) {
        __atomic_store_n(&status, (uint64_t)GICC_ETIMEDOUT, __ATOMIC_RELEASE);
        return;
      }
      if (c.op == proto::CMD_EXIT) {
        proto::cmdring_complete<HostMem>(v, i);
        __atomic_store_n(&status, (uint64_t)GICC_OK, __ATOMIC_RELEASE);
        return;
      }
      if (c.op == proto::CMD_PUT) std::memcpy(reinterpret_cast<void*>(c.dst), reinterpret_cast<const void*>(c.src), c.size);
      if (c.op == proto::CMD_ADD) HostMem::add_release(reinterpret_cast<uint64_t*>(c.dst), c.value);
      proto::cmdring_complete<HostMem>(v, i);
    }
  });
  int rc = 0;
  uint64_t next = 0;
  for (int k = 0; k < ncmds && rc == 0; ++k) {
    proto::Command c{};
    const size_t off = ((size_t)k * 977) % (dst.size() - 4096), len = 1 + ((size_t)k * 131) % 4096;
    c.op = proto::CMD_PUT;
    c.src = reinterpret_cast<uint64_t>(src.data() + off);
    c.dst = reinterpret_cast<uint64_t>(dst.data() + off);
    c.size = len;
    if (!proto::cmdring_push<HostMem>(v, next++, c, 10000000000ull)) rc = 3;
    if (k % 8 == 7) {
      proto::Command a{};
      a.op = proto::CMD_ADD;
      a.dst = reinterpret_cast<uint64_t>(&sig);
      a.value = 1;
      if (!proto::cmdring_push<HostMem>(v, next++, a, 10000000000ull)) rc = 3;
    }
  }
  proto::Command e{};
  e.op = proto::CMD_EXIT;
  if (rc == 0 && !proto::cmdring_push<HostMem>(v, next++, e, 10000000000ull)) rc = 3;
  consumer.join();
  if (rc) return rc;
  if (status != GICC_OK || done != next) return 1;
  if (sig != (uint64_t)(ncmds / 8)) return 2;
  for (int k = 0; k < ncmds; ++k) {
    const size_t off = ((size_t)k * 977) % (dst.size() - 4096), len = 1 + ((size_t)k * 131) % 4096;
    for (size_t j = off; j < off + len; ++j)
      if (dst[j] != src[j]) return 2;
  }
  return 0;
}

}  // namespace fake
}  // namespace gicc
