// am.cu -- active-message host class and device kernels (poll, ping-pong).
#include "gicc/am.hpp"

#include <chrono>
#include <cstring>
#include <thread>

#include "gicc/device/am.cuh"
#include "gicc/device/ptx.cuh"
#include "gicc/host_util.hpp"

namespace gicc {
namespace am {
namespace {

using proto::DevMem;

__global__ void k_am_poll(AmView v, int max_per_peer, int* count) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  *count = am_poll_all(&v, max_per_peer);
}

// mode 0: request/reply (ECHO request, 8-byte reply); mode 1: request/request (NOOP both ways).
__global__ void k_am_pingpong(AmView v, int peer, int iters, int mode, int initiator, unsigned long long* out_ns) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  const uint64_t t0 = ptx::globaltimer();
  am_args_t a;
  for (int q = 0; q < 6; ++q) a.data[q] = 0;
  for (int i = 0; i < iters; ++i) {
    a.data[0] = (uint64_t)i + 1;
    if (mode == 0) {
      if (initiator) {
        const uint64_t seq = am_send_request(&v, peer, AM_HANDLER_ECHO, a);
        uint64_t val = 0;
        if (seq == 0 || !am_wait_reply(&v, peer, seq, &val) || val != a.data[0]) {
          report_error(v.err, GICC_ETIMEDOUT, W_AM_WAIT, v.rank, peer, val, a.data[0]);
          return;
        }
      } else if (!am_recv_and_reply_fast(&v, peer)) {
        report_error(v.err, GICC_ETIMEDOUT, W_AM_WAIT, v.rank, peer, 0, (uint64_t)i);
        return;
      }
    } else {
      if (initiator) {
        if (!am_send_short(&v, peer, AM_HANDLER_NOOP, a) || !am_wait_one(&v, peer)) {
          report_error(v.err, GICC_ETIMEDOUT, W_AM_WAIT, v.rank, peer, 0, (uint64_t)i);
          return;
        }
      } else {
        if (!am_wait_one(&v, peer) || !am_send_short(&v, peer, AM_HANDLER_NOOP, a)) {
          report_error(v.err, GICC_ETIMEDOUT, W_AM_WAIT, v.rank, peer, 0, (uint64_t)i);
          return;
        }
      }
    }
  }
  *out_ns = ptx::globaltimer() - t0;
}

size_t region_bytes(int n, int nslots, uint32_t slot_bytes) {
  return (size_t)n * nslots * slot_bytes + (size_t)5 * n * 8 + 16;
}

}  // namespace

Am::Am(Runtime& rt, int nslots, uint32_t max_payload) : rt_(rt) {
  n_ = rt.size();
  me_ = rt.rank();
  if (n_ > AM_MAX_PEERS) throw std::runtime_error("gicc::am::Am: too many ranks");
  if (max_payload > AM_MAX_PAYLOAD_SIZE) throw std::runtime_error("gicc::am::Am: payload > 8192 bytes");
  nslots_ = nslots;
  slot_bytes_ = (AM_SHORT_SIZE + max_payload + 15) & ~15u;
  const size_t bytes = region_bytes(n_, nslots_, slot_bytes_);
  Buffer b = rt.alloc(bytes);  // zero-filled by alloc
  buf_ = b.index;
  rt.exchange();
  auto base = [&](int r) { return static_cast<uint8_t*>(rt.remote_ptr(r, buf_, 0)); };
  auto words = [&](int r, int which) {
    return reinterpret_cast<uint64_t*>(base(r) + (size_t)n_ * nslots_ * slot_bytes_) + (size_t)which * n_;
  };
  std::memset(&view_, 0, sizeof(view_));
  view_.rank = me_;
  view_.size = n_;
  view_.nslots = nslots_;
  view_.slot_bytes = slot_bytes_;
  view_.inbox = base(me_);
  for (int p = 0; p < n_; ++p) {
    view_.peer_inbox[p] = base(p);
    view_.peer_credit[p] = words(p, 2);
    view_.peer_ack[p] = words(p, 3);
    view_.peer_ack_val[p] = words(p, 4);
  }
  view_.head = words(me_, 0);
  view_.tail = words(me_, 1);
  view_.credit = words(me_, 2);
  view_.ack = words(me_, 3);
  view_.ack_val = words(me_, 4);
  view_.counter = words(me_, 5);
  view_.checksum = view_.counter + 1;
  view_.timeout_ns = rt.timeout_ns();
  view_.err = rt.error_record();
  GICC_CUDA(cudaMalloc(&dview_, sizeof(AmView)));
  GICC_CUDA(cudaMemcpy(dview_, &view_, sizeof(AmView), cudaMemcpyHostToDevice));
  GICC_CUDA(cudaMalloc(&dcount_, sizeof(int)));
  rt.barrier();
}

Am::~Am() {
  cudaDeviceSynchronize();
  if (dview_) cudaFree(dview_);
  if (dcount_) cudaFree(dcount_);
}

// The send cursor of every direction lives in device memory (view_.head), shared by host
// sends and device sends, so both kinds can be mixed on one direction in stream order.
uint64_t Am::head(int dst) {
  uint64_t h = 0;
  GICC_CUDA(cudaMemcpy(&h, view_.head + dst, sizeof(h), cudaMemcpyDeviceToHost));
  return h;
}

bool Am::check_can_send(int dst) {
  uint64_t credit = 0;
  GICC_CUDA(cudaMemcpy(&credit, view_.credit + dst, sizeof(credit), cudaMemcpyDeviceToHost));
  return head(dst) - credit < (uint64_t)nslots_;
}

uint64_t Am::host_send(int dst, uint16_t handler, const am_args_t& args, const void* payload, uint32_t len,
                       uint8_t flags) {
  if (dst < 0 || dst >= n_) throw std::runtime_error("gicc::am::Am: bad destination");
  if (AM_SHORT_SIZE + len > slot_bytes_) throw std::runtime_error("gicc::am::Am: payload larger than a slot");
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(rt_.timeout_ns());
  while (!check_can_send(dst)) {
    if (std::chrono::steady_clock::now() > deadline) return 0;
    std::this_thread::yield();
  }
  const uint64_t cur = head(dst);
  const uint64_t seq = cur + 1;
  uint8_t* slot = view_.peer_inbox[dst] + ((size_t)me_ * nslots_ + cur % nslots_) * slot_bytes_;
  std::vector<uint8_t> body(AM_SHORT_SIZE - 8 + len);
  am_hdr_t h{handler, (uint16_t)me_, (uint16_t)len,
             (uint8_t)(flags | (len ? AM_FLAG_HAS_PAYLOAD : AM_FLAG_HANDLE_ONLY)), 0};
  std::memcpy(body.data(), &h, sizeof(h));
  std::memcpy(body.data() + 8, &args, sizeof(args));
  if (len) std::memcpy(body.data() + AM_SHORT_SIZE - 8, payload, len);
  // body first, then the sequence word: synchronous copies complete in this order
  GICC_CUDA(cudaMemcpy(slot + 8, body.data(), body.size(), cudaMemcpyHostToDevice));
  GICC_CUDA(cudaMemcpy(slot, &seq, sizeof(seq), cudaMemcpyHostToDevice));
  GICC_CUDA(cudaMemcpy(view_.head + dst, &seq, sizeof(seq), cudaMemcpyHostToDevice));
  return seq;
}

uint64_t Am::send_handle(int dst, uint16_t handler, const am_args_t& args, bool request) {
  return host_send(dst, handler, args, nullptr, 0, request ? AM_FLAG_REQUEST : 0);
}

uint64_t Am::send_payload(int dst, uint16_t handler, const am_args_t& args, const void* payload, uint32_t len) {
  return host_send(dst, handler, args, payload, len, 0);
}

int Am::poll_once(int max_per_peer) {
  k_am_poll<<<1, 32>>>(view_, max_per_peer, dcount_);
  GICC_CUDA(cudaGetLastError());
  int c = 0;
  GICC_CUDA(cudaMemcpy(&c, dcount_, sizeof(c), cudaMemcpyDeviceToHost));
  return c;
}

void Am::reply(int src, uint64_t seq, uint64_t value) {
  GICC_CUDA(cudaMemcpy(view_.peer_ack_val[src] + me_, &value, sizeof(value), cudaMemcpyHostToDevice));
  GICC_CUDA(cudaMemcpy(view_.peer_ack[src] + me_, &seq, sizeof(seq), cudaMemcpyHostToDevice));
}

uint64_t Am::wait_reply(int dst, uint64_t seq) {
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(rt_.timeout_ns());
  for (;;) {
    uint64_t a = 0;
    GICC_CUDA(cudaMemcpy(&a, view_.ack + dst, sizeof(a), cudaMemcpyDeviceToHost));
    if (a >= seq) break;
    if (std::chrono::steady_clock::now() > deadline) throw std::runtime_error("gicc::am::Am: reply timed out");
    std::this_thread::yield();
  }
  uint64_t v = 0;
  GICC_CUDA(cudaMemcpy(&v, view_.ack_val + dst, sizeof(v), cudaMemcpyDeviceToHost));
  return v;
}

uint64_t Am::counter() {
  uint64_t v = 0;
  GICC_CUDA(cudaMemcpy(&v, view_.counter, sizeof(v), cudaMemcpyDeviceToHost));
  return v;
}

uint64_t Am::checksum() {
  uint64_t v = 0;
  GICC_CUDA(cudaMemcpy(&v, view_.checksum, sizeof(v), cudaMemcpyDeviceToHost));
  return v;
}

}  // namespace am

namespace ops {
void am_pingpong(am::AmView* view, int peer, int iters, int mode, bool initiator, unsigned long long* out_ns,
                 cudaStream_t s) {
  am::AmView v;
  GICC_CUDA(cudaMemcpy(&v, view, sizeof(v), cudaMemcpyDeviceToHost));
  am::k_am_pingpong<<<1, 32, 0, s>>>(v, peer, iters, mode, initiator ? 1 : 0, out_ns);
  GICC_CUDA(cudaGetLastError());
}
}  // namespace ops
}  // namespace gicc
