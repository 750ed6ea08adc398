// api.cpp -- NVSHMEM-style API (gicc/api.hpp) over a process-wide Runtime.
#include "gicc/api.hpp"

#include <cuda_runtime.h>

#include <memory>
#include <mutex>
#include <stdexcept>
#include <unordered_set>

#include "gicc/config.hpp"
#include "gicc/host_util.hpp"

namespace gicc {
namespace {

struct ApiState {
  std::unique_ptr<Runtime> rt;
  GiccContext* ctx = nullptr;
  int ctx_bufs = -1;                 // buffers covered by ctx
  std::unordered_set<void*> live;    // addresses handed out by malloc and not freed
};

std::mutex g_mu;
ApiState* g_api = nullptr;

ApiState& st() {
  if (!g_api || !g_api->rt) throw std::runtime_error("gicc: call gicc::init() first");
  return *g_api;
}

}  // namespace

void init() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_api && g_api->rt) return;
  auto* s = new ApiState;
  s->rt = std::make_unique<Runtime>();
  g_api = s;
}

void* malloc(size_t size) {
  NvtxRange nvtx("gicc::malloc");
  std::lock_guard<std::mutex> lk(g_mu);
  ApiState& s = st();
  const Buffer b = s.rt->alloc(size ? size : 1);  // zero-filled
  s.rt->exchange();                                // collective: maps it on every peer
  s.live.insert(b.ptr);
  return b.ptr;
}

void free(void* ptr) {
  std::lock_guard<std::mutex> lk(g_mu);
  ApiState& s = st();
  if (ptr && !s.live.erase(ptr)) throw std::runtime_error("gicc::free: not an address from gicc::malloc");
  s.rt->barrier();  // collective, like malloc: no peer uses the address after this
}

GiccContext* context() {
  std::lock_guard<std::mutex> lk(g_mu);
  ApiState& s = st();
  if (!s.ctx || s.ctx_bufs != s.rt->num_buffers()) {
    s.ctx = s.rt->build_context();  // owned (and freed) by the runtime
    s.ctx_bufs = s.rt->num_buffers();
  }
  return s.ctx;
}

void* remote_ptr(void* local_ptr, int peer) {
  std::lock_guard<std::mutex> lk(g_mu);
  return st().rt->translate(local_ptr, peer);
}

void barrier() {
  NvtxRange nvtx("gicc::barrier");
  GICC_CUDA(cudaDeviceSynchronize());  // this rank's device work (and its puts) is done
  std::lock_guard<std::mutex> lk(g_mu);
  st().rt->barrier();
}

int my_pe() { return runtime().rank(); }
int n_pes() { return runtime().size(); }

Runtime& runtime() {
  std::lock_guard<std::mutex> lk(g_mu);
  return *st().rt;
}

void finalize() {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_api) return;
  cudaDeviceSynchronize();
  if (g_api->rt) {
    g_api->rt->barrier();
    g_api->rt->finalize();
  }
  delete g_api;
  g_api = nullptr;
}

}  // namespace gicc
