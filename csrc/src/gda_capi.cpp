// gda_capi.cpp -- the OpenGDA C API (gda.h) on top of gicc::Runtime / gicc::Barrier.
//
// The reference's examples (examples/put_example.cpp:81-244, test_example.cpp:55-213,
// mr_example.cpp:26-85, gda_get_bw.cpp:96, barrier_test.cpp:124-202, mm_hip_gda.cpp:71-235,
// mm_hip_gda_proxy.cpp:97-377) call this API; its header and library are not in the
// reference tree, so the semantics here follow those call sites, mapped to NVLink: a
// transfer is loads/stores through the peer mapping of the target's symmetric buffer, its
// completion a release store into pinned host memory.
#include "gda/gda.h"

#include <cuda_runtime.h>

#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <exception>
#include <memory>
#include <mutex>
#include <thread>
#include <vector>

#include "gicc/barrier.hpp"
#include "gicc/host_util.hpp"
#include "gicc/runtime.hpp"

namespace {

constexpr int kSlots = 4096;  // completion words (concurrently live transfers)

struct GdaState {
  std::unique_ptr<gicc::Runtime> rt;
  gicc::Buffer buf{};
  uint64_t* completion_host = nullptr;  // [kSlots] pinned, mapped
  uint64_t* completion_dev = nullptr;
  std::vector<int> free_slots;
  std::vector<uint64_t> slot_seq;
  std::vector<std::unique_ptr<gicc::Barrier>> barriers;
  std::mutex mu;
};

GdaState* g = nullptr;

void report(const char* fn, const char* what) { std::fprintf(stderr, "%s: %s\n", fn, what); }

bool ready(const char* fn) {
  if (!g || !g->rt) {
    report(fn, "gda_init() has not been called");
    return false;
  }
  return true;
}

template <class F>
auto guarded(const char* fn, F&& f, decltype(f()) fail) -> decltype(f()) {
  try {
    return f();
  } catch (const std::exception& e) {
    report(fn, e.what());
    return fail;
  }
}

}  // namespace

struct gda_proxy_barrier {
  gda_gpu_barrier_t* dev_host;  // host copy handed to the caller
  gicc::Barrier* barrier;
};

namespace {
gicc::Barrier* barrier_of(const gda_gpu_barrier_t* b) {
  for (auto& p : g->barriers)
    if (p && p->device_ctx() && b && b->ctx.signals) {
      gicc::BarrierCtx c;
      GICC_CUDA(cudaMemcpy(&c, p->device_ctx(), sizeof(c), cudaMemcpyDeviceToHost));
      if (c.signals == b->ctx.signals) return p.get();
    }
  return nullptr;
}

gda_gpu_barrier_t* new_gpu_barrier() {
  auto bar = std::make_unique<gicc::Barrier>(*g->rt, false);
  auto* out = new gda_gpu_barrier_t;
  GICC_CUDA(cudaMemcpy(&out->ctx, bar->device_ctx(), sizeof(out->ctx), cudaMemcpyDeviceToHost));
  g->barriers.push_back(std::move(bar));
  return out;
}

gda_handle_t* new_transfer(const char* fn, const void* local, size_t size, int peer, size_t remote_offset,
                           bool is_get) {
  if (!ready(fn)) return nullptr;
  return guarded(
      fn,
      [&]() -> gda_handle_t* {
        if (peer < 0 || peer >= g->rt->size()) throw std::runtime_error("peer out of range");
        if (remote_offset > g->buf.size || size > g->buf.size - remote_offset)
          throw std::runtime_error("remote_offset + size is outside the peer's gda_gpu_buf");
        int slot;
        {
          std::lock_guard<std::mutex> lk(g->mu);
          if (g->free_slots.empty()) throw std::runtime_error("too many live transfers (gda_free the finished ones)");
          slot = g->free_slots.back();
          g->free_slots.pop_back();
        }
        void* remote = g->rt->remote_ptr(peer, g->buf.index, remote_offset);
        auto* h = new gda_handle_t;
        std::memset(h, 0, sizeof(*h));
        h->gpu.src = is_get ? remote : local;
        h->gpu.dst = is_get ? const_cast<void*>(local) : remote;
        h->gpu.size = size;
        h->gpu.completion = g->completion_dev + slot;
        h->gpu.seq = ++g->slot_seq[slot];
        h->gpu.timeout_ns = g->rt->timeout_ns();
        h->peer = peer;
        h->is_get = is_get ? 1 : 0;
        h->remote_offset = remote_offset;
        h->slot = slot;
        return h;
      },
      nullptr);
}

bool done(const gda_handle_t* h) {
  return reinterpret_cast<volatile uint64_t*>(g->completion_host)[h->slot] >= h->gpu.seq;
}
}  // namespace

GDA_API int gda_init(void) {
  if (g && g->rt) return 0;
  return guarded(
      "gda_init",
      [&]() -> int {
        auto* s = new GdaState;
        s->rt = std::make_unique<gicc::Runtime>();
        size_t bytes = 64ull << 20;
        if (const char* e = std::getenv("GDA_GPU_BUF_SIZE")) bytes = std::strtoull(e, nullptr, 0);
        s->buf = s->rt->alloc(bytes);
        s->rt->exchange();
        void* h = nullptr;
        GICC_CUDA(cudaHostAlloc(&h, kSlots * sizeof(uint64_t), cudaHostAllocMapped | cudaHostAllocPortable));
        std::memset(h, 0, kSlots * sizeof(uint64_t));
        s->completion_host = static_cast<uint64_t*>(h);
        void* d = nullptr;
        GICC_CUDA(cudaHostGetDevicePointer(&d, h, 0));
        s->completion_dev = static_cast<uint64_t*>(d);
        s->slot_seq.assign(kSlots, 0);
        for (int i = kSlots - 1; i >= 0; --i) s->free_slots.push_back(i);
        g = s;
        return 0;
      },
      -1);
}

GDA_API void gda_finalize(void) {
  if (!g) return;
  cudaDeviceSynchronize();
  try {
    g->barriers.clear();
    if (g->rt) {
      g->rt->barrier();
      g->rt->finalize();
    }
  } catch (const std::exception& e) {
    report("gda_finalize", e.what());
  }
  if (g->completion_host) cudaFreeHost(g->completion_host);
  delete g;
  g = nullptr;
}

GDA_API int gda_rank(void) { return g && g->rt ? g->rt->rank() : -1; }
GDA_API int gda_size(void) { return g && g->rt ? g->rt->size() : -1; }
GDA_API const char* gda_get_version(void) { return "opengda_b200 1.0 (OpenGDA C API over NVLink / NVSwitch)"; }

GDA_API int gda_barrier(void) {
  if (!ready("gda_barrier")) return -1;
  return guarded(
      "gda_barrier",
      [&]() -> int {
        GICC_CUDA(cudaDeviceSynchronize());  // this rank's device-side transfers are done
        g->rt->barrier();
        return 0;
      },
      -1);
}

GDA_API void* gda_gpu_buf(void) { return g && g->rt ? g->buf.ptr : nullptr; }
GDA_API size_t gda_gpu_buf_size(void) { return g && g->rt ? g->buf.size : 0; }

GDA_API gda_mr_t* gda_register_memory(void* buf, size_t size, int is_gpu) {
  if (!ready("gda_register_memory")) return nullptr;
  return guarded(
      "gda_register_memory",
      [&]() -> gda_mr_t* {
        const gicc::Buffer b = g->rt->register_buffer(buf, size, is_gpu != 0);
        auto* mr = new gda_mr_t;
        mr->addr = buf;
        mr->size = size;
        mr->is_gpu = is_gpu;
        mr->index = b.index;
        mr->key = b.lkey;
        return mr;
      },
      nullptr);
}

GDA_API uint64_t gda_mr_get_key(gda_mr_t* mr) { return mr ? mr->key : 0; }
// On NVLink the "descriptor" of a region is its address: peers reach it through a mapping.
GDA_API void* gda_mr_get_desc(gda_mr_t* mr) { return mr ? mr->addr : nullptr; }

GDA_API int gda_deregister_memory(gda_mr_t* mr) {
  // The runtime keeps the registration (its buffer table is append-only and index-stable);
  // the handle is released.
  if (!mr) return -1;
  delete mr;
  return 0;
}

GDA_API gda_handle_t* gda_put(const void* local, size_t size, int peer, size_t remote_offset) {
  return new_transfer("gda_put", local, size, peer, remote_offset, false);
}

GDA_API gda_handle_t* gda_get(void* local, size_t size, int peer, size_t remote_offset) {
  return new_transfer("gda_get", local, size, peer, remote_offset, true);
}

GDA_API int gda_wait(gda_handle_t* h) {
  if (!h || !ready("gda_wait")) return -1;
  const auto deadline = std::chrono::steady_clock::now() + std::chrono::nanoseconds(g->rt->timeout_ns());
  while (!done(h)) {
    if (std::chrono::steady_clock::now() > deadline) {
      report("gda_wait", "timed out (was the transfer triggered?)");
      return -1;
    }
    std::this_thread::yield();
  }
  return 0;
}

GDA_API int gda_test(gda_handle_t* h) { return h && g && done(h) ? 1 : 0; }

GDA_API int gda_test_any(gda_handle_t** hs, int n, int* idx) {
  if (!g || !hs) return 0;
  for (int i = 0; i < n; ++i)
    if (hs[i] && done(hs[i])) {
      if (idx) *idx = i;
      return 1;
    }
  return 0;
}

GDA_API int gda_test_all(gda_handle_t** hs, int n) {
  if (!g || !hs) return 0;
  for (int i = 0; i < n; ++i)
    if (!hs[i] || !done(hs[i])) return 0;
  return 1;
}

GDA_API int gda_flush(void) {
  // Triggered transfers finish inside the kernels that trigger them; flushing is waiting
  // for those kernels.
  return cudaDeviceSynchronize() == cudaSuccess ? 0 : -1;
}

GDA_API void gda_free(gda_handle_t* h) {
  if (!h) return;
  if (g) {
    std::lock_guard<std::mutex> lk(g->mu);
    g->free_slots.push_back(h->slot);
  }
  delete h;
}

GDA_API gda_gpu_barrier_t* gda_gpu_barrier_alloc(int /*max_iters: epochs have no per-iteration state*/) {
  if (!ready("gda_gpu_barrier_alloc")) return nullptr;
  return guarded("gda_gpu_barrier_alloc", [&]() { return new_gpu_barrier(); }, (gda_gpu_barrier_t*)nullptr);
}

GDA_API int gda_gpu_barrier_reset(gda_gpu_barrier_t* b) {
  // Continue from the epoch after the last barrier this rank completed (the device advanced
  // its own copy); the caller copies the host struct to the device again afterwards.
  if (!b || !ready("gda_gpu_barrier_reset")) return -1;
  return guarded(
      "gda_gpu_barrier_reset",
      [&]() -> int {
        GICC_CUDA(cudaDeviceSynchronize());
        gicc::Barrier* bar = barrier_of(b);
        if (!bar) throw std::runtime_error("not a barrier from gda_gpu_barrier_alloc");
        b->ctx.expected_signal = bar->count() + 1;
        g->rt->barrier();
        return 0;
      },
      -1);
}

GDA_API void gda_gpu_barrier_free(gda_gpu_barrier_t* b) {
  if (!b) return;
  if (g) {
    gicc::Barrier* bar = barrier_of(b);
    for (auto& p : g->barriers)
      if (p.get() == bar) p.reset();
  }
  delete b;
}

GDA_API gda_proxy_barrier_t* gda_proxy_barrier_alloc(int /*window_size*/) {
  if (!ready("gda_proxy_barrier_alloc")) return nullptr;
  return guarded(
      "gda_proxy_barrier_alloc",
      [&]() -> gda_proxy_barrier_t* {
        auto* p = new gda_proxy_barrier;
        p->dev_host = new_gpu_barrier();
        p->barrier = g->barriers.back().get();
        return p;
      },
      nullptr);
}

GDA_API gda_proxy_barrier_dev_t* gda_proxy_barrier_get_dev(gda_proxy_barrier_t* b) { return b ? b->dev_host : nullptr; }
GDA_API int gda_proxy_start(gda_proxy_barrier_t* b) { return b ? 0 : -1; }
GDA_API void gda_proxy_stop(gda_proxy_barrier_t*) {}

GDA_API int gda_proxy_barrier_get_stats(gda_proxy_barrier_t* b, gda_proxy_stats_t* out) {
  if (!b || !out) return -1;
  cudaDeviceSynchronize();
  std::memset(out, 0, sizeof(*out));
  out->barriers_completed = b->barrier ? b->barrier->count() : 0;
  return 0;
}

GDA_API void gda_proxy_barrier_free(gda_proxy_barrier_t* b) {
  if (!b) return;
  gda_gpu_barrier_free(b->dev_host);
  delete b;
}
