// gda_api_example -- walks the OpenGDA C API (gda.h) end to end on 1..8 ranks and checks
// every result: memory registration, device-triggered puts and gets (one thread per
// transfer and whole-block), host-side wait / test / test_any / test_all, the device
// barrier with reset, and the proxy-barrier entry points.  The reference's examples that
// exercise the same calls: examples/put_example.cpp, test_example.cpp, mr_example.cpp,
// gda_get_bw.cpp, barrier_test.cpp, mm_hip_gda_proxy.cpp.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gda_api_example
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <vector>

#include "gda/gda.h"

#define CK(x)                                                                            \
  do {                                                                                   \
    cudaError_t e_ = (x);                                                                \
    if (e_ != cudaSuccess) {                                                             \
      std::fprintf(stderr, "rank %d: %s:%d %s\n", gda_rank(), __FILE__, __LINE__,       \
                   cudaGetErrorString(e_));                                              \
      std::exit(1);                                                                      \
    }                                                                                    \
  } while (0)

static int failures = 0;
#define EXPECT(c, msg)                                                                   \
  do {                                                                                   \
    if (!(c)) {                                                                          \
      std::fprintf(stderr, "rank %d: FAILED %s (%s:%d)\n", gda_rank(), msg, __FILE__, __LINE__); \
      ++failures;                                                                        \
    }                                                                                    \
  } while (0)

constexpr int kOps = 16;
constexpr size_t kChunk = 4096;

__global__ void fill(uint8_t* p, size_t n, int tag) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = (uint8_t)((i * 7 + tag * 31) & 0xff);
}

__global__ void count_bad(const uint8_t* p, size_t n, int tag, unsigned long long* bad) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    if (p[i] != (uint8_t)((i * 7 + tag * 31) & 0xff)) atomicAdd(bad, 1ull);
}

// one thread per transfer, each triggers and waits for its own
__global__ void trigger_and_wait(const gda_gpu_handle_t* hs, int n, int* status) {
  const int i = threadIdx.x;
  if (i < n) {
    gda_gpu_trigger(hs[i]);
    if (gda_gpu_wait(hs[i]) != 0) atomicAdd(status, 1);
  }
}

__global__ void trigger_block(gda_gpu_handle_t h) { gda_gpu_trigger_all(h); }

__global__ void trigger_one(gda_gpu_handle_t h) {
  if (threadIdx.x == 0) gda_gpu_trigger(h);
}

__global__ void barrier_loop(gda_gpu_barrier_t* b, int iters, int* status) {
  if (threadIdx.x != 0) return;
  for (int i = 0; i < iters; ++i)
    if (gda_gpu_barrier_wait(b) != 0) {
      atomicAdd(status, 1);
      return;
    }
}

__global__ void proxy_barrier_loop(gda_proxy_barrier_dev_t* b, int iters, int* status) {
  if (threadIdx.x != 0) return;
  for (int i = 0; i < iters; ++i)
    if (gda_gpu_proxy_barrier_wait(b) != 0) {
      atomicAdd(status, 1);
      return;
    }
}

static unsigned long long bad_bytes(const uint8_t* p, size_t n, int tag) {
  unsigned long long* d = nullptr;
  CK(cudaMalloc(&d, sizeof(*d)));
  CK(cudaMemset(d, 0, sizeof(*d)));
  count_bad<<<64, 256>>>(p, n, tag, d);
  unsigned long long h = 0;
  CK(cudaMemcpy(&h, d, sizeof(h), cudaMemcpyDeviceToHost));
  CK(cudaFree(d));
  return h;
}

int main() {
  if (gda_init() != 0) return 1;
  const int rank = gda_rank(), n = gda_size();
  const int right = (rank + 1) % n, left = (rank + n - 1) % n;
  uint8_t* buf = static_cast<uint8_t*>(gda_gpu_buf());
  const size_t bsz = gda_gpu_buf_size();
  if (rank == 0) std::printf("%s, %d ranks, gda_gpu_buf %zu bytes\n", gda_get_version(), n, bsz);
  int* status = nullptr;
  CK(cudaMalloc(&status, sizeof(int)));
  CK(cudaMemset(status, 0, sizeof(int)));

  // 1. memory registration
  {
    std::vector<uint8_t> host(1 << 16);
    gda_mr_t* hm = gda_register_memory(host.data(), host.size(), 0);
    void* dptr = nullptr;
    CK(cudaMalloc(&dptr, 1 << 20));
    gda_mr_t* dm = gda_register_memory(dptr, 1 << 20, 1);
    EXPECT(hm && dm, "register_memory");
    EXPECT(hm && gda_mr_get_desc(hm) == host.data(), "mr desc");
    EXPECT(hm && dm && gda_mr_get_key(hm) != gda_mr_get_key(dm), "distinct keys");
    EXPECT(gda_deregister_memory(dm) == 0 && gda_deregister_memory(hm) == 0, "deregister");
    CK(cudaFree(dptr));
  }

  // 2. per-thread puts into the right neighbour's second half
  const size_t half = bsz / 2;
  fill<<<64, 256>>>(buf, kOps * kChunk, rank);
  CK(cudaDeviceSynchronize());
  std::vector<gda_handle_t*> hs(kOps);
  std::vector<gda_gpu_handle_t> gh(kOps);
  for (int i = 0; i < kOps; ++i) {
    hs[i] = gda_put(buf + i * kChunk, kChunk, right, half + i * kChunk);
    EXPECT(hs[i] != nullptr, "gda_put");
    gh[i] = hs[i]->gpu;
  }
  EXPECT(gda_test_all(hs.data(), kOps) == 0, "nothing complete before the trigger");
  gda_gpu_handle_t* dh = nullptr;
  CK(cudaMalloc(&dh, kOps * sizeof(gda_gpu_handle_t)));
  CK(cudaMemcpy(dh, gh.data(), kOps * sizeof(gda_gpu_handle_t), cudaMemcpyHostToDevice));
  trigger_and_wait<<<1, kOps>>>(dh, kOps, status);
  for (int i = 0; i < kOps; ++i) EXPECT(gda_wait(hs[i]) == 0, "gda_wait");
  EXPECT(gda_test_all(hs.data(), kOps) == 1, "gda_test_all");
  EXPECT(gda_flush() == 0, "gda_flush");
  for (auto* h : hs) gda_free(h);
  gda_barrier();
  EXPECT(bad_bytes(buf + half, kOps * kChunk, left) == 0, "per-thread put data");

  // 3. one whole-block put of 1 MiB (second half, after the chunks)
  const size_t big = 1 << 20, boff = half + kOps * kChunk;
  fill<<<64, 256>>>(buf, big, rank + 100);
  CK(cudaDeviceSynchronize());
  gda_handle_t* hb = gda_put(buf, big, right, boff);
  trigger_block<<<1, 512>>>(hb->gpu);
  EXPECT(gda_wait(hb) == 0 && gda_test(hb) == 1, "block put complete");
  gda_free(hb);
  gda_barrier();
  EXPECT(bad_bytes(buf + boff, big, left + 100) == 0, "block put data");

  // 4. get: read the right neighbour's first chunk region into a local scratch area
  uint8_t* scratch = buf + half + kOps * kChunk + big;
  gda_barrier();
  fill<<<64, 256>>>(buf, kChunk, rank + 200);  // what the left neighbour will read from us
  gda_barrier();
  gda_handle_t* hg = gda_get(scratch, kChunk, right, 0);
  trigger_one<<<1, 32>>>(hg->gpu);
  EXPECT(gda_wait(hg) == 0, "get complete");
  CK(cudaDeviceSynchronize());
  EXPECT(bad_bytes(scratch, kChunk, right + 200) == 0, "get data");
  gda_free(hg);
  gda_barrier();

  // 5. test_any: only the third of four transfers is triggered
  {
    std::vector<gda_handle_t*> t(4);
    for (int i = 0; i < 4; ++i) t[i] = gda_put(buf + i * 64, 64, right, half + i * 64);
    int idx = -1;
    EXPECT(gda_test_any(t.data(), 4, &idx) == 0, "test_any before trigger");
    trigger_one<<<1, 32>>>(t[2]->gpu);
    EXPECT(gda_wait(t[2]) == 0, "wait third");
    EXPECT(gda_test_any(t.data(), 4, &idx) == 1 && idx == 2, "test_any finds the third");
    EXPECT(gda_test(t[0]) == 0 && gda_test_all(t.data(), 4) == 0, "others pending");
    for (int i : {0, 1, 3}) trigger_one<<<1, 32>>>(t[i]->gpu);
    CK(cudaDeviceSynchronize());
    EXPECT(gda_test_all(t.data(), 4) == 1, "all complete");
    for (auto* h : t) gda_free(h);
    gda_barrier();
  }

  // 6. device barrier, reset, more barriers
  {
    gda_gpu_barrier_t* b = gda_gpu_barrier_alloc(1000);
    EXPECT(b != nullptr, "gpu_barrier_alloc");
    gda_gpu_barrier_t* db = nullptr;
    CK(cudaMalloc(&db, sizeof(*db)));
    CK(cudaMemcpy(db, b, sizeof(*b), cudaMemcpyHostToDevice));
    barrier_loop<<<1, 32>>>(db, 1000, status);
    CK(cudaDeviceSynchronize());
    EXPECT(gda_gpu_barrier_reset(b) == 0 && b->ctx.expected_signal == 1001, "reset continues at 1001");
    CK(cudaMemcpy(db, b, sizeof(*b), cudaMemcpyHostToDevice));
    barrier_loop<<<1, 32>>>(db, 500, status);
    CK(cudaDeviceSynchronize());
    CK(cudaFree(db));
    gda_gpu_barrier_free(b);
  }

  // 7. proxy barrier
  {
    gda_proxy_barrier_t* pb = gda_proxy_barrier_alloc(64);
    gda_proxy_barrier_dev_t* dev_host = gda_proxy_barrier_get_dev(pb);
    EXPECT(pb && dev_host && gda_proxy_start(pb) == 0, "proxy barrier");
    gda_proxy_barrier_dev_t* d = nullptr;
    CK(cudaMalloc(&d, sizeof(*d)));
    CK(cudaMemcpy(d, dev_host, sizeof(*d), cudaMemcpyHostToDevice));
    proxy_barrier_loop<<<1, 32>>>(d, 100, status);
    CK(cudaDeviceSynchronize());
    gda_proxy_stop(pb);
    gda_proxy_stats_t st;
    EXPECT(gda_proxy_barrier_get_stats(pb, &st) == 0 && st.barriers_completed == 100 && st.total_rearms == 0,
           "proxy stats");
    CK(cudaFree(d));
    gda_proxy_barrier_free(pb);
  }

  int hst = 0;
  CK(cudaMemcpy(&hst, status, sizeof(int), cudaMemcpyDeviceToHost));
  EXPECT(hst == 0, "device-side waits and barriers");
  CK(cudaFree(status));
  CK(cudaFree(dh));
  gda_barrier();
  std::printf("rank %d: %s\n", rank, failures == 0 ? "PASS" : "FAIL");
  gda_finalize();
  return failures == 0 ? 0 : 1;
}
