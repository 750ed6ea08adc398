// gicc_put_bw -- one-sided put and get bandwidth from rank 0 to rank 1 over a size sweep
// (8 B .. 256 MiB by default), the counterpart of the reference's put-bandwidth programs
// (examples/gda_put_bw.cpp: a window of puts triggered from the GPU per iteration;
// examples/ofi/benchmark.cpp: a byte pattern that is unique per size, so a partial or
// missing write shows up without re-initialising the receiver).
//
// Each window is one kernel: `window` messages of `size` bytes into the same region of the
// peer's buffer (OSU style), each message split over the kernel's CTAs and copied with
// block-scope gicc::put (16-byte stores over NVLink), then a fence so the kernel ends when
// the data is delivered.  Bandwidth = iters * window * size / device time.  After each size
// rank 1 checks every byte of the region against rank 0's pattern on its own GPU; the get
// pass reads rank 1's buffer back into rank 0 and checks it there.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gicc_put_bw [-min 8] [-max 268435456]
//       [-window 64] [-iters 10] [-csv]
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "gicc/coll.hpp"
#include "gicc/device/comm.cuh"
#include "gicc/host_util.hpp"
#include "gicc/runtime.hpp"

namespace {

long long arg_ll(int argc, char** argv, const char* name, long long def) {
  for (int i = 1; i + 1 < argc; ++i)
    if (!std::strcmp(argv[i], name)) return std::atoll(argv[i + 1]);
  return def;
}
bool arg_flag(int argc, char** argv, const char* name) {
  for (int i = 1; i < argc; ++i)
    if (!std::strcmp(argv[i], name)) return true;
  return false;
}

__host__ __device__ inline uint8_t pattern(size_t i, size_t size) { return (uint8_t)((i * 131u + size * 7u + 0xA0u) & 0xFF); }

__global__ void fill(uint8_t* p, size_t n, size_t size) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    p[i] = pattern(i, size);
}

__global__ void check(const uint8_t* p, size_t n, size_t size, unsigned long long* bad) {
  unsigned long long mine = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    mine += p[i] != pattern(i, size);
  if (mine) atomicAdd(bad, mine);
}

// `window` messages of `size` bytes from src to dst; CTA b copies bytes [b*chunk, ...) of
// each message.  get = true reads a remote src into a local dst.
__global__ void __launch_bounds__(512) window_kernel(uint8_t* dst, const uint8_t* src, size_t size, int window,
                                                    bool get) {
  const size_t chunk = ((size + gridDim.x - 1) / gridDim.x + 15) & ~size_t(15);
  const size_t lo = (size_t)blockIdx.x * chunk;
  if (lo < size) {
    const size_t n = size - lo < chunk ? size - lo : chunk;
    for (int w = 0; w < window; ++w) {
      if (get)
        gicc::get<gicc::Scope::Block>(dst + lo, src + lo, n);
      else
        gicc::put<gicc::Scope::Block>(dst + lo, src + lo, n);
    }
  }
  gicc::quiet();
}

}  // namespace

int main(int argc, char** argv) {
  const size_t min_size = (size_t)arg_ll(argc, argv, "-min", 8);
  const size_t max_size = (size_t)arg_ll(argc, argv, "-max", 256ll << 20);
  const int window_arg = (int)arg_ll(argc, argv, "-window", 64);
  const int iters = (int)arg_ll(argc, argv, "-iters", 10);
  const bool csv = arg_flag(argc, argv, "-csv");
  try {
    gicc::Runtime rt;
    const int r = rt.rank(), n = rt.size();
    if (n < 2) throw std::runtime_error("gicc_put_bw needs 2 ranks");
    if (min_size < 1 || max_size < min_size) throw std::runtime_error("need 1 <= -min <= -max");
    gicc::Buffer buf = rt.alloc(max_size);
    rt.exchange();
    uint8_t* src = nullptr;
    unsigned long long* bad = nullptr;
    GICC_CUDA(cudaMalloc(&src, max_size));
    GICC_CUDA(cudaMalloc(&bad, sizeof(*bad)));
    cudaEvent_t e0, e1;
    GICC_CUDA(cudaEventCreate(&e0));
    GICC_CUDA(cudaEventCreate(&e1));
    uint8_t* peer = static_cast<uint8_t*>(rt.remote_ptr(1, buf.index, 0));
    uint8_t* mine = static_cast<uint8_t*>(buf.ptr);
    if (r == 0 && csv) std::printf("size,window,put_GBps,get_GBps,verify\n");
    int all_bad_total = 0;
    for (size_t size = min_size; size <= max_size; size *= 2) {
      // at most 256 MiB per window and 1 GiB per size (at least 2 timed windows), so the
      // large sizes stay short
      const int window = (int)std::max<size_t>(1, std::min<size_t>(window_arg, (256ull << 20) / size));
      const int its = (int)std::max<size_t>(2, std::min<size_t>(iters, (1ull << 30) / ((size_t)window * size)));
      const int grid = size < (64u << 10) ? 1 : gicc::num_sms();
      double put_ms = 0, get_ms = 0;
      fill<<<256, 256>>>(src, size, size);
      GICC_CUDA(cudaDeviceSynchronize());
      rt.barrier();
      if (r == 0) {  // put: rank 0 -> rank 1
        window_kernel<<<grid, 512>>>(peer, src, size, window, false);  // warm-up
        GICC_CUDA(cudaEventRecord(e0));
        for (int i = 0; i < its; ++i) window_kernel<<<grid, 512>>>(peer, src, size, window, false);
        GICC_CUDA(cudaEventRecord(e1));
        GICC_CUDA(cudaEventSynchronize(e1));
        float ms = 0;
        GICC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        put_ms = ms;
      }
      rt.barrier();
      unsigned long long nbad = 0;
      if (r == 1) {  // every byte of the region holds rank 0's pattern for this size
        GICC_CUDA(cudaMemset(bad, 0, sizeof(*bad)));
        check<<<256, 256>>>(mine, size, size, bad);
        GICC_CUDA(cudaMemcpy(&nbad, bad, sizeof(nbad), cudaMemcpyDeviceToHost));
      }
      rt.barrier();
      if (r == 0) {  // get: rank 0 reads rank 1's region (rank 0's pattern, put above) into src
        GICC_CUDA(cudaMemset(src, 0, size));
        window_kernel<<<grid, 512>>>(src, peer, size, window, true);
        GICC_CUDA(cudaEventRecord(e0));
        for (int i = 0; i < its; ++i) window_kernel<<<grid, 512>>>(src, peer, size, window, true);
        GICC_CUDA(cudaEventRecord(e1));
        GICC_CUDA(cudaEventSynchronize(e1));
        float ms = 0;
        GICC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
        get_ms = ms;
        GICC_CUDA(cudaMemset(bad, 0, sizeof(*bad)));
        check<<<256, 256>>>(src, size, size, bad);
        unsigned long long gbad = 0;
        GICC_CUDA(cudaMemcpy(&gbad, bad, sizeof(gbad), cudaMemcpyDeviceToHost));
        nbad += gbad;
      }
      rt.check_device_errors();
      const int size_bad = gicc::coll::allreduce_sum(rt.boot(), (int)(nbad != 0));
      all_bad_total += size_bad;
      if (r == 0) {
        const double bytes = (double)its * window * size;
        const double put_gbs = bytes / (put_ms * 1e-3) / 1e9, get_gbs = bytes / (get_ms * 1e-3) / 1e9;
        if (csv)
          std::printf("%zu,%d,%.3f,%.3f,%s\n", size, window, put_gbs, get_gbs, size_bad ? "FAIL" : "PASS");
        else
          std::printf("%12zu B  window %4d  put %9.3f GB/s  get %9.3f GB/s  %s\n", size, window, put_gbs, get_gbs,
                      size_bad ? "FAIL" : "PASS");
      }
      if (size > max_size / 2) break;
    }
    if (r == 0) std::printf("%s\n", all_bad_total ? "FAIL" : "PASS");
    GICC_CUDA(cudaFree(src));
    GICC_CUDA(cudaFree(bad));
    rt.barrier();
    return all_bad_total ? 1 : 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_put_bw: %s\n", e.what());
    return 1;
  }
}
