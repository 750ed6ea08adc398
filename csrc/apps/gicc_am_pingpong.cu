// gicc_am_pingpong -- active-message round-trip latency between ranks 0 and 1, the
// counterpart of the reference's examples/ofi/am_pingpong.cpp (request/reply with a 64-byte
// request and an 8-byte reply, and request/request with 64 bytes both ways; command line
// `[n_batches] [warmup]` as there).  Both sides run on the GPU (ops::am_pingpong): each batch
// is one kernel per rank doing `rtts` round trips, timed with %globaltimer on rank 0; the
// report is mean / min / p50 / p99 of the per-round-trip time over the batches.
//
//   python -m opengda_b200.parallel.launch -n 2 opengda_b200/bin/gicc_am_pingpong [n_batches] [warmup] [rtts]
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "gicc/am.hpp"
#include "gicc/host_util.hpp"
#include "gicc/runtime.hpp"

int main(int argc, char** argv) {
  const int batches = argc > 1 ? std::atoi(argv[1]) : 100;
  const int warmup = argc > 2 ? std::atoi(argv[2]) : 10;
  const int rtts = argc > 3 ? std::atoi(argv[3]) : 10;
  try {
    gicc::Runtime rt;
    const int r = rt.rank(), n = rt.size();
    if (n < 2) throw std::runtime_error("gicc_am_pingpong needs 2 ranks");
    if (batches < 1 || warmup < 0 || rtts < 1) throw std::runtime_error("need n_batches >= 1, warmup >= 0, rtts >= 1");
    gicc::am::Am am(rt, 128, 0);
    unsigned long long* ns = nullptr;
    GICC_CUDA(cudaMalloc(&ns, sizeof(*ns)));
    const char* names[2] = {"request/reply", "request/request"};
    for (int mode = 0; mode < 2; ++mode) {
      std::vector<double> us;
      for (int b = 0; b < warmup + batches; ++b) {
        rt.barrier();
        if (r < 2) gicc::ops::am_pingpong(am.device_view(), 1 - r, rtts, mode, r == 0, ns, nullptr);
        GICC_CUDA(cudaDeviceSynchronize());
        if (b >= warmup && r == 0) {
          unsigned long long v = 0;
          GICC_CUDA(cudaMemcpy(&v, ns, sizeof(v), cudaMemcpyDeviceToHost));
          us.push_back((double)v / 1e3 / rtts);
        }
      }
      rt.check_device_errors();
      if (r == 0) {
        std::sort(us.begin(), us.end());
        double mean = 0;
        for (double x : us) mean += x;
        mean /= us.size();
        auto pct = [&](double p) { return us[std::min(us.size() - 1, (size_t)(p * (us.size() - 1) + 0.5))]; };
        std::printf("%-16s round trip: mean %.3f us  min %.3f  p50 %.3f  p99 %.3f  (half: p50 %.3f us)\n", names[mode],
                    mean, us.front(), pct(0.5), pct(0.99), pct(0.5) / 2);
      }
    }
    GICC_CUDA(cudaFree(ns));
    rt.barrier();
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_am_pingpong: %s\n", e.what());
    return 1;
  }
}
