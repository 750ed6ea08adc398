// gicc_jacobi -- the Jacobi example program: 2-D 5-point stencil, fp32, rows split over
// the ranks, halo rows pushed over NVLink by the stencil kernel itself (ops::jacobi_step),
// with the command line of the reference's examples/gicc/jacobi.cu (-niter, -nccheck, -nx,
// -ny, -csv, -skip_verify).  Verification: rank 0 runs the same iterations on the whole
// grid on its own GPU; every rank hashes its owned rows and rank 0 compares the hashes with
// those of the matching rows of its single-GPU field (the update is bit-reproducible, so
// the comparison is exact).
//
//   python -m opengda_b200.parallel.launch -n 8 opengda_b200/bin/gicc_jacobi -nx 8192 -ny 8192 -niter 1000
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "gicc/coll.hpp"
#include "gicc/host_util.hpp"
#include "gicc/ops.hpp"
#include "gicc/runtime.hpp"

namespace {

int arg_int(int argc, char** argv, const char* name, int def) {
  for (int i = 1; i + 1 < argc; ++i)
    if (!std::strcmp(argv[i], name)) return std::atoi(argv[i + 1]);
  return def;
}
bool arg_flag(int argc, char** argv, const char* name) {
  for (int i = 1; i < argc; ++i)
    if (!std::strcmp(argv[i], name)) return true;
  return false;
}

void split_rows(int ny, int world, int rank, int* rows, int* g0) {
  const int interior = ny - 2, base = interior / world, extra = interior % world;
  *rows = base + (rank < extra ? 1 : 0);
  *g0 = 1 + rank * base + (rank < extra ? rank : extra);
}

uint64_t fnv1a(const void* p, size_t n) {
  const uint8_t* b = static_cast<const uint8_t*>(p);
  uint64_t h = 1469598103934665603ull;
  for (size_t i = 0; i < n; ++i) h = (h ^ b[i]) * 1099511628211ull;
  return h;
}

}  // namespace

int main(int argc, char** argv) {
  const int niter = arg_int(argc, argv, "-niter", 1000);
  const int nccheck = arg_int(argc, argv, "-nccheck", 0);
  const int nx = arg_int(argc, argv, "-nx", 8192);
  const int ny = arg_int(argc, argv, "-ny", 8192);
  const bool csv = arg_flag(argc, argv, "-csv");
  const bool skip_verify = arg_flag(argc, argv, "-skip_verify");
  const uint64_t seed = 3;
  try {
    if (nx % 4 || nx < 8 || ny < 3) throw std::runtime_error("need nx % 4 == 0, nx >= 8, ny >= 3");
    gicc::Runtime rt;
    const int rank = rt.rank(), n = rt.size();
    int rows = 0, g0 = 0;
    split_rows(ny, n, rank, &rows, &g0);
    if (rows < 1) throw std::runtime_error("more ranks than interior rows");
    std::vector<int> nrows(n);
    for (int q = 0; q < n; ++q) {
      int gq;
      split_rows(ny, n, q, &nrows[q], &gq);
    }
    const size_t field_bytes = (size_t)(rows + 2) * nx * sizeof(float);
    gicc::Buffer buf[2] = {rt.alloc(field_bytes), rt.alloc(field_bytes)};
    rt.exchange();
    const size_t flags = rt.signal_alloc(2);  // [0] top-halo arrivals, [1] bottom-halo arrivals
    float* a[2] = {static_cast<float*>(buf[0].ptr), static_cast<float*>(buf[1].ptr)};
    gicc::ops::jacobi_init(a[0], a[1], nx, ny, rows, g0, seed, nullptr);
    // The init writes both buffers' halo rows; no rank may push a row into a neighbour before
    // that neighbour's init has completed, or the init would overwrite it.
    GICC_CUDA(cudaDeviceSynchronize());
    rt.barrier();
    const int ctas = gicc::ops::jacobi_ctas_per_row(nx);
    double* norm = nullptr;
    GICC_CUDA(cudaMalloc(&norm, sizeof(double)));

    auto step = [&](int it, bool with_norm) {
      const int cur = it & 1;
      gicc::ops::JacobiStep st;
      st.a = a[cur];
      st.b = a[1 - cur];
      st.nx = nx;
      st.rows = rows;
      if (n > 1) {
        const int wb = buf[1 - cur].index;
        if (rank > 0) {  // first owned row -> upper neighbour's bottom halo
          st.top_dst = static_cast<float*>(rt.remote_ptr(rank - 1, wb, (size_t)(nrows[rank - 1] + 1) * nx * 4));
          st.top_sig_remote = rt.signal_peer(rank - 1, flags + 1);
          st.top_flag = rt.signal_local(flags);
        }
        if (rank < n - 1) {  // last owned row -> lower neighbour's top halo
          st.bot_dst = static_cast<float*>(rt.remote_ptr(rank + 1, wb, 0));
          st.bot_sig_remote = rt.signal_peer(rank + 1, flags);
          st.bot_flag = rt.signal_local(flags + 1);
        }
        st.wait_top = st.wait_bot = (uint64_t)it * ctas;
      }
      st.norm = with_norm ? norm : nullptr;
      st.timeout_ns = rt.timeout_ns();
      st.rank = rank;
      gicc::ops::jacobi_step(st, nullptr);
    };

    GICC_CUDA(cudaDeviceSynchronize());
    rt.barrier();
    cudaEvent_t e0, e1;
    GICC_CUDA(cudaEventCreate(&e0));
    GICC_CUDA(cudaEventCreate(&e1));
    GICC_CUDA(cudaEventRecord(e0));
    double last_norm = -1.0;
    for (int it = 0; it < niter; ++it) {
      const bool check = nccheck > 0 && ((it + 1) % nccheck == 0 || it == niter - 1);
      if (check) GICC_CUDA(cudaMemsetAsync(norm, 0, sizeof(double)));
      step(it, check);
      if (check) {
        double local = 0;
        GICC_CUDA(cudaMemcpy(&local, norm, sizeof(double), cudaMemcpyDeviceToHost));
        last_norm = std::sqrt(gicc::coll::allreduce_sum(rt.boot(), local));
        if (rank == 0 && !csv) std::printf("%5d, %0.6f\n", it + 1, last_norm);
      }
    }
    GICC_CUDA(cudaEventRecord(e1));
    GICC_CUDA(cudaEventSynchronize(e1));
    float ms = 0;
    GICC_CUDA(cudaEventElapsedTime(&ms, e0, e1));
    rt.check_device_errors();
    const double total_s = gicc::coll::allreduce_max(rt.boot(), (double)ms / 1e3);

    // verification against a single-GPU run of the whole grid on rank 0
    int ok = 1;
    if (!skip_verify) {
      std::vector<float> mine((size_t)rows * nx);
      GICC_CUDA(cudaMemcpy(mine.data(), a[niter & 1] + nx, mine.size() * 4, cudaMemcpyDeviceToHost));
      const auto hashes = rt.boot().allgather_fixed<uint64_t>(fnv1a(mine.data(), mine.size() * 4));
      if (rank == 0) {
        float *r0 = nullptr, *r1 = nullptr;
        const size_t whole = (size_t)ny * nx * sizeof(float);
        GICC_CUDA(cudaMalloc(&r0, whole));
        GICC_CUDA(cudaMalloc(&r1, whole));
        gicc::ops::jacobi_init(r0, r1, nx, ny, ny - 2, 1, seed, nullptr);
        float* rr[2] = {r0, r1};
        for (int it = 0; it < niter; ++it) {
          gicc::ops::JacobiStep st;
          st.a = rr[it & 1];
          st.b = rr[1 - (it & 1)];
          st.nx = nx;
          st.rows = ny - 2;
          st.timeout_ns = rt.timeout_ns();
          gicc::ops::jacobi_step(st, nullptr);
        }
        std::vector<float> ref((size_t)ny * nx);
        GICC_CUDA(cudaMemcpy(ref.data(), rr[niter & 1], whole, cudaMemcpyDeviceToHost));
        for (int q = 0; q < n; ++q) {
          int rq, gq;
          split_rows(ny, n, q, &rq, &gq);
          if (fnv1a(ref.data() + (size_t)gq * nx, (size_t)rq * nx * 4) != hashes[q]) {
            std::fprintf(stderr, "gicc_jacobi: rank %d's rows differ from the single-GPU run\n", q);
            ok = 0;
          }
        }
        GICC_CUDA(cudaFree(r0));
        GICC_CUDA(cudaFree(r1));
      }
      rt.boot().broadcast(ok, 0);
    }
    if (rank == 0) {
      const double glups = (double)(nx - 2) * (ny - 2) * niter / total_s / 1e9;
      if (csv) {
        std::printf("gicc_jacobi,%d,%d,%d,%d,%.6f,%.4f,%.3f,%s\n", n, nx, ny, niter, total_s,
                    total_s * 1e3 / niter, glups, skip_verify ? "skipped" : (ok ? "PASS" : "FAIL"));
      } else {
        std::printf("%dx%d, %d iterations on %d GPUs: %.4f s (%.4f ms/iter, %.2f GLU/s, max over ranks)\n", ny, nx,
                    niter, n, total_s, total_s * 1e3 / niter, glups);
        std::printf("%s\n", skip_verify ? "verification skipped" : (ok ? "PASS" : "FAIL"));
      }
    }
    GICC_CUDA(cudaFree(norm));
    rt.barrier();
    return ok ? 0 : 1;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_jacobi: %s\n", e.what());
    return 1;
  }
}
