// gicc_coll_test -- the bootstrap's host collectives from C++ (no GPU needed): scalar
// allreduce sum / min / max (gicc/coll.hpp), allgather, broadcast and a ring sendrecv.
//
//   python -m opengda_b200.parallel.launch -n 4 opengda_b200/bin/gicc_coll_test
#include <cstdio>
#include <string>

#include "gicc/bootstrap.hpp"
#include "gicc/coll.hpp"

int main() {
  try {
    gicc::Bootstrap boot;
    const int r = boot.rank(), n = boot.size();
    int bad = 0;
    bad += gicc::coll::allreduce_sum(boot, (long long)r + 1) != (long long)n * (n + 1) / 2;
    bad += gicc::coll::allreduce_min(boot, 10.0 * r - 3.0) != -3.0;
    bad += gicc::coll::allreduce_max(boot, 10.0 * r - 3.0) != 10.0 * (n - 1) - 3.0;
    auto all = boot.allgather_fixed<int>(r * r);
    for (int q = 0; q < n; ++q) bad += all[q] != q * q;
    double v = r == n - 1 ? 2.5 : 0.0;
    boot.broadcast(v, n - 1);
    bad += v != 2.5;
    int right = (r + 1) % n, left = (r + n - 1) % n, got = -1;
    boot.sendrecv(&r, sizeof(r), right, &got, sizeof(got), left, 3);
    bad += got != left;
    boot.barrier();
    std::printf("rank %d of %d: %s\n", r, n, bad ? "FAIL" : "PASS");
    return bad ? 1 : 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "gicc_coll_test: %s\n", e.what());
    return 1;
  }
}
