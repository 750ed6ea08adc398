// coll.hpp -- host scalar reductions over the bootstrap (the reference's
// src/gicc/coll.hpp:15-39: gicc::coll::allreduce_sum / _min / _max on a Bootstrap).
// Every rank calls them in the same order; the result is the same on every rank.
#pragma once
#include <algorithm>

#include "gicc/bootstrap.hpp"

namespace gicc {
namespace coll {

template <class T>
T allreduce_sum(Bootstrap& boot, const T& v) {
  const std::vector<T> all = boot.allgather_fixed<T>(v);
  T acc = T();
  for (const T& x : all) acc += x;  // rank order, so every rank adds in the same order
  return acc;
}

template <class T>
T allreduce_min(Bootstrap& boot, const T& v) {
  const std::vector<T> all = boot.allgather_fixed<T>(v);
  return *std::min_element(all.begin(), all.end());
}

template <class T>
T allreduce_max(Bootstrap& boot, const T& v) {
  const std::vector<T> all = boot.allgather_fixed<T>(v);
  return *std::max_element(all.begin(), all.end());
}

}  // namespace coll
}  // namespace gicc
