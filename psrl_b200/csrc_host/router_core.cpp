// Native core of the rollout router (the role of the reference's Rust SMG
// router, psrl/workers/gen/smg_adapter.py:47-153): per-instance prefix indexes
// for cache-aware routing and the load-based policy choices, on plain arrays so
// a routing decision makes no Python-object allocations.
//
//  PrefixIndex   LRU set of block-hash chains of recently routed prompts.  The
//                chain hash of block i mixes the previous chain hash with the
//                block's token ids (SplitMix64 finaliser, Steele et al. 2014),
//                so a match of i blocks means the first i * block_size tokens
//                agree (up to 64-bit collisions).
//  pick          policy over candidate instances: round_robin, request_num_balance
//                (fewest running + waiting, then KV usage), throughput_optimal
//                (largest marginal tokens/s of the fitted curve
//                A (1 - (B x + 1)^-k)), and cache_aware (longest prefix match
//                unless the load imbalance exceeds the absolute and relative
//                thresholds, then the least loaded).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cmath>
#include <stdexcept>
#include <cstdint>
#include <list>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

inline uint64_t mix64(uint64_t z) {
  z += 0x9e3779b97f4a7c15ull;
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

class PrefixIndex {
 public:
  PrefixIndex(int block_size, size_t max_entries) : bs_(block_size), max_(max_entries) {}

  std::vector<uint64_t> chain(py::array_t<int64_t, py::array::c_style | py::array::forcecast> tokens) const {
    auto t = tokens.unchecked<1>();
    const int64_t n = t.shape(0) / bs_;
    std::vector<uint64_t> out;
    out.reserve(n);
    uint64_t h = 0;
    for (int64_t i = 0; i < n; ++i) {
      for (int j = 0; j < bs_; ++j) h = mix64(h ^ (uint64_t)t(i * bs_ + j));
      out.push_back(h);
    }
    return out;
  }

  // tokens of the longest indexed prefix (whole blocks); touches matched entries
  int64_t match(py::array_t<int64_t, py::array::c_style | py::array::forcecast> tokens) {
    int64_t n = 0;
    for (uint64_t h : chain(tokens)) {
      auto it = map_.find(h);
      if (it == map_.end()) break;
      lru_.splice(lru_.end(), lru_, it->second);
      ++n;
    }
    return n * bs_;
  }

  void insert(py::array_t<int64_t, py::array::c_style | py::array::forcecast> tokens) {
    for (uint64_t h : chain(tokens)) {
      auto it = map_.find(h);
      if (it != map_.end()) {
        lru_.splice(lru_.end(), lru_, it->second);
      } else {
        lru_.push_back(h);
        map_[h] = std::prev(lru_.end());
      }
    }
    while (map_.size() > max_) {
      map_.erase(lru_.front());
      lru_.pop_front();
    }
  }

  size_t size() const { return map_.size(); }

 private:
  int bs_;
  size_t max_;
  std::list<uint64_t> lru_;
  std::unordered_map<uint64_t, std::list<uint64_t>::iterator> map_;
};

struct Curve {
  double A, B, k;
  double rate(double x) const { return A * (1.0 - std::pow(B * x + 1.0, -k)); }
  double marginal(double x) const { return rate(x + 1) - rate(x); }
};

// Index into the candidate arrays of the chosen instance (-1 if none).
int pick(const std::string& method, const std::vector<int64_t>& load, const std::vector<double>& kv_usage,
         const std::vector<int64_t>& prefix_match, int64_t rr_counter, int64_t request_budget,
         int64_t balance_abs, double balance_rel, double A, double B, double k) {
  const int n = (int)load.size();
  if (n == 0) return -1;
  if (method == "round_robin") return (int)(rr_counter % n);
  auto least_loaded = [&]() {
    int best = 0;
    for (int i = 1; i < n; ++i)
      if (load[i] < load[best] || (load[i] == load[best] && kv_usage[i] < kv_usage[best])) best = i;
    return best;
  };
  if (method == "request_num_balance") return least_loaded();
  if (method == "throughput_optimal" || method == "throughput_optimal_with_budget") {
    Curve c{A, B, k};
    bool any_under = false;
    if (method == "throughput_optimal_with_budget")
      for (int i = 0; i < n; ++i) any_under |= load[i] < request_budget;
    int best = -1;
    double bv = -1e300;
    for (int i = 0; i < n; ++i) {
      if (any_under && load[i] >= request_budget) continue;
      const double v = c.marginal((double)load[i]);
      if (v > bv) {
        bv = v;
        best = i;
      }
    }
    return best;
  }
  if (method == "cache_aware" || method == "cache_aware_v1") {
    int64_t lo = load[0], hi = load[0];
    for (int i = 1; i < n; ++i) {
      lo = std::min(lo, load[i]);
      hi = std::max(hi, load[i]);
    }
    if (hi - lo > balance_abs && (double)hi > balance_rel * (double)std::max<int64_t>(lo, 1)) {
      int best = 0;
      for (int i = 1; i < n; ++i)
        if (load[i] < load[best]) best = i;
      return best;
    }
    int best = 0;
    for (int i = 1; i < n; ++i)
      if (prefix_match[i] > prefix_match[best] || (prefix_match[i] == prefix_match[best] && load[i] < load[best]))
        best = i;
    return best;
  }
  throw std::invalid_argument("unknown routing policy " + method);
}

}  // namespace

PYBIND11_MODULE(_router, m) {
  m.doc() = "native rollout-router core";
  py::class_<PrefixIndex>(m, "PrefixIndex")
      .def(py::init<int, size_t>(), py::arg("block_size") = 16, py::arg("max_entries") = 1 << 16)
      .def("match", &PrefixIndex::match)
      .def("insert", &PrefixIndex::insert)
      .def("chain", &PrefixIndex::chain)
      .def("__len__", &PrefixIndex::size);
  m.def("pick", &pick);
}
