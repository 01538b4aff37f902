// Expert-tier bookkeeping in C++ (the reference's `tier` crate role): a byte-range arena that
// sub-allocates one VRAM slab (staging banks, prefetch slots) and the residency planner that
// picks (cold resident, hot host) swaps from decayed-LFU scores with hysteresis.
// Reference: crates/tier (expert-cache slot table, decayed LFU, arenas); RFC-0023 §5.
#include <torch/extension.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <utility>
#include <vector>

namespace syn {

// First-fit arena over [0, capacity) with coalescing free list; offsets, no memory of its own.
class Arena {
 public:
  explicit Arena(int64_t capacity) : cap_(capacity) { free_[0] = capacity; }

  int64_t alloc(int64_t bytes, int64_t align) {
    TORCH_CHECK(bytes > 0 && align > 0 && (align & (align - 1)) == 0, "arena: bytes > 0, power-of-two align");
    for (auto it = free_.begin(); it != free_.end(); ++it) {
      const int64_t start = it->first, len = it->second;
      const int64_t a = (start + align - 1) & ~(align - 1);
      if (a + bytes > start + len) continue;
      free_.erase(it);
      if (a > start) free_[start] = a - start;
      if (a + bytes < start + len) free_[a + bytes] = start + len - (a + bytes);
      used_[a] = bytes;
      return a;
    }
    return -1;
  }

  void release(int64_t off) {
    auto it = used_.find(off);
    TORCH_CHECK(it != used_.end(), "arena: offset ", off, " is not allocated");
    int64_t start = off, len = it->second;
    used_.erase(it);
    auto nx = free_.lower_bound(start);
    if (nx != free_.end() && nx->first == start + len) {  // merge with the next free range
      len += nx->second;
      nx = free_.erase(nx);
    }
    if (nx != free_.begin()) {
      auto pv = std::prev(nx);
      if (pv->first + pv->second == start) {  // merge with the previous free range
        pv->second += len;
        return;
      }
    }
    free_[start] = len;
  }

  int64_t used() const {
    int64_t u = 0;
    for (auto& kv : used_) u += kv.second;
    return u;
  }
  int64_t capacity() const { return cap_; }
  int64_t largest_free() const {
    int64_t m = 0;
    for (auto& kv : free_) m = std::max(m, kv.second);
    return m;
  }

 private:
  int64_t cap_;
  std::map<int64_t, int64_t> free_, used_;
};

// Swap plan for one layer: repeatedly pair the coldest resident with the hottest host expert
// while hot > hysteresis * cold and hot > 0 (at most max_swaps pairs).  Ties: lower index.
std::vector<std::pair<int64_t, int64_t>> tier_plan_swaps(std::vector<double> score, std::vector<bool> resident,
                                                        int64_t max_swaps, double hysteresis) {
  TORCH_CHECK(score.size() == resident.size(), "score / resident sizes differ");
  std::vector<std::pair<int64_t, int64_t>> out;
  const int64_t E = (int64_t)score.size();
  for (int64_t k = 0; k < max_swaps; ++k) {
    int64_t cold = -1, hot = -1;
    for (int64_t e = 0; e < E; ++e) {
      if (resident[e]) {
        if (cold < 0 || score[e] < score[cold]) cold = e;
      } else {
        if (hot < 0 || score[e] > score[hot]) hot = e;
      }
    }
    if (cold < 0 || hot < 0) break;
    if (!(score[hot] > hysteresis * score[cold]) || score[hot] <= 0.0) break;
    out.emplace_back(cold, hot);
    resident[cold] = false;
    resident[hot] = true;
  }
  return out;
}

void register_tier(pybind11::module& m) {
  pybind11::class_<Arena>(m, "Arena")
      .def(pybind11::init<int64_t>())
      .def("alloc", &Arena::alloc)
      .def("release", &Arena::release)
      .def("used", &Arena::used)
      .def("capacity", &Arena::capacity)
      .def("largest_free", &Arena::largest_free);
  m.def("tier_plan_swaps", &tier_plan_swaps, "decayed-LFU residency swaps with hysteresis");
}

}  // namespace syn
