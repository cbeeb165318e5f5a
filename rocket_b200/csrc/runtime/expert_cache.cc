#include "expert_cache.h"

#include <algorithm>
#include <stdexcept>

namespace rkt_rt {

ExpertSlotCache::ExpertSlotCache(int num_experts, int num_slots) {
  if (num_experts < 1 || num_slots < 1) throw std::invalid_argument("ExpertSlotCache: experts and slots must be >= 1");
  slot_of_.assign(num_experts, -1);
  expert_in_.assign(num_slots, -1);
  last_use_.assign(num_slots, 0);
}

void ExpertSlotCache::reset() {
  std::fill(slot_of_.begin(), slot_of_.end(), -1);
  std::fill(expert_in_.begin(), expert_in_.end(), -1);
  std::fill(last_use_.begin(), last_use_.end(), 0);
}

int ExpertSlotCache::take_slot(const std::vector<uint8_t>& pinned) {
  // a free slot first, else the least recently used slot this pass does not use
  int best = -1;
  for (int s = 0; s < num_slots(); ++s) {
    if (pinned[s]) continue;
    if (expert_in_[s] < 0) return s;
    if (best < 0 || last_use_[s] < last_use_[best]) best = s;
  }
  if (best < 0) throw std::logic_error("ExpertSlotCache: no slot left in the pass");
  slot_of_[expert_in_[best]] = -1;
  expert_in_[best] = -1;
  ++evictions_;
  return best;
}

std::vector<ExpertPass> ExpertSlotCache::plan(const std::vector<int32_t>& needed_in) {
  std::vector<int32_t> needed(needed_in);
  std::sort(needed.begin(), needed.end());
  needed.erase(std::unique(needed.begin(), needed.end()), needed.end());
  for (int32_t e : needed)
    if (e < 0 || e >= num_experts()) throw std::out_of_range("ExpertSlotCache: expert id out of range");
  std::vector<int32_t> resident, missing;
  for (int32_t e : needed) (slot_of_[e] >= 0 ? resident : missing).push_back(e);
  hits_ += resident.size();
  misses_ += missing.size();
  ++tick_;
  std::vector<ExpertPass> out;
  size_t mi = 0;
  bool first = true;
  while (first || mi < missing.size()) {
    ExpertPass p;
    p.remap.assign(num_experts(), -1);
    std::vector<uint8_t> pinned(num_slots(), 0);
    int used = 0;
    if (first) {
      for (int32_t e : resident) {
        const int s = slot_of_[e];
        pinned[s] = 1;
        p.remap[e] = s;
        last_use_[s] = tick_;
        ++used;
      }
    }
    while (mi < missing.size() && used < num_slots()) {
      const int32_t e = missing[mi++];
      const int s = take_slot(pinned);
      expert_in_[s] = e;
      slot_of_[e] = s;
      pinned[s] = 1;
      last_use_[s] = tick_;
      p.remap[e] = s;
      p.loads.emplace_back(e, s);
      ++used;
    }
    out.push_back(std::move(p));
    first = false;
    ++passes_;
    ++tick_;  // slots of earlier passes age before later passes pick victims
  }
  return out;
}

}  // namespace rkt_rt
