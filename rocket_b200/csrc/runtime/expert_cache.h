// Streamed routed experts: a bounded set of device slots per MoE layer, filled from
// host memory on demand, least recently used slot evicted first.
//
// plan(needed) partitions the experts one step routes to into passes of at most
// `num_slots` experts.  Resident experts go into the first pass (no copy); missing
// experts take free slots, then the least recently used slots that the pass does
// not use.  Each pass gives the expert -> slot map the routing plan is rewritten
// with (-1 = not in this pass) and the (expert, slot) copies the caller issues
// before the pass's GEMMs.  Copies and GEMMs run in stream order, so a later pass
// may reuse a slot that an earlier pass read.
//
// Behavioural counterpart of the streamed half of the reference's weight store
// (engines/glm5-moe-nvfp4-2b/src/weights.h:1-16, ExpertDev / WeightStore :149-204):
// a bounded device LRU of expert slots.  The pass split and the data structures
// here are this build's own.
#pragma once
#include <cstdint>
#include <utility>
#include <vector>

namespace rkt_rt {

struct ExpertPass {
  std::vector<int32_t> remap;                    // [num_experts]: slot, or -1
  std::vector<std::pair<int32_t, int32_t>> loads;  // (expert, slot) host -> device copies
};

class ExpertSlotCache {
 public:
  ExpertSlotCache(int num_experts, int num_slots);
  std::vector<ExpertPass> plan(const std::vector<int32_t>& needed);
  int num_experts() const { return (int)slot_of_.size(); }
  int num_slots() const { return (int)expert_in_.size(); }
  int slot_of(int e) const { return slot_of_.at(e); }
  int expert_in(int s) const { return expert_in_.at(s); }
  void reset();
  uint64_t hits() const { return hits_; }
  uint64_t misses() const { return misses_; }
  uint64_t evictions() const { return evictions_; }
  uint64_t passes() const { return passes_; }

 private:
  int take_slot(const std::vector<uint8_t>& pinned);
  std::vector<int32_t> slot_of_;    // expert -> slot or -1
  std::vector<int32_t> expert_in_;  // slot -> expert or -1
  std::vector<uint64_t> last_use_;  // slot -> tick of last use
  uint64_t tick_ = 0, hits_ = 0, misses_ = 0, evictions_ = 0, passes_ = 0;
};

}  // namespace rkt_rt
