// Expert-parallel placement from an expert firing histogram (host side, C++).
//
// Equal-cardinality greedy LPT: experts sorted by load (descending, ties by id)
// are placed one by one on the least-loaded rank that still has room for
// E / ranks experts (ties by rank id).  Every rank computes the same placement
// from the same histogram, so it never has to be exchanged.
//
// Behavioural counterpart of the reference's balance_experts
// (engines/glm5-moe-nvfp4-2b/src/fabric/expert_balance.h:37-53, .cc:58-102).
#pragma once
#include <cstdint>
#include <vector>

namespace rkt_rt {

struct ExpertPlacement {
  std::vector<int32_t> owner;       // [E] rank owning expert e
  std::vector<int32_t> order;       // [E] experts grouped by rank (rank r owns order[r*E/R .. (r+1)*E/R))
  std::vector<int64_t> rank_load;   // [R] summed histogram per rank
};

ExpertPlacement balance_experts(const std::vector<int64_t>& hist, int ranks);

}  // namespace rkt_rt
