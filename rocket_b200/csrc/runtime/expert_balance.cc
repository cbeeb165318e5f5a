#include "expert_balance.h"

#include <algorithm>
#include <numeric>
#include <stdexcept>

namespace rkt_rt {

ExpertPlacement balance_experts(const std::vector<int64_t>& hist, int ranks) {
  const int E = (int)hist.size();
  if (ranks <= 0 || E % ranks) throw std::invalid_argument("balance_experts: experts must divide ranks");
  const int cap = E / ranks;
  std::vector<int32_t> ids(E);
  std::iota(ids.begin(), ids.end(), 0);
  std::stable_sort(ids.begin(), ids.end(), [&](int a, int b) { return hist[a] > hist[b]; });
  ExpertPlacement p;
  p.owner.assign(E, -1);
  p.rank_load.assign(ranks, 0);
  std::vector<int> used(ranks, 0);
  std::vector<std::vector<int32_t>> per(ranks);
  for (int e : ids) {
    int best = -1;
    for (int r = 0; r < ranks; ++r) {
      if (used[r] == cap) continue;
      if (best < 0 || p.rank_load[r] < p.rank_load[best]) best = r;
    }
    p.owner[e] = best;
    p.rank_load[best] += hist[e];
    ++used[best];
    per[best].push_back(e);
  }
  for (int r = 0; r < ranks; ++r) {
    std::sort(per[r].begin(), per[r].end());
    p.order.insert(p.order.end(), per[r].begin(), per[r].end());
  }
  return p;
}

}  // namespace rkt_rt
