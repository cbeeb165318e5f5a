#include "bpe.h"

#include <queue>
#include <stdexcept>
#include <tuple>

namespace rkt_rt {

BpeModel::BpeModel(const std::vector<std::pair<std::string, int32_t>>& vocab,
                   const std::vector<std::pair<std::string, std::string>>& merges, bool ignore_merges)
    : ignore_merges_(ignore_merges) {
  int32_t max_id = -1;
  for (auto& kv : vocab) {
    if (kv.second < 0) throw std::invalid_argument("bpe: negative token id");
    vocab_[kv.first] = kv.second;
    max_id = std::max(max_id, kv.second);
  }
  id_to_bytes_.assign((size_t)max_id + 1, std::string());
  for (auto& kv : vocab) id_to_bytes_[kv.second] = kv.first;
  for (int b = 0; b < 256; ++b) {
    auto it = vocab_.find(std::string(1, (char)b));
    byte_id_[b] = it == vocab_.end() ? -1 : it->second;
  }
  int32_t rank = 0;
  for (auto& m : merges) {
    auto a = vocab_.find(m.first), b = vocab_.find(m.second), ab = vocab_.find(m.first + m.second);
    if (a == vocab_.end() || b == vocab_.end() || ab == vocab_.end())
      throw std::invalid_argument("bpe: merge refers to a token outside the vocabulary");
    ranks_.emplace(std::make_pair(a->second, b->second), std::make_pair(rank++, ab->second));
  }
}

int32_t BpeModel::token_id(const std::string& bytes) const {
  auto it = vocab_.find(bytes);
  return it == vocab_.end() ? -1 : it->second;
}

std::vector<int32_t> BpeModel::encode_piece(const std::string& piece) {
  if (piece.empty()) return {};
  if (ignore_merges_) {
    auto it = vocab_.find(piece);
    if (it != vocab_.end()) return {it->second};
  }
  auto hit = cache_.find(piece);
  if (hit != cache_.end()) return hit->second;
  const int n = (int)piece.size();
  std::vector<int32_t> sym(n), prev(n), next(n);
  std::vector<uint8_t> alive(n, 1);
  for (int i = 0; i < n; ++i) {
    const int32_t id = byte_id_[(uint8_t)piece[i]];
    if (id < 0) throw std::invalid_argument("bpe: byte missing from the vocabulary");
    sym[i] = id;
    prev[i] = i - 1;
    next[i] = i + 1 < n ? i + 1 : -1;
  }
  // heap entries: (rank, left position, left symbol, right symbol); stale entries are skipped
  using E = std::tuple<int32_t, int32_t, int32_t, int32_t>;
  std::priority_queue<E, std::vector<E>, std::greater<E>> heap;
  auto push = [&](int i) {
    const int j = next[i];
    if (i < 0 || j < 0) return;
    auto it = ranks_.find({sym[i], sym[j]});
    if (it != ranks_.end()) heap.emplace(it->second.first, i, sym[i], sym[j]);
  };
  for (int i = 0; i + 1 < n; ++i) push(i);
  while (!heap.empty()) {
    auto [rk, i, a, b] = heap.top();
    heap.pop();
    const int j = alive[i] ? next[i] : -1;
    if (j < 0 || sym[i] != a || sym[j] != b) continue;  // stale
    sym[i] = ranks_.at({a, b}).second;
    alive[j] = 0;
    next[i] = next[j];
    if (next[j] >= 0) prev[next[j]] = i;
    if (prev[i] >= 0) push(prev[i]);
    push(i);
  }
  std::vector<int32_t> out;
  for (int i = 0; i >= 0; i = next[i]) out.push_back(sym[i]);
  if (cache_.size() < (1u << 16)) cache_.emplace(piece, out);
  return out;
}

std::vector<int32_t> BpeModel::encode_pieces(const std::vector<std::string>& pieces) {
  std::vector<int32_t> out;
  for (auto& p : pieces) {
    auto v = encode_piece(p);
    out.insert(out.end(), v.begin(), v.end());
  }
  return out;
}

std::string BpeModel::decode(const std::vector<int32_t>& ids) const {
  std::string s;
  for (int32_t id : ids) {
    if (id < 0 || (size_t)id >= id_to_bytes_.size()) throw std::out_of_range("bpe: token id out of range");
    s += id_to_bytes_[id];
  }
  return s;
}

}  // namespace rkt_rt
