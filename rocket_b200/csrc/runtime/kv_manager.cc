#include "kv_manager.h"

#include <algorithm>
#include <string>

namespace rkt_rt {

// ------------------------------------------------------------------ PagePool
PagePool::PagePool(int num_pages)
    : ref_(num_pages, 0), key_(num_pages, 0), has_key_(num_pages, 0), lru_pos_(num_pages), in_lru_(num_pages, 0) {
  free_.reserve(num_pages);
  for (int p = num_pages - 1; p >= 0; --p) free_.push_back(p);
}

int PagePool::num_free() const { return (int)(free_.size() + lru_.size()); }

int PagePool::alloc(uint64_t* evicted_key) {
  if (evicted_key) *evicted_key = 0;
  int p;
  if (!free_.empty()) {
    p = free_.back();
    free_.pop_back();
  } else if (!lru_.empty()) {
    p = lru_.front();
    lru_.pop_front();
    in_lru_[p] = 0;
    if (evicted_key) *evicted_key = key_[p];
    has_key_[p] = 0;
  } else {
    return -1;
  }
  ref_[p] = 1;
  return p;
}

void PagePool::incref(int p) {
  if (ref_.at(p) == 0 && in_lru_[p]) {
    lru_.erase(lru_pos_[p]);
    in_lru_[p] = 0;
  }
  ++ref_[p];
}

void PagePool::decref(int p) {
  if (ref_.at(p) <= 0) throw std::runtime_error("PagePool: decref of free page " + std::to_string(p));
  if (--ref_[p] == 0) {
    if (has_key_[p]) {
      lru_.push_back(p);
      lru_pos_[p] = std::prev(lru_.end());
      in_lru_[p] = 1;
    } else {
      free_.push_back(p);
    }
  }
}

void PagePool::set_key(int p, uint64_t key) {
  key_.at(p) = key;
  has_key_[p] = 1;
}

// ------------------------------------------------------------------ PrefixTree
uint64_t PrefixTree::block_key(uint64_t parent, const int32_t* tokens, int n) {
  uint64_t h = parent ^ 0xcbf29ce484222325ull;
  for (int i = 0; i < n; ++i) {
    uint32_t t = (uint32_t)tokens[i];
    for (int b = 0; b < 4; ++b) {
      h ^= (t >> (8 * b)) & 0xff;
      h *= 0x100000001b3ull;
    }
  }
  return h ? h : 1;  // 0 means "no key"
}

// ------------------------------------------------------------------ KvManager
KvManager::KvManager(int num_pages, int page_size, int max_pages_per_seq, bool prefix_cache)
    : pool_(num_pages), page_size_(page_size), max_pages_(max_pages_per_seq), prefix_cache_(prefix_cache) {
  if (page_size <= 0 || num_pages <= 0) throw std::invalid_argument("KvManager: bad geometry");
}

int KvManager::alloc_page() {
  uint64_t ev = 0;
  const int p = pool_.alloc(&ev);
  if (p < 0) throw std::runtime_error("KvManager: out of KV pages");
  if (ev) tree_.erase(ev);
  return p;
}

int KvManager::open(int64_t seq, const std::vector<int32_t>& tokens) {
  if (seqs_.count(seq)) throw std::invalid_argument("KvManager: sequence already open");
  Seq s;
  int cached = 0;
  if (prefix_cache_) {
    // reuse whole cached pages, but always leave >= 1 token to compute
    uint64_t parent = 0;
    const int full = ((int)tokens.size() - 1) / page_size_;
    for (int b = 0; b < full; ++b) {
      const uint64_t k = PrefixTree::block_key(parent, tokens.data() + b * page_size_, page_size_);
      ++lookups_;
      const int p = tree_.find(k);
      if (p < 0) break;
      ++hits_;
      pool_.incref(p);
      s.pages.push_back(p);
      s.keys.push_back(k);
      parent = k;
      cached += page_size_;
    }
  }
  s.tokens.assign(tokens.begin(), tokens.begin() + cached);
  seqs_.emplace(seq, std::move(s));
  return cached;
}

int KvManager::pages_needed(int64_t seq, int n) const {
  const Seq& s = seqs_.at(seq);
  const int len = (int)s.tokens.size();
  const int need = (len + n + page_size_ - 1) / page_size_;
  return std::max(0, need - (int)s.pages.size());
}

bool KvManager::can_append(int64_t seq, int n) const {
  const Seq& s = seqs_.at(seq);
  const int need = (int)s.pages.size() + pages_needed(seq, n);
  return need <= max_pages_ && pages_needed(seq, n) <= pool_.num_free();
}

std::vector<int32_t> KvManager::append(int64_t seq, const std::vector<int32_t>& tokens) {
  Seq& s = seqs_.at(seq);
  std::vector<int32_t> slots;
  slots.reserve(tokens.size());
  for (int32_t t : tokens) {
    const int len = (int)s.tokens.size();
    const int pi = len / page_size_;
    if (pi >= (int)s.pages.size()) {
      if ((int)s.pages.size() >= max_pages_) throw std::runtime_error("KvManager: sequence exceeds max pages");
      s.pages.push_back(alloc_page());
    }
    slots.push_back(s.pages[pi] * page_size_ + len % page_size_);
    s.tokens.push_back(t);
  }
  return slots;
}

std::vector<CopyOp> KvManager::truncate(int64_t seq, int len) {
  Seq& s = seqs_.at(seq);
  std::vector<CopyOp> ops;
  if (len >= (int)s.tokens.size()) return ops;
  s.tokens.resize(len);
  const int keep_pages = (len + page_size_ - 1) / page_size_;
  while ((int)s.pages.size() > keep_pages) {
    pool_.decref(s.pages.back());
    s.pages.pop_back();
  }
  const int sealed = len / page_size_;
  if (sealed < (int)s.pages.size()) {
    // the partial page `sealed` will be written again: it must be private (copy-on-write
    // when a prefix hit or a fork shares it) and must leave the prefix index
    const int p = s.pages[sealed];
    if (pool_.refcount(p) > 1) {
      const int np = alloc_page();
      ops.push_back({p, np});
      pool_.decref(p);
      s.pages[sealed] = np;
    } else if (pool_.cached(p)) {
      tree_.erase(pool_.key(p));
      pool_.clear_key(p);
    }
  }
  if ((int)s.keys.size() > sealed) s.keys.resize(sealed);
  return ops;
}

std::vector<CopyOp> KvManager::fork(int64_t parent, int64_t child) {
  if (seqs_.count(child)) throw std::invalid_argument("KvManager: child already open");
  const Seq& ps = seqs_.at(parent);
  Seq cs;
  cs.tokens = ps.tokens;
  cs.keys = ps.keys;
  std::vector<CopyOp> ops;
  const int full = (int)ps.tokens.size() / page_size_;
  for (int i = 0; i < (int)ps.pages.size(); ++i) {
    if (i < full) {
      pool_.incref(ps.pages[i]);
      cs.pages.push_back(ps.pages[i]);
    } else {
      const int np = alloc_page();
      ops.push_back({ps.pages[i], np});
      cs.pages.push_back(np);
    }
  }
  seqs_.emplace(child, std::move(cs));
  return ops;
}

void KvManager::free(int64_t seq) {
  auto it = seqs_.find(seq);
  if (it == seqs_.end()) return;
  for (int p : it->second.pages) pool_.decref(p);
  seqs_.erase(it);
}

void KvManager::commit_prefix(int64_t seq) {
  if (!prefix_cache_) return;
  Seq& s = seqs_.at(seq);
  const int full = (int)s.tokens.size() / page_size_;
  uint64_t parent = s.keys.empty() ? 0 : s.keys.back();
  for (int b = (int)s.keys.size(); b < full; ++b) {
    const uint64_t k = PrefixTree::block_key(parent, s.tokens.data() + b * page_size_, page_size_);
    s.keys.push_back(k);
    parent = k;
    if (tree_.find(k) < 0) {
      tree_.insert(k, s.pages[b]);
      pool_.set_key(s.pages[b], k);
    }
  }
}

void KvManager::block_table(const std::vector<int64_t>& seqs, int32_t* out, int max_pages) const {
  for (size_t i = 0; i < seqs.size(); ++i) {
    const Seq& s = seqs_.at(seqs[i]);
    int32_t* row = out + i * max_pages;
    const int n = std::min((int)s.pages.size(), max_pages);
    for (int j = 0; j < n; ++j) row[j] = s.pages[j];
    for (int j = n; j < max_pages; ++j) row[j] = 0;
  }
}

std::vector<uint64_t> KvManager::block_keys(const std::vector<int32_t>& tokens) const {
  std::vector<uint64_t> keys;
  uint64_t parent = 0;
  for (int b = 0; (b + 1) * page_size_ <= (int)tokens.size(); ++b) {
    parent = PrefixTree::block_key(parent, tokens.data() + b * page_size_, page_size_);
    keys.push_back(parent);
  }
  return keys;
}

int KvManager::cached_prefix_blocks(const std::vector<uint64_t>& keys) const {
  int n = 0;
  while (n < (int)keys.size() && tree_.find(keys[n]) >= 0) ++n;
  return n;
}

int KvManager::import_block(uint64_t key) {
  if (!prefix_cache_ || tree_.find(key) >= 0) return -1;
  uint64_t ev = 0;
  const int p = pool_.alloc(&ev);
  if (p < 0) return -1;
  if (ev) tree_.erase(ev);
  pool_.set_key(p, key);
  tree_.insert(key, p);
  pool_.decref(p);  // reference 0 with a key: cached and evictable
  return p;
}

std::vector<std::pair<uint64_t, int>> KvManager::sealed_blocks(int64_t seq) const {
  const Seq& s = seqs_.at(seq);
  std::vector<std::pair<uint64_t, int>> out;
  for (size_t i = 0; i < s.keys.size(); ++i) out.emplace_back(s.keys[i], s.pages[i]);
  return out;
}

}  // namespace rkt_rt
