// Paged KV bookkeeping for the engine (host side, C++).
//
//  PagePool    refcounted fixed-size pages; pages that hold a sealed, hashed
//              prefix block stay cached after their last reference drops and
//              are evicted least-recently-used when the free list runs dry.
//  PrefixTree  content-addressed radix index at page granularity.  The key of
//              a full page is FNV-1a-64 over its token ids seeded with the
//              parent page's key, so equal keys mean equal whole prefixes.
//  KvManager   sequences: open (with prefix reuse), append, truncate (drop
//              rejected speculative tokens), fork (share full pages; the
//              partial boundary page is copied on extend), free, block tables.
//
// Behavioural counterpart of the reference's PagePool / PrefixTree / KvCache
// (engines/glm5-moe-nvfp4-2b/src/kv/page_pool.h:41-237, page_pool.cc:32-496);
// the data structures here are this build's own.
#pragma once
#include <cstdint>
#include <list>
#include <stdexcept>
#include <unordered_map>
#include <utility>
#include <vector>

namespace rkt_rt {

class PagePool {
 public:
  explicit PagePool(int num_pages);
  int num_pages() const { return (int)ref_.size(); }
  int num_free() const;            // free + evictable cached pages
  int num_free_uncached() const { return (int)free_.size(); }
  // Returns -1 when nothing is free or evictable.  `evicted_key` is set when a
  // cached page was reclaimed (the caller drops it from its index).
  int alloc(uint64_t* evicted_key);
  void incref(int page);
  void decref(int page);
  int refcount(int page) const { return ref_.at(page); }
  void set_key(int page, uint64_t key);   // page now caches prefix block `key`
  void clear_key(int page) { has_key_.at(page) = 0; }
  uint64_t key(int page) const { return key_.at(page); }
  bool cached(int page) const { return has_key_.at(page) != 0; }

 private:
  std::vector<int> ref_;
  std::vector<uint64_t> key_;
  std::vector<uint8_t> has_key_;
  std::vector<int> free_;                       // never-cached or dropped pages
  std::list<int> lru_;                          // cached pages with ref 0, oldest first
  std::vector<std::list<int>::iterator> lru_pos_;
  std::vector<uint8_t> in_lru_;
};

class PrefixTree {
 public:
  static uint64_t block_key(uint64_t parent, const int32_t* tokens, int n);
  void insert(uint64_t key, int page) { map_[key] = page; }
  int find(uint64_t key) const {
    auto it = map_.find(key);
    return it == map_.end() ? -1 : it->second;
  }
  void erase(uint64_t key) { map_.erase(key); }
  size_t size() const { return map_.size(); }

 private:
  std::unordered_map<uint64_t, int> map_;
};

struct CopyOp {
  int src, dst;  // device page copies the caller must perform before the next step
};

class KvManager {
 public:
  KvManager(int num_pages, int page_size, int max_pages_per_seq, bool prefix_cache);

  // Open a sequence for `tokens`.  Returns how many leading tokens are already
  // cached (a multiple of page_size, < len(tokens)), whose KV need no prefill.
  int open(int64_t seq, const std::vector<int32_t>& tokens);
  // Reserve KV slots for `n` more tokens; returns their slot ids (page*page_size+off).
  std::vector<int32_t> append(int64_t seq, const std::vector<int32_t>& tokens);
  // Keep only the first `len` tokens (speculative rollback).  A sealed page
  // that becomes partial again is un-indexed, or copied if another sequence
  // shares it (returned CopyOp).
  std::vector<CopyOp> truncate(int64_t seq, int len);
  // New sequence `child` sharing `parent`'s full pages; the boundary page is
  // copied (returned as a CopyOp) so both can extend it.
  std::vector<CopyOp> fork(int64_t parent, int64_t child);
  void free(int64_t seq);
  // Seal full pages of `seq` into the prefix index (after their KV is written).
  void commit_prefix(int64_t seq);

  int length(int64_t seq) const { return (int)seqs_.at(seq).tokens.size(); }
  const std::vector<int32_t>& pages(int64_t seq) const { return seqs_.at(seq).pages; }
  bool can_append(int64_t seq, int n) const;
  int pages_needed(int64_t seq, int n) const;
  int num_free_pages() const { return pool_.num_free(); }
  int num_pages() const { return pool_.num_pages(); }
  int page_size() const { return page_size_; }
  size_t num_seqs() const { return seqs_.size(); }
  size_t cached_blocks() const { return tree_.size(); }
  // Fill a [n_seqs, max_pages] int32 block table (row i = seqs[i]), unused = 0.
  void block_table(const std::vector<int64_t>& seqs, int32_t* out, int max_pages) const;
  // Chained block keys of the full pages of `tokens` (what the prefix index stores).
  std::vector<uint64_t> block_keys(const std::vector<int32_t>& tokens) const;
  // How many leading `keys` the index holds.
  int cached_prefix_blocks(const std::vector<uint64_t>& keys) const;
  // Index a block restored from a lower tier (host / NVMe): a page for `key`, held
  // by no sequence (evictable).  Returns the page, whose KV the caller must fill
  // before the next step, or -1 if `key` is indexed already or nothing is free.
  int import_block(uint64_t key);
  // Sealed pages of `seq` as (key, page), prefix order.
  std::vector<std::pair<uint64_t, int>> sealed_blocks(int64_t seq) const;
  bool prefix_cache() const { return prefix_cache_; }
  int64_t hits() const { return hits_; }
  int64_t lookups() const { return lookups_; }

 private:
  struct Seq {
    std::vector<int32_t> tokens;
    std::vector<int32_t> pages;
    std::vector<uint64_t> keys;  // keys of sealed (full, hashed) pages, prefix order
  };
  int alloc_page();
  PagePool pool_;
  PrefixTree tree_;
  int page_size_;
  int max_pages_;
  bool prefix_cache_;
  std::unordered_map<int64_t, Seq> seqs_;
  int64_t hits_ = 0, lookups_ = 0;
};

}  // namespace rkt_rt
