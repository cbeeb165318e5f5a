// Persistent prefix / session store on a local filesystem or NVMe (host side, C++).
//
//  * data lives in append-only segment files (segments/seg-NNNNNN.bin); every
//    record starts on a 64 KiB boundary, so the files also work with O_DIRECT;
//  * an append-only manifest of fixed-size binary entries maps (key, config
//    fingerprint) -> (segment, offset, component sizes, 256-bit checksum);
//    each entry carries its own check word, so a torn manifest tail (a crash
//    mid-append) is detected and truncated on open;
//  * data is synced before its manifest entry is written, so an entry never
//    points at bytes that were not written;
//  * get() verifies the checksum of what it read; a mismatch counts a failure,
//    drops the entry and reports a miss (the caller recomputes);
//  * capacity: when live bytes exceed the budget the oldest segment is deleted
//    with all its records; the manifest is compacted when mostly dead; a put that
//    would leave the filesystem with less than a free-space headroom is skipped.
//
// Behavioural counterpart of the reference's NVMe prefix store
// (engines/glm5-moe-nvfp4-2b/src/kv/nvme_prefix_store.h:69-78,
// nvme_prefix_store.cc:389-480: 64 KiB-aligned segments, append-only manifest,
// torn-tail recovery, multi-component records, 256-bit checksums).  The file
// formats and code here are this build's own.
#pragma once
#include <cstdint>
#include <map>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

namespace rkt_rt {

// 256-bit digest: four independent 64-bit multiply-xorshift lanes over 8-byte
// words (lane seeds differ), each finished with a splitmix64 avalanche.
struct Digest256 {
  uint64_t w[4];
  bool operator==(const Digest256& o) const {
    return w[0] == o.w[0] && w[1] == o.w[1] && w[2] == o.w[2] && w[3] == o.w[3];
  }
};
Digest256 digest256(const std::vector<std::pair<const uint8_t*, size_t>>& parts);

struct PrefixStoreStats {
  int64_t puts = 0, gets = 0, hits = 0, misses = 0, checksum_failures = 0, torn_tail_recoveries = 0;
  int64_t evicted_records = 0, bytes_written = 0, bytes_read = 0, live_records = 0, live_bytes = 0;
  int64_t refused_low_space = 0;  // puts skipped to keep the filesystem's free-space headroom
};

class PrefixStore {
 public:
  static constexpr int kMaxComponents = 6;
  static constexpr uint64_t kAlign = 64 * 1024;

  PrefixStore(const std::string& dir, uint64_t max_bytes, uint64_t segment_bytes, bool direct_io);
  ~PrefixStore();

  // Store `parts` under (key, fp).  False if the entry exists already.
  bool put(uint64_t key, uint64_t fp, const std::vector<std::pair<const uint8_t*, size_t>>& parts);
  bool contains(uint64_t key, uint64_t fp) const;
  // Component sizes of an entry (empty if absent).
  std::vector<uint64_t> sizes(uint64_t key, uint64_t fp) const;
  // Read an entry into caller buffers (sizes must match sizes()); false on a miss or
  // a checksum failure (the entry is then dropped).
  bool get_into(uint64_t key, uint64_t fp, const std::vector<std::pair<uint8_t*, size_t>>& out);
  bool erase(uint64_t key, uint64_t fp);
  PrefixStoreStats stats() const;
  void flush();
  // Free-space headroom: a put that would leave less than this many bytes free on the
  // store's filesystem is skipped (put returns false; the caller recomputes later).
  void set_min_free_bytes(uint64_t b) { min_free_ = b; }
  uint64_t min_free_bytes() const { return min_free_; }

 private:
  struct Entry {
    uint32_t segment;
    uint64_t offset, length;
    uint16_t n_comp;
    uint64_t sizes[kMaxComponents];
    Digest256 digest;
  };
  using Key = std::pair<uint64_t, uint64_t>;  // (key, fingerprint)

  void open_manifest();
  void append_manifest(uint64_t key, uint64_t fp, const Entry* e);  // e == nullptr: tombstone
  int open_segment(uint32_t id, bool create);
  std::string seg_path(uint32_t id) const;
  uint64_t min_free_ = 256ull << 20;
  void enforce_capacity();
  void compact_manifest();
  void drop_segment(uint32_t id);

  std::string dir_;
  uint64_t max_bytes_, segment_bytes_;
  bool direct_;
  int manifest_fd_ = -1;
  uint64_t manifest_records_ = 0;
  std::map<Key, Entry> index_;
  std::map<uint32_t, uint64_t> seg_bytes_;  // live + dead bytes written per segment
  uint32_t cur_seg_ = 0;
  int cur_fd_ = -1;
  uint64_t cur_size_ = 0;
  mutable std::mutex mu_;
  PrefixStoreStats st_;
};

}  // namespace rkt_rt
