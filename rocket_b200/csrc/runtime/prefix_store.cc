#include "prefix_store.h"

#include <dirent.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <sys/statvfs.h>
#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstddef>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <stdexcept>

namespace rkt_rt {

// ------------------------------------------------------------------ digest
namespace {

inline uint64_t mix64(uint64_t x) {  // splitmix64 finaliser
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

inline uint64_t rotl(uint64_t x, int r) { return (x << r) | (x >> (64 - r)); }

struct Lanes {
  uint64_t h[4] = {0x6a09e667f3bcc908ull, 0xbb67ae8584caa73bull, 0x3c6ef372fe94f82bull, 0xa54ff53a5f1d36f1ull};
  static constexpr uint64_t P[4] = {0x9e3779b97f4a7c15ull, 0xc2b2ae3d27d4eb4full, 0x165667b19e3779f9ull,
                                    0xd6e8feb86659fd93ull};
  uint64_t n = 0;
  void word(uint64_t w) {
    for (int i = 0; i < 4; ++i) h[i] = rotl((h[i] ^ (w + (uint64_t)i)) * P[i], 23 + 7 * i);
    ++n;
  }
};

}  // namespace

Digest256 digest256(const std::vector<std::pair<const uint8_t*, size_t>>& parts) {
  Lanes L;
  for (auto& pt : parts) {
    L.word((uint64_t)pt.second);  // part boundaries are part of the digest
    const uint8_t* p = pt.first;
    size_t n = pt.second, i = 0;
    for (; i + 8 <= n; i += 8) {
      uint64_t w;
      memcpy(&w, p + i, 8);
      L.word(w);
    }
    if (i < n) {
      uint64_t w = 0;
      memcpy(&w, p + i, n - i);
      L.word(w ^ ((uint64_t)(n - i) << 56));
    }
  }
  Digest256 d;
  for (int i = 0; i < 4; ++i) d.w[i] = mix64(L.h[i] ^ mix64(L.n + (uint64_t)i));
  return d;
}

// ------------------------------------------------------------------ manifest record
namespace {

constexpr uint32_t kMagic = 0x524b544d;  // "RKTM"
constexpr uint16_t kVersion = 1;
constexpr uint16_t kTombstone = 0xffff;

#pragma pack(push, 1)
struct Rec {
  uint32_t magic;
  uint16_t version;
  uint16_t n_comp;  // kTombstone: the (key, fp) entry is deleted
  uint64_t key, fp;
  uint32_t segment, pad;
  uint64_t offset, length;
  uint64_t sizes[PrefixStore::kMaxComponents];
  uint64_t digest[4];
  uint64_t check;  // mix of every field above
};
#pragma pack(pop)
static_assert(sizeof(Rec) == 8 + 16 + 8 + 16 + 8 * PrefixStore::kMaxComponents + 32 + 8, "record layout");

uint64_t rec_check(const Rec& r) {
  const uint8_t* p = reinterpret_cast<const uint8_t*>(&r);
  uint64_t h = 0x243f6a8885a308d3ull;
  for (size_t i = 0; i + 8 <= offsetof(Rec, check); i += 8) {
    uint64_t w;
    memcpy(&w, p + i, 8);
    h = mix64(h ^ w);
  }
  return h;
}

void write_all(int fd, const void* buf, size_t n, uint64_t off) {
  const uint8_t* p = static_cast<const uint8_t*>(buf);
  while (n) {
    const ssize_t w = pwrite(fd, p, n, (off_t)off);
    if (w < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(std::string("prefix store: write failed: ") + strerror(errno));
    }
    p += w;
    n -= (size_t)w;
    off += (uint64_t)w;
  }
}

bool read_all(int fd, void* buf, size_t n, uint64_t off) {
  uint8_t* p = static_cast<uint8_t*>(buf);
  while (n) {
    const ssize_t r = pread(fd, p, n, (off_t)off);
    if (r < 0 && errno == EINTR) continue;
    if (r <= 0) return false;
    p += r;
    n -= (size_t)r;
    off += (uint64_t)r;
  }
  return true;
}

uint64_t round_up(uint64_t x, uint64_t a) { return (x + a - 1) / a * a; }

}  // namespace

// ------------------------------------------------------------------ store
PrefixStore::PrefixStore(const std::string& dir, uint64_t max_bytes, uint64_t segment_bytes, bool direct_io)
    : dir_(dir), max_bytes_(max_bytes), segment_bytes_(std::max<uint64_t>(segment_bytes, kAlign)), direct_(direct_io) {
  mkdir(dir_.c_str(), 0755);
  mkdir((dir_ + "/segments").c_str(), 0755);
  open_manifest();
  // the next appends go to a fresh segment after the highest one seen
  uint32_t hi = 0;
  for (auto& s : seg_bytes_) hi = std::max(hi, s.first + 1);
  DIR* d = opendir((dir_ + "/segments").c_str());
  if (d) {
    while (dirent* e = readdir(d)) {
      unsigned id;
      if (sscanf(e->d_name, "seg-%06u.bin", &id) == 1) hi = std::max(hi, (uint32_t)id + 1);
    }
    closedir(d);
  }
  cur_seg_ = hi;
}

PrefixStore::~PrefixStore() {
  if (cur_fd_ >= 0) close(cur_fd_);
  if (manifest_fd_ >= 0) close(manifest_fd_);
}

std::string PrefixStore::seg_path(uint32_t id) const {
  char b[64];
  snprintf(b, sizeof b, "/segments/seg-%06u.bin", id);
  return dir_ + b;
}

int PrefixStore::open_segment(uint32_t id, bool create) {
  int flags = create ? (O_RDWR | O_CREAT) : O_RDONLY;
  flags |= O_CLOEXEC;
#ifdef O_DIRECT
  if (direct_) flags |= O_DIRECT;
#endif
  return open(seg_path(id).c_str(), flags, 0644);
}

void PrefixStore::open_manifest() {
  const std::string path = dir_ + "/manifest.bin";
  manifest_fd_ = open(path.c_str(), O_RDWR | O_CREAT | O_CLOEXEC, 0644);
  if (manifest_fd_ < 0) throw std::runtime_error("prefix store: cannot open " + path);
  struct stat stt {};
  fstat(manifest_fd_, &stt);
  const uint64_t size = (uint64_t)stt.st_size;
  uint64_t good = 0;
  Rec r;
  while (good + sizeof(Rec) <= size) {
    if (!read_all(manifest_fd_, &r, sizeof r, good)) break;
    if (r.magic != kMagic || r.version != kVersion || r.check != rec_check(r)) break;
    const Key k{r.key, r.fp};
    if (r.n_comp == kTombstone) {
      index_.erase(k);
    } else if (r.n_comp <= kMaxComponents) {
      Entry e{};
      e.segment = r.segment;
      e.offset = r.offset;
      e.length = r.length;
      e.n_comp = r.n_comp;
      memcpy(e.sizes, r.sizes, sizeof e.sizes);
      memcpy(e.digest.w, r.digest, sizeof r.digest);
      index_[k] = e;
    } else {
      break;
    }
    good += sizeof(Rec);
  }
  manifest_records_ = good / sizeof(Rec);
  if (good != size) {  // torn tail: drop the partial / corrupt suffix
    if (ftruncate(manifest_fd_, (off_t)good) != 0)
      throw std::runtime_error("prefix store: cannot truncate a torn manifest tail");
    ++st_.torn_tail_recoveries;
  }
  // drop entries whose segment bytes are missing (a segment deleted or cut short)
  std::map<uint32_t, uint64_t> seg_size;
  for (auto it = index_.begin(); it != index_.end();) {
    const Entry& e = it->second;
    auto sit = seg_size.find(e.segment);
    if (sit == seg_size.end()) {
      struct stat ss {};
      const uint64_t sz = stat(seg_path(e.segment).c_str(), &ss) == 0 ? (uint64_t)ss.st_size : 0;
      sit = seg_size.emplace(e.segment, sz).first;
    }
    if (e.offset + e.length > sit->second) {
      it = index_.erase(it);
      continue;
    }
    seg_bytes_[e.segment] += round_up(e.length, kAlign);
    st_.live_bytes += (int64_t)e.length;
    ++it;
  }
  st_.live_records = (int64_t)index_.size();
}

void PrefixStore::append_manifest(uint64_t key, uint64_t fp, const Entry* e) {
  Rec r{};
  r.magic = kMagic;
  r.version = kVersion;
  r.key = key;
  r.fp = fp;
  if (e) {
    r.n_comp = e->n_comp;
    r.segment = e->segment;
    r.offset = e->offset;
    r.length = e->length;
    memcpy(r.sizes, e->sizes, sizeof r.sizes);
    memcpy(r.digest, e->digest.w, sizeof r.digest);
  } else {
    r.n_comp = kTombstone;
  }
  r.check = rec_check(r);
  write_all(manifest_fd_, &r, sizeof r, manifest_records_ * sizeof(Rec));
  ++manifest_records_;
  fdatasync(manifest_fd_);
}

bool PrefixStore::put(uint64_t key, uint64_t fp, const std::vector<std::pair<const uint8_t*, size_t>>& parts) {
  std::lock_guard<std::mutex> g(mu_);
  if ((int)parts.size() > kMaxComponents || parts.empty())
    throw std::invalid_argument("prefix store: 1..6 components per record");
  const Key k{key, fp};
  if (index_.count(k)) return false;
  uint64_t len = 0;
  for (auto& p : parts) len += p.second;
  const uint64_t padded = round_up(std::max<uint64_t>(len, 1), kAlign);
  if (min_free_) {
    struct statvfs vs {};
    if (statvfs(dir_.c_str(), &vs) == 0) {
      const uint64_t avail = (uint64_t)vs.f_bavail * vs.f_frsize;
      if (avail < padded + min_free_) {
        ++st_.refused_low_space;
        return false;
      }
    }
  }
  if (cur_fd_ < 0 || cur_size_ + padded > segment_bytes_) {
    if (cur_fd_ >= 0) {
      close(cur_fd_);
      ++cur_seg_;
    }
    cur_fd_ = open_segment(cur_seg_, true);
    if (cur_fd_ < 0) throw std::runtime_error("prefix store: cannot create " + seg_path(cur_seg_));
    struct stat ss {};
    fstat(cur_fd_, &ss);
    cur_size_ = round_up((uint64_t)ss.st_size, kAlign);
  }
  // staging buffer aligned for O_DIRECT; the record is padded to the 64 KiB boundary
  void* buf = nullptr;
  if (posix_memalign(&buf, 4096, padded) != 0) throw std::bad_alloc();
  uint8_t* b = static_cast<uint8_t*>(buf);
  uint64_t o = 0;
  for (auto& p : parts) {
    memcpy(b + o, p.first, p.second);
    o += p.second;
  }
  memset(b + o, 0, padded - o);
  Entry e{};
  e.segment = cur_seg_;
  e.offset = cur_size_;
  e.length = len;
  e.n_comp = (uint16_t)parts.size();
  for (size_t i = 0; i < parts.size(); ++i) e.sizes[i] = parts[i].second;
  e.digest = digest256(parts);
  try {
    write_all(cur_fd_, b, padded, e.offset);
  } catch (...) {
    free(buf);
    throw;
  }
  free(buf);
  fdatasync(cur_fd_);  // data before its manifest entry
  cur_size_ += padded;
  append_manifest(key, fp, &e);
  index_[k] = e;
  seg_bytes_[e.segment] += padded;
  ++st_.puts;
  st_.bytes_written += (int64_t)len;
  st_.live_bytes += (int64_t)len;
  st_.live_records = (int64_t)index_.size();
  enforce_capacity();
  return true;
}

bool PrefixStore::contains(uint64_t key, uint64_t fp) const {
  std::lock_guard<std::mutex> g(mu_);
  return index_.count({key, fp}) > 0;
}

std::vector<uint64_t> PrefixStore::sizes(uint64_t key, uint64_t fp) const {
  std::lock_guard<std::mutex> g(mu_);
  auto it = index_.find({key, fp});
  if (it == index_.end()) return {};
  return std::vector<uint64_t>(it->second.sizes, it->second.sizes + it->second.n_comp);
}

bool PrefixStore::get_into(uint64_t key, uint64_t fp, const std::vector<std::pair<uint8_t*, size_t>>& out) {
  std::lock_guard<std::mutex> g(mu_);
  ++st_.gets;
  auto it = index_.find({key, fp});
  if (it == index_.end()) {
    ++st_.misses;
    return false;
  }
  const Entry e = it->second;
  if (out.size() != e.n_comp) throw std::invalid_argument("prefix store: component count mismatch");
  for (size_t i = 0; i < out.size(); ++i)
    if (out[i].second != e.sizes[i]) throw std::invalid_argument("prefix store: component size mismatch");
  const uint64_t padded = round_up(std::max<uint64_t>(e.length, 1), kAlign);
  void* buf = nullptr;
  if (posix_memalign(&buf, 4096, padded) != 0) throw std::bad_alloc();
  int fd = e.segment == cur_seg_ && cur_fd_ >= 0 ? cur_fd_ : open_segment(e.segment, false);
  const bool own = fd != cur_fd_;
  bool ok = fd >= 0 && read_all(fd, buf, padded, e.offset);
  if (own && fd >= 0) close(fd);
  if (ok) {
    const uint8_t* b = static_cast<const uint8_t*>(buf);
    std::vector<std::pair<const uint8_t*, size_t>> parts;
    uint64_t o = 0;
    for (int i = 0; i < e.n_comp; ++i) {
      parts.emplace_back(b + o, e.sizes[i]);
      o += e.sizes[i];
    }
    ok = digest256(parts) == e.digest;
    if (ok) {
      for (int i = 0; i < e.n_comp; ++i) memcpy(out[i].first, parts[i].first, parts[i].second);
      st_.bytes_read += (int64_t)e.length;
    } else {
      ++st_.checksum_failures;
    }
  }
  free(buf);
  if (!ok) {  // unreadable or corrupt: forget it, the caller recomputes
    index_.erase({key, fp});
    append_manifest(key, fp, nullptr);
    st_.live_bytes -= (int64_t)e.length;
    st_.live_records = (int64_t)index_.size();
    ++st_.misses;
    return false;
  }
  ++st_.hits;
  return true;
}

bool PrefixStore::erase(uint64_t key, uint64_t fp) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = index_.find({key, fp});
  if (it == index_.end()) return false;
  st_.live_bytes -= (int64_t)it->second.length;
  index_.erase(it);
  append_manifest(key, fp, nullptr);
  st_.live_records = (int64_t)index_.size();
  return true;
}

void PrefixStore::drop_segment(uint32_t id) {
  for (auto it = index_.begin(); it != index_.end();) {
    if (it->second.segment == id) {
      st_.live_bytes -= (int64_t)it->second.length;
      ++st_.evicted_records;
      it = index_.erase(it);
    } else {
      ++it;
    }
  }
  seg_bytes_.erase(id);
  unlink(seg_path(id).c_str());
  st_.live_records = (int64_t)index_.size();
}

void PrefixStore::enforce_capacity() {
  uint64_t total = 0;
  for (auto& s : seg_bytes_) total += s.second;
  while (total > max_bytes_ && seg_bytes_.size() > 1) {
    const uint32_t oldest = seg_bytes_.begin()->first;
    if (oldest == cur_seg_) break;
    total -= seg_bytes_.begin()->second;
    drop_segment(oldest);
  }
  if (manifest_records_ > 64 && manifest_records_ > 4 * index_.size()) compact_manifest();
}

void PrefixStore::compact_manifest() {
  const std::string path = dir_ + "/manifest.bin", tmp = dir_ + "/manifest.tmp";
  const int fd = open(tmp.c_str(), O_RDWR | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
  if (fd < 0) return;
  const int old = manifest_fd_;
  const uint64_t old_n = manifest_records_;
  manifest_fd_ = fd;
  manifest_records_ = 0;
  try {
    for (auto& kv : index_) append_manifest(kv.first.first, kv.first.second, &kv.second);
  } catch (...) {
    close(fd);
    manifest_fd_ = old;
    manifest_records_ = old_n;
    return;
  }
  fsync(fd);
  if (rename(tmp.c_str(), path.c_str()) != 0) {
    close(fd);
    manifest_fd_ = old;
    manifest_records_ = old_n;
    return;
  }
  close(old);
}

PrefixStoreStats PrefixStore::stats() const {
  std::lock_guard<std::mutex> g(mu_);
  return st_;
}

void PrefixStore::flush() {
  std::lock_guard<std::mutex> g(mu_);
  if (cur_fd_ >= 0) fdatasync(cur_fd_);
  if (manifest_fd_ >= 0) fdatasync(manifest_fd_);
}

}  // namespace rkt_rt
