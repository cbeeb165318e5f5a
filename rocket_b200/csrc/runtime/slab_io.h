// Asynchronous slab reader: file ranges -> caller-owned (pinned) host buffers.
//
// A pool of reader threads serves requests "read [offset, offset + n) of the file
// into buffer b, then check the digest of each listed slot".  Reads use O_DIRECT
// (bypassing the page cache: a 100+ GB weight set is read once and would only evict
// everything else) when the buffer address, offset and length are all 4 KiB
// aligned, and plain pread otherwise.  The caller owns the buffers (pinned host
// memory allocated by the framework) and must not reuse a buffer before `wait` on
// it returned; `wait` releases the caller as soon as that request is complete, so
// the device copy of buffer b overlaps the reads of the other buffers (a ring).
//
// Counterpart of the reference's O_DIRECT resident / expert-slab preload
// (engines/glm5-moe-nvfp4-2b/src/weights.cu:161 copy_in_direct, :777-925
// preload_expert_slab) and its authenticated disk -> pinned -> H2D ring
// (qwen38 cuda_slab_loader.py:145); thread pool and request protocol are new.
#pragma once
#include <condition_variable>
#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace rkt_rt {

struct SlotCheck {
  uint64_t rel = 0, n = 0;  // slot bytes inside the request
  std::string digest;       // expected hex digest256 (empty: not checked)
};

class SlabReader {
 public:
  SlabReader(const std::string& path, int threads, bool direct);
  ~SlabReader();
  SlabReader(const SlabReader&) = delete;
  SlabReader& operator=(const SlabReader&) = delete;

  uint64_t file_size() const { return size_; }
  // Queue a read into host buffer `dst` (caller-owned, >= n bytes); returns a ticket.
  int64_t submit(uintptr_t dst, uint64_t offset, uint64_t n, std::vector<SlotCheck> checks);
  // Block until the ticket's read finished; returns -1 on success, else the index of
  // the first slot whose digest did not match.  Throws on I/O errors.
  int64_t wait(int64_t ticket);
  uint64_t bytes_read() const { return bytes_read_; }
  uint64_t direct_reads() const { return direct_reads_; }

 private:
  struct Req {
    int64_t ticket;
    uint8_t* dst;
    uint64_t off, n;
    std::vector<SlotCheck> checks;
  };
  struct Done {
    int64_t bad = -1;
    std::string error;
  };
  void worker();

  std::string path_;
  int fd_ = -1, fd_direct_ = -1;
  uint64_t size_ = 0;
  std::mutex mu_;
  std::condition_variable cv_req_, cv_done_;
  std::deque<Req> queue_;
  std::vector<std::pair<int64_t, Done>> done_;
  int64_t next_ = 0;
  bool stop_ = false;
  uint64_t bytes_read_ = 0, direct_reads_ = 0;
  std::vector<std::thread> threads_;
};

// hex digest256 of a host byte range
std::string digest_hex(const uint8_t* p, uint64_t n);

}  // namespace rkt_rt
