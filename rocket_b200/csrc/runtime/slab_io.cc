#include "slab_io.h"

#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstdio>
#include <cstring>
#include <stdexcept>

#include "prefix_store.h"

namespace rkt_rt {

std::string digest_hex(const uint8_t* p, uint64_t n) {
  const Digest256 d = digest256({{p, (size_t)n}});
  char b[65];
  for (int i = 0; i < 4; ++i) snprintf(b + 16 * i, 17, "%016llx", (unsigned long long)d.w[i]);
  return std::string(b, 64);
}

SlabReader::SlabReader(const std::string& path, int threads, bool direct) : path_(path) {
  fd_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
  if (fd_ < 0) throw std::runtime_error("cannot open " + path + ": " + strerror(errno));
  struct stat st;
  fstat(fd_, &st);
  size_ = (uint64_t)st.st_size;
#ifdef O_DIRECT
  if (direct) fd_direct_ = ::open(path.c_str(), O_RDONLY | O_CLOEXEC | O_DIRECT);  // may fail (tmpfs): pread then
#endif
  if (threads < 1) threads = 1;
  for (int i = 0; i < threads; ++i) threads_.emplace_back([this] { worker(); });
}

SlabReader::~SlabReader() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_req_.notify_all();
  for (auto& t : threads_) t.join();
  if (fd_direct_ >= 0) ::close(fd_direct_);
  if (fd_ >= 0) ::close(fd_);
}

int64_t SlabReader::submit(uintptr_t dst, uint64_t offset, uint64_t n, std::vector<SlotCheck> checks) {
  if (offset + n > size_) throw std::out_of_range("slab read past the end of " + path_);
  for (auto& c : checks)
    if (c.rel + c.n > n) throw std::out_of_range("slot check outside the request");
  std::lock_guard<std::mutex> g(mu_);
  const int64_t t = next_++;
  queue_.push_back(Req{t, reinterpret_cast<uint8_t*>(dst), offset, n, std::move(checks)});
  cv_req_.notify_one();
  return t;
}

int64_t SlabReader::wait(int64_t ticket) {
  std::unique_lock<std::mutex> lk(mu_);
  for (;;) {
    for (size_t i = 0; i < done_.size(); ++i) {
      if (done_[i].first == ticket) {
        Done d = done_[i].second;
        done_.erase(done_.begin() + (long)i);
        if (!d.error.empty()) throw std::runtime_error(d.error);
        return d.bad;
      }
    }
    if (ticket >= next_) throw std::invalid_argument("wait on a ticket that was never submitted");
    cv_done_.wait(lk);
  }
}

void SlabReader::worker() {
  for (;;) {
    Req r;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_req_.wait(lk, [this] { return stop_ || !queue_.empty(); });
      if (stop_ && queue_.empty()) return;
      r = std::move(queue_.front());
      queue_.pop_front();
    }
    Done d;
    const bool aligned = fd_direct_ >= 0 && ((uintptr_t)r.dst % 4096 == 0) && (r.off % 4096 == 0);
    uint64_t got = 0;
    bool used_direct = false;
    while (got < r.n) {
      ssize_t k;
      const uint64_t left = r.n - got;
      if (aligned && left >= 4096) {
        // O_DIRECT for the 4 KiB-aligned body; the ragged tail (if any) through the page cache
        k = ::pread(fd_direct_, r.dst + got, (size_t)(left & ~uint64_t(4095)), (off_t)(r.off + got));
        used_direct = true;
      } else {
        k = ::pread(fd_, r.dst + got, (size_t)left, (off_t)(r.off + got));
      }
      if (k < 0 && errno == EINTR) continue;
      if (k <= 0) {
        d.error = "read of " + path_ + " failed at " + std::to_string(r.off + got) + ": " +
                  (k < 0 ? strerror(errno) : "unexpected end of file");
        break;
      }
      got += (uint64_t)k;
    }
    if (d.error.empty()) {
      for (size_t i = 0; i < r.checks.size(); ++i) {
        const SlotCheck& c = r.checks[i];
        if (!c.digest.empty() && digest_hex(r.dst + c.rel, c.n) != c.digest) {
          d.bad = (int64_t)i;
          break;
        }
      }
    }
    {
      std::lock_guard<std::mutex> g(mu_);
      bytes_read_ += got;
      direct_reads_ += used_direct ? 1 : 0;
      done_.emplace_back(r.ticket, d);
    }
    cv_done_.notify_all();
  }
}

}  // namespace rkt_rt
