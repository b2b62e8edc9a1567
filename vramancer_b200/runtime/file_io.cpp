// File spill / restore of raw memory (KV pages, tensors) with pwrite / pread, outside
// the Python interpreter lock, plus a worker pool for overlapped I/O.
//
// Reference parity: csrc/file_offload.cpp (cxl_direct_memory_dump / load) and
// rust_core/src/lib.rs:1012-1052 (file dump/load); the reference's NVMe tier tries
// io_uring / O_DIRECT in core/hierarchical_memory.py.
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>

#include "runtime.h"

namespace vrt {
namespace {

constexpr size_t kAlign = 4096;
constexpr size_t kIoChunk = 64ull << 20;

bool aligned(const void* p, size_t n, size_t off) {
  return (reinterpret_cast<uintptr_t>(p) % kAlign) == 0 && n % kAlign == 0 && off % kAlign == 0;
}

std::string err(const char* what, const std::string& path) {
  return std::string(what) + " " + path + ": " + std::strerror(errno);
}

}  // namespace

size_t file_write(const std::string& path, const void* p, size_t n, size_t offset, bool direct, bool sync) {
  int flags = O_WRONLY | O_CREAT;
#ifdef O_DIRECT
  if (direct && aligned(p, n, offset)) flags |= O_DIRECT;
#endif
  const int fd = ::open(path.c_str(), flags, 0600);
  if (fd < 0) throw std::runtime_error(err("open", path));
  size_t done = 0;
  const auto* src = static_cast<const uint8_t*>(p);
  while (done < n) {
    const size_t want = std::min(kIoChunk, n - done);
    const ssize_t w = ::pwrite(fd, src + done, want, (off_t)(offset + done));
    if (w < 0) {
      if (errno == EINTR) continue;
      const std::string e = err("pwrite", path);
      ::close(fd);
      throw std::runtime_error(e);
    }
    done += (size_t)w;
  }
  if (sync) ::fsync(fd);
  ::close(fd);
  return done;
}

size_t file_read(const std::string& path, void* p, size_t n, size_t offset, bool direct) {
  int flags = O_RDONLY;
#ifdef O_DIRECT
  if (direct && aligned(p, n, offset)) flags |= O_DIRECT;
#endif
  const int fd = ::open(path.c_str(), flags);
  if (fd < 0) throw std::runtime_error(err("open", path));
  size_t done = 0;
  auto* dst = static_cast<uint8_t*>(p);
  while (done < n) {
    const size_t want = std::min(kIoChunk, n - done);
    const ssize_t r = ::pread(fd, dst + done, want, (off_t)(offset + done));
    if (r < 0) {
      if (errno == EINTR) continue;
      const std::string e = err("pread", path);
      ::close(fd);
      throw std::runtime_error(e);
    }
    if (r == 0) {
      ::close(fd);
      throw std::runtime_error("short read " + path + ": " + std::to_string(done) + " of " + std::to_string(n));
    }
    done += (size_t)r;
  }
  ::close(fd);
  return done;
}

AsyncIO::AsyncIO(int workers) {
  for (int i = 0; i < std::max(1, workers); ++i) workers_.emplace_back([this] { loop(); });
}

AsyncIO::~AsyncIO() {
  {
    std::lock_guard<std::mutex> g(mu_);
    stop_ = true;
  }
  cv_.notify_all();
  for (auto& t : workers_) t.join();
}

int64_t AsyncIO::submit(std::function<size_t()> fn) {
  std::lock_guard<std::mutex> g(mu_);
  const int64_t id = next_++;
  results_[id] = Result{};
  q_.emplace_back(id, std::move(fn));
  cv_.notify_one();
  return id;
}

int64_t AsyncIO::submit_write(const std::string& path, const void* p, size_t n, size_t offset, bool direct) {
  return submit([=] { return file_write(path, p, n, offset, direct, false); });
}

int64_t AsyncIO::submit_read(const std::string& path, void* p, size_t n, size_t offset, bool direct) {
  return submit([=] { return file_read(path, p, n, offset, direct); });
}

void AsyncIO::loop() {
  for (;;) {
    std::pair<int64_t, std::function<size_t()>> job;
    {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [this] { return stop_ || !q_.empty(); });
      if (stop_ && q_.empty()) return;
      job = std::move(q_.front());
      q_.pop_front();
    }
    Result r;
    try {
      r.bytes = job.second();
    } catch (const std::exception& e) {
      r.error = e.what();
    }
    r.finished = true;
    {
      std::lock_guard<std::mutex> g(mu_);
      results_[job.first] = r;
    }
    done_cv_.notify_all();
  }
}

size_t AsyncIO::wait(int64_t ticket) {
  std::unique_lock<std::mutex> lk(mu_);
  auto it = results_.find(ticket);
  if (it == results_.end()) throw std::invalid_argument("unknown I/O ticket");
  done_cv_.wait(lk, [&] { return results_[ticket].finished; });
  Result r = results_[ticket];
  results_.erase(ticket);
  if (!r.error.empty()) throw std::runtime_error(r.error);
  return r.bytes;
}

bool AsyncIO::done(int64_t ticket) {
  std::lock_guard<std::mutex> g(mu_);
  auto it = results_.find(ticket);
  return it == results_.end() || it->second.finished;
}

size_t AsyncIO::pending() {
  std::lock_guard<std::mutex> g(mu_);
  size_t n = 0;
  for (auto& kv : results_) n += kv.second.finished ? 0 : 1;
  return n;
}

}  // namespace vrt
