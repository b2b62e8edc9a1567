// Host-side native runtime of vramancer_b200 (module vramancer_b200._runtime): no CUDA,
// no torch; buffers cross the boundary as raw pointers + sizes or Python buffers.
#pragma once
#include <atomic>
#include <condition_variable>
#include <cstddef>
#include <cstdint>
#include <deque>
#include <functional>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <utility>
#include <vector>

namespace vrt {

// ---------------------------------------------------------------- crypto.cpp
class Sha256 {
 public:
  Sha256();
  void reset();
  void update(const uint8_t* p, size_t n);
  void finish(uint8_t out[32]);

 private:
  void block(const uint8_t* p);
  uint32_t h_[8];
  uint64_t len_;
  uint8_t buf_[64];
  size_t fill_;
};

class HmacSha256 {
 public:
  HmacSha256(const uint8_t* key, size_t klen);
  void update(const uint8_t* p, size_t n);
  void finish(uint8_t out[32]);

 private:
  uint8_t ipad_[64], opad_[64];
  Sha256 inner_;
};

void hmac_sha256(const uint8_t* key, size_t klen, const uint8_t* msg, size_t n, uint8_t out[32]);
bool ct_equal(const uint8_t* a, const uint8_t* b, size_t n);
void hmac_batch(const uint8_t* key, size_t klen, const std::vector<std::pair<const uint8_t*, size_t>>& msgs,
                uint8_t* out, int threads);

// ---------------------------------------------------------------- parity.cpp
// out = XOR of the n shards (each `len` bytes); threads split the byte range.
void xor_parity(const std::vector<const uint8_t*>& shards, size_t len, uint8_t* out, int threads);

// ---------------------------------------------------------------- file_io.cpp
// Whole-buffer file dump / load with pwrite / pread (optionally O_DIRECT when the
// buffer, length and offset are 4 KiB aligned).  Return bytes moved; throw on error.
size_t file_write(const std::string& path, const void* p, size_t n, size_t offset, bool direct, bool sync);
size_t file_read(const std::string& path, void* p, size_t n, size_t offset, bool direct);

// Background I/O: a fixed pool of worker threads executing queued reads / writes.
class AsyncIO {
 public:
  explicit AsyncIO(int workers);
  ~AsyncIO();
  int64_t submit_write(const std::string& path, const void* p, size_t n, size_t offset, bool direct);
  int64_t submit_read(const std::string& path, void* p, size_t n, size_t offset, bool direct);
  // waits for a ticket; returns bytes moved or throws the worker's error
  size_t wait(int64_t ticket);
  bool done(int64_t ticket);
  size_t pending();

 private:
  struct Result {
    bool finished = false;
    size_t bytes = 0;
    std::string error;
  };
  int64_t submit(std::function<size_t()> fn);
  void loop();
  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::deque<std::pair<int64_t, std::function<size_t()>>> q_;
  std::unordered_map<int64_t, Result> results_;
  std::vector<std::thread> workers_;
  int64_t next_ = 1;
  bool stop_ = false;
};

// ---------------------------------------------------------------- transport.cpp
// Framed tensor transport over TCP ("VTP" frames):
//   magic "VRT1" | u32 header_len | u64 payload_len | u32 chunk | u32 flags |
//   header bytes | payload in chunks [| 32-byte HMAC(key, seq || chunk) after each
//   chunk when flags & 1]
// Payloads are bounded by kMaxPayload; a bad tag or a short read throws.
constexpr uint64_t kMaxPayload = 16ull << 30;
class Connection {
 public:
  explicit Connection(int fd) : fd_(fd) {}
  ~Connection();
  void send_frame(const std::string& header, const uint8_t* payload, uint64_t n, const std::string& key,
                  uint32_t chunk);
  // receives a frame; the payload is written into a buffer allocated by `alloc`
  std::string recv_frame(const std::string& key, const std::function<uint8_t*(uint64_t)>& alloc, uint64_t* n);
  void close();
  int fd() const { return fd_; }

 private:
  int fd_;
};
Connection* tcp_connect(const std::string& host, int port, double timeout_s);
class Listener {
 public:
  Listener(const std::string& host, int port);
  ~Listener();
  Connection* accept(double timeout_s);
  int port() const { return port_; }
  void close();

 private:
  int fd_ = -1;
  int port_ = 0;
};

// ---------------------------------------------------------------- page_alloc.cpp
// KV page allocator: free list + reference counts (shared prefix pages), O(1) alloc /
// free per page, all-or-nothing multi-page allocation.
class PageAllocator {
 public:
  explicit PageAllocator(int64_t num_pages);
  // n pages or an empty vector when fewer than n are free
  std::vector<int32_t> alloc(int64_t n);
  void incref(int32_t page);
  // returns true when the page went back to the free list
  bool decref(int32_t page);
  void free_all(const std::vector<int32_t>& pages);
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t num_pages() const { return (int64_t)refs_.size(); }
  int32_t refcount(int32_t page) const;

 private:
  std::vector<int32_t> free_;
  std::vector<int32_t> refs_;
};

// ---------------------------------------------------------------- tokenizer.cpp
// Basic GIL-free tokenizer: splits on whitespace and punctuation, maps each piece to
// an id by FNV-1a hash modulo vocab (a stand-in when no tokenizer files exist).
std::vector<std::vector<int32_t>> basic_tokenize(const std::vector<std::string>& texts, int32_t vocab,
                                                 int threads);

// ---------------------------------------------------------------- ngram.cpp
// Prompt-lookup draft index of one growing token sequence (see ngram.cpp).
class NgramIndex {
 public:
  NgramIndex(int max_n, int min_n);
  void extend(const int32_t* tokens, size_t count);
  std::vector<int32_t> draft(int num_draft) const;
  size_t size() const { return seq_.size(); }

 private:
  uint64_t key(size_t start, int n) const;
  bool same(size_t a, size_t b, int n) const;
  int max_n_, min_n_;
  std::vector<int32_t> seq_;
  std::vector<std::unordered_map<uint64_t, size_t>> maps_;   // [n]: n-gram -> latest earlier start
};

}  // namespace vrt
