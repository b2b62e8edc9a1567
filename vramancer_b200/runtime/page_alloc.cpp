// KV page allocator with reference counts (prefix-shared pages).
//
// Reference parity: core/paged_attention.py PagedKVCacheManager._free_pages list and
// per-page refcounts (Python); this is the same bookkeeping off the interpreter.
#include <stdexcept>

#include "runtime.h"

namespace vrt {

PageAllocator::PageAllocator(int64_t num_pages) : refs_(num_pages, 0) {
  if (num_pages < 0 || num_pages > (1ll << 31) - 1) throw std::invalid_argument("page count out of range");
  free_.reserve(num_pages);
  // pop_back hands out low page ids first
  for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back((int32_t)p);
}

std::vector<int32_t> PageAllocator::alloc(int64_t n) {
  std::vector<int32_t> out;
  if (n <= 0 || n > (int64_t)free_.size()) return out;
  out.reserve(n);
  for (int64_t i = 0; i < n; ++i) {
    const int32_t p = free_.back();
    free_.pop_back();
    refs_[p] = 1;
    out.push_back(p);
  }
  return out;
}

void PageAllocator::incref(int32_t page) {
  if (page < 0 || page >= (int32_t)refs_.size() || refs_[page] <= 0) throw std::invalid_argument("incref: page not allocated");
  ++refs_[page];
}

bool PageAllocator::decref(int32_t page) {
  if (page < 0 || page >= (int32_t)refs_.size() || refs_[page] <= 0) throw std::invalid_argument("decref: page not allocated");
  if (--refs_[page] == 0) {
    free_.push_back(page);
    return true;
  }
  return false;
}

void PageAllocator::free_all(const std::vector<int32_t>& pages) {
  for (int32_t p : pages) decref(p);
}

int32_t PageAllocator::refcount(int32_t page) const {
  if (page < 0 || page >= (int32_t)refs_.size()) throw std::invalid_argument("refcount: bad page");
  return refs_[page];
}

}  // namespace vrt
