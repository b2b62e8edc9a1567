// Incremental n-gram index for prompt-lookup speculative decoding.
//
// Draft rule (the engine's Python `find_draft`): for n from max_n down to min_n, take
// the latest earlier occurrence of the sequence's last n tokens and propose the tokens
// that followed it (up to num_draft).  The Python rule rescans the sequence every step
// (O(length x n) per request); here each n keeps a hash map from an n-gram to the start
// of its latest occurrence that is not the current tail, updated in O(max_n) per
// appended token, so a draft costs O(max_n) lookups.  Hash collisions are resolved by
// comparing the stored tokens.
//
// Reference parity: the reference's prompt lookup (core/backends.py:1920-1925) scans
// the prompt on the host each step.
#include <algorithm>
#include <stdexcept>

#include "runtime.h"

namespace vrt {

namespace {
uint64_t mix(uint64_t h, uint32_t t) {
  h ^= (uint64_t)t + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
  return h * 0xBF58476D1CE4E5B9ull;
}
}  // namespace

NgramIndex::NgramIndex(int max_n, int min_n) : max_n_(max_n), min_n_(min_n), maps_(max_n + 1) {
  if (min_n < 1 || max_n < min_n || max_n > 64) throw std::invalid_argument("NgramIndex: need 1 <= min_n <= max_n <= 64");
}

uint64_t NgramIndex::key(size_t start, int n) const {
  uint64_t h = (uint64_t)n;
  for (int j = 0; j < n; ++j) h = mix(h, (uint32_t)seq_[start + j]);
  return h;
}

bool NgramIndex::same(size_t a, size_t b, int n) const {
  for (int j = 0; j < n; ++j)
    if (seq_[a + j] != seq_[b + j]) return false;
  return true;
}

void NgramIndex::extend(const int32_t* tokens, size_t count) {
  seq_.reserve(seq_.size() + count);
  for (size_t c = 0; c < count; ++c) {
    seq_.push_back(tokens[c]);
    const size_t L = seq_.size();
    // the n-gram that was the tail before this token (start L - 1 - n) is now an
    // earlier occurrence: record it as the latest one
    for (int n = min_n_; n <= max_n_; ++n) {
      if (L < (size_t)n + 1) break;
      const size_t s = L - 1 - (size_t)n;
      maps_[n][key(s, n)] = s;
    }
  }
}

std::vector<int32_t> NgramIndex::draft(int num_draft) const {
  std::vector<int32_t> out;
  const size_t L = seq_.size();
  if (num_draft <= 0) return out;
  for (int n = std::min<int>(max_n_, (int)L - 1); n >= min_n_; --n) {
    const size_t tail = L - (size_t)n;
    auto it = maps_[n].find(key(tail, n));
    if (it == maps_[n].end() || !same(it->second, tail, n)) continue;
    const size_t from = it->second + (size_t)n;
    const size_t to = std::min(L, from + (size_t)num_draft);
    if (from < to) return std::vector<int32_t>(seq_.begin() + from, seq_.begin() + to);
  }
  return out;
}

}  // namespace vrt
