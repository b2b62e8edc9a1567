// Basic tokenizer for when no tokenizer files are available: whitespace / punctuation
// split, FNV-1a hash of each piece modulo the vocabulary, threads across texts.
//
// Reference parity: rust_core/src/lib.rs:1501-1558 (basic whitespace tokenizer,
// batch_tokenize_fast).
#include <cctype>
#include <thread>

#include "runtime.h"

namespace vrt {

static std::vector<int32_t> tok_one(const std::string& s, int32_t vocab) {
  std::vector<int32_t> out;
  size_t i = 0;
  auto emit = [&](size_t b, size_t e) {
    uint32_t h = 2166136261u;
    for (size_t k = b; k < e; ++k) {
      h ^= (uint8_t)s[k];
      h *= 16777619u;
    }
    out.push_back((int32_t)(h % (uint32_t)vocab));
  };
  while (i < s.size()) {
    const unsigned char c = (unsigned char)s[i];
    if (std::isspace(c)) {
      ++i;
      continue;
    }
    if (std::ispunct(c)) {
      emit(i, i + 1);
      ++i;
      continue;
    }
    size_t j = i;
    while (j < s.size() && !std::isspace((unsigned char)s[j]) && !std::ispunct((unsigned char)s[j])) ++j;
    emit(i, j);
    i = j;
  }
  return out;
}

std::vector<std::vector<int32_t>> basic_tokenize(const std::vector<std::string>& texts, int32_t vocab, int threads) {
  std::vector<std::vector<int32_t>> out(texts.size());
  if (vocab <= 0) return out;
  threads = std::max(1, std::min<int>(threads, (int)texts.size()));
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t)
    pool.emplace_back([&, t] {
      for (size_t i = t; i < texts.size(); i += threads) out[i] = tok_one(texts[i], vocab);
    });
  for (auto& th : pool) th.join();
  return out;
}

}  // namespace vrt
