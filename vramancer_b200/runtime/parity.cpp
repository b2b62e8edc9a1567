// XOR parity over equal-length byte shards (N data shards -> 1 parity shard; any one
// missing shard is the XOR of the others and the parity).
//
// Reference parity: csrc/swarm_core.cpp (xor parity generate / repair, 64-bit
// chunks) and rust_core/src/lib.rs:1057-1108.
#include <algorithm>
#include <cstring>
#include <thread>

#include "runtime.h"

namespace vrt {

static void xor_range(const std::vector<const uint8_t*>& shards, size_t b, size_t e, uint8_t* out) {
  size_t i = b;
  // 64-bit words (memcpy keeps it alignment-agnostic; compiles to plain loads)
  for (; i + 8 <= e; i += 8) {
    uint64_t acc = 0;
    for (const uint8_t* s : shards) {
      uint64_t w;
      std::memcpy(&w, s + i, 8);
      acc ^= w;
    }
    std::memcpy(out + i, &acc, 8);
  }
  for (; i < e; ++i) {
    uint8_t acc = 0;
    for (const uint8_t* s : shards) acc ^= s[i];
    out[i] = acc;
  }
}

void xor_parity(const std::vector<const uint8_t*>& shards, size_t len, uint8_t* out, int threads) {
  if (shards.empty()) {
    std::memset(out, 0, len);
    return;
  }
  threads = std::max(1, std::min(threads, (int)(len / (1 << 20)) + 1));
  if (threads == 1) {
    xor_range(shards, 0, len, out);
    return;
  }
  const size_t per = ((len + threads - 1) / threads + 63) & ~(size_t)63;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    const size_t b = std::min(len, per * t), e = std::min(len, b + per);
    if (b < e) pool.emplace_back(xor_range, std::cref(shards), b, e, out);
  }
  for (auto& th : pool) th.join();
}

}  // namespace vrt
