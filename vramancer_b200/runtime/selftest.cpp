// Standalone self-test of the host runtime (no Python, no torch), built with
// AddressSanitizer + UndefinedBehaviorSanitizer and separately with ThreadSanitizer by
// tests/test_runtime_sanitizers.py:
//
//   g++ -std=c++17 -O1 -g -fsanitize=address,undefined -pthread selftest.cpp crypto.cpp \
//       parity.cpp file_io.cpp page_alloc.cpp tokenizer.cpp transport.cpp -o selftest
//   ./selftest <scratch dir>
//
// Every check that fails prints a line and the exit status counts the failures; the
// sanitizers abort on the first memory error or data race.  The multi-threaded paths
// (batched HMAC, parity, tokenizer, the async I/O pool driven from several submitting
// threads, a TCP sender thread) are the ones ThreadSanitizer is there for.
//
// Reference parity: the reference has no sanitizer builds (its race coverage is a
// 50-thread chaos test, tests/test_chaos_concurrency.py:27-62); this binary is the
// host-side race / memory check of this runtime.
#include <cstdio>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "runtime.h"

namespace {

int g_fail = 0;

void check(bool ok, const char* what) {
  if (!ok) {
    std::printf("FAIL: %s\n", what);
    ++g_fail;
  }
}

std::string hex(const uint8_t* p, size_t n) {
  static const char* d = "0123456789abcdef";
  std::string s;
  for (size_t i = 0; i < n; ++i) {
    s.push_back(d[p[i] >> 4]);
    s.push_back(d[p[i] & 15]);
  }
  return s;
}

void test_crypto() {
  // FIPS 180-2 "abc" and RFC 4231 test case 2 (published test vectors)
  vrt::Sha256 h;
  h.update(reinterpret_cast<const uint8_t*>("abc"), 3);
  uint8_t out[32];
  h.finish(out);
  check(hex(out, 32) == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad", "sha256(abc)");
  const char* key = "Jefe";
  const char* msg = "what do ya want for nothing?";
  vrt::hmac_sha256(reinterpret_cast<const uint8_t*>(key), 4, reinterpret_cast<const uint8_t*>(msg),
                   std::strlen(msg), out);
  check(hex(out, 32) == "5bdcc146bf60754e6a042426089575c75a003f089d2739839dec58b964ec3843", "hmac rfc4231 #2");
  uint8_t a[32], b[32];
  std::memcpy(a, out, 32);
  std::memcpy(b, out, 32);
  check(vrt::ct_equal(a, b, 32), "ct_equal same");
  b[31] ^= 1;
  check(!vrt::ct_equal(a, b, 32), "ct_equal differs");

  // batched HMAC on 4 threads == one at a time
  std::vector<std::vector<uint8_t>> bufs(37);
  std::vector<std::pair<const uint8_t*, size_t>> msgs;
  for (size_t i = 0; i < bufs.size(); ++i) {
    bufs[i].resize(1 + i * 97);
    for (size_t j = 0; j < bufs[i].size(); ++j) bufs[i][j] = (uint8_t)(i * 31 + j);
    msgs.emplace_back(bufs[i].data(), bufs[i].size());
  }
  std::vector<uint8_t> tags(32 * msgs.size());
  vrt::hmac_batch(reinterpret_cast<const uint8_t*>(key), 4, msgs, tags.data(), 4);
  for (size_t i = 0; i < msgs.size(); ++i) {
    vrt::hmac_sha256(reinterpret_cast<const uint8_t*>(key), 4, msgs[i].first, msgs[i].second, out);
    check(std::memcmp(out, tags.data() + 32 * i, 32) == 0, "hmac_batch row");
  }
}

void test_parity() {
  const size_t len = 100003;
  std::vector<std::vector<uint8_t>> shards(5, std::vector<uint8_t>(len));
  std::vector<const uint8_t*> ptrs;
  for (size_t s = 0; s < shards.size(); ++s) {
    for (size_t i = 0; i < len; ++i) shards[s][i] = (uint8_t)(s * 7 + i * 13);
    ptrs.push_back(shards[s].data());
  }
  std::vector<uint8_t> p1(len), p4(len);
  vrt::xor_parity(ptrs, len, p1.data(), 1);
  vrt::xor_parity(ptrs, len, p4.data(), 4);
  check(p1 == p4, "parity threads agree");
  // a lost shard is the XOR of the parity and the others
  std::vector<const uint8_t*> rest = {p1.data(), ptrs[0], ptrs[1], ptrs[3], ptrs[4]};
  std::vector<uint8_t> rec(len);
  vrt::xor_parity(rest, len, rec.data(), 3);
  check(rec == shards[2], "parity rebuilds a shard");
}

void test_file_io(const std::string& dir) {
  std::vector<uint8_t> w(1 << 20), r(1 << 20);
  for (size_t i = 0; i < w.size(); ++i) w[i] = (uint8_t)(i * 2654435761u >> 13);
  const std::string path = dir + "/selftest_spill.bin";
  check(vrt::file_write(path, w.data(), w.size(), 0, false, true) == w.size(), "file_write");
  check(vrt::file_read(path, r.data(), r.size(), 0, false) == r.size() && r == w, "file_read");
  bool threw = false;
  try {
    vrt::file_read(dir + "/missing.bin", r.data(), 16, 0, false);
  } catch (const std::exception&) {
    threw = true;
  }
  check(threw, "file_read of a missing file throws");

  // async pool: 4 submitting threads x 8 writes each, then read everything back
  vrt::AsyncIO io(3);
  const int kThreads = 4, kPer = 8, kLen = 4096;
  std::vector<std::vector<uint8_t>> data(kThreads * kPer, std::vector<uint8_t>(kLen));
  std::vector<int64_t> tickets(kThreads * kPer);
  std::vector<std::thread> th;
  for (int t = 0; t < kThreads; ++t) {
    th.emplace_back([&, t] {
      for (int k = 0; k < kPer; ++k) {
        const int id = t * kPer + k;
        for (int i = 0; i < kLen; ++i) data[id][i] = (uint8_t)(id + i);
        tickets[id] = io.submit_write(dir + "/selftest_async_" + std::to_string(id) + ".bin", data[id].data(),
                                      kLen, 0, false);
      }
    });
  }
  for (auto& x : th) x.join();
  size_t moved = 0;
  for (int64_t tk : tickets) moved += io.wait(tk);
  check(moved == (size_t)kThreads * kPer * kLen, "async writes moved every byte");
  std::vector<std::vector<uint8_t>> back(kThreads * kPer, std::vector<uint8_t>(kLen));
  for (int id = 0; id < kThreads * kPer; ++id)
    tickets[id] = io.submit_read(dir + "/selftest_async_" + std::to_string(id) + ".bin", back[id].data(), kLen, 0,
                                 false);
  for (int id = 0; id < kThreads * kPer; ++id) io.wait(tickets[id]);
  check(back == data, "async reads return what was written");
  check(io.pending() == 0, "async pool drained");
}

void test_pages() {
  vrt::PageAllocator pa(64);
  auto a = pa.alloc(40);
  check(a.size() == 40 && pa.num_free() == 24, "alloc 40");
  check(pa.alloc(25).empty() && pa.num_free() == 24, "all-or-nothing alloc");
  pa.incref(a[0]);
  check(pa.refcount(a[0]) == 2, "incref");
  check(!pa.decref(a[0]) && pa.decref(a[0]), "shared page returns on the last decref");
  std::vector<int32_t> rest(a.begin() + 1, a.end());
  pa.free_all(rest);
  check(pa.num_free() == 64, "every page back");
}

void test_tokenizer() {
  std::vector<std::string> texts;
  for (int i = 0; i < 50; ++i) texts.push_back("the quick, brown fox #" + std::to_string(i) + " jumps!");
  auto t1 = vrt::basic_tokenize(texts, 50000, 1);
  auto t4 = vrt::basic_tokenize(texts, 50000, 4);
  check(t1 == t4 && !t1[0].empty(), "tokenizer threads agree");
}

void test_transport() {
  vrt::Listener lst("127.0.0.1", 0);
  const int port = lst.port();
  std::vector<uint8_t> payload(3 * 1000 + 17);
  for (size_t i = 0; i < payload.size(); ++i) payload[i] = (uint8_t)(i * 7);
  std::string sender_error;
  std::thread sender([&] {
    try {
      std::unique_ptr<vrt::Connection> c(vrt::tcp_connect("127.0.0.1", port, 5.0));
      c->send_frame("{\"name\": \"kv\"}", payload.data(), payload.size(), "secret", 1000);
      try {
        // the receiver hangs up at the first bad tag, so this send may fail midway
        c->send_frame("bad", payload.data(), payload.size(), "other-key", 1000);
      } catch (const std::exception&) {
      }
    } catch (const std::exception& e) {
      sender_error = e.what();
    }
  });
  vrt::Connection* s = lst.accept(5.0);
  check(s != nullptr, "accept");
  if (s) {
    std::vector<uint8_t> got;
    uint64_t n = 0;
    const std::string hdr = s->recv_frame("secret", [&](uint64_t m) {
      got.resize(m);
      return got.data();
    }, &n);
    check(hdr == "{\"name\": \"kv\"}" && n == payload.size() && got == payload, "signed frame round trip");
    bool threw = false;
    try {
      s->recv_frame("secret", [&](uint64_t m) {
        got.resize(m);
        return got.data();
      }, &n);
    } catch (const std::exception&) {
      threw = true;
    }
    check(threw, "frame signed with another key is rejected");
    delete s;
  }
  sender.join();
  check(sender_error.empty(), "sender thread");
}

}  // namespace

int main(int argc, char** argv) {
  const std::string dir = argc > 1 ? argv[1] : "/tmp";
  test_crypto();
  test_parity();
  test_file_io(dir);
  test_pages();
  test_tokenizer();
  test_transport();
  std::printf("runtime selftest: %d failure(s)\n", g_fail);
  return g_fail;
}
