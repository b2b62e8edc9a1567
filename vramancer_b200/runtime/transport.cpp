// Framed tensor transport over TCP with optional per-chunk HMAC-SHA256 tags.
//
// Reference parity: rust_core/src/lib.rs:857-980, 1123-1250 (Tokio TCP tensor
// send / recv, chunked with a per-chunk HMAC, 16 GiB bound) and the VTP framing of
// core/network/llm_transport.py.  Blocking sockets; the caller releases the GIL.
#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <stdexcept>

#include "runtime.h"

namespace vrt {
namespace {

constexpr char kMagic[4] = {'V', 'R', 'T', '1'};

void send_all(int fd, const void* p, size_t n) {
  const auto* b = static_cast<const uint8_t*>(p);
  while (n) {
    const ssize_t w = ::send(fd, b, n, MSG_NOSIGNAL);
    if (w < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(std::string("send: ") + std::strerror(errno));
    }
    b += w;
    n -= (size_t)w;
  }
}

void recv_all(int fd, void* p, size_t n) {
  auto* b = static_cast<uint8_t*>(p);
  while (n) {
    const ssize_t r = ::recv(fd, b, n, 0);
    if (r < 0) {
      if (errno == EINTR) continue;
      throw std::runtime_error(std::string("recv: ") + std::strerror(errno));
    }
    if (r == 0) throw std::runtime_error("recv: connection closed");
    b += r;
    n -= (size_t)r;
  }
}

void chunk_tag(const std::string& key, uint64_t seq, const uint8_t* p, size_t n, uint8_t out[32]) {
  HmacSha256 h(reinterpret_cast<const uint8_t*>(key.data()), key.size());
  uint8_t s[8];
  for (int i = 0; i < 8; ++i) s[i] = (uint8_t)(seq >> (8 * i));
  h.update(s, 8);
  h.update(p, n);
  h.finish(out);
}

void tune(int fd) {
  int one = 1;
  ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  int buf = 8 << 20;
  ::setsockopt(fd, SOL_SOCKET, SO_SNDBUF, &buf, sizeof(buf));
  ::setsockopt(fd, SOL_SOCKET, SO_RCVBUF, &buf, sizeof(buf));
}

}  // namespace

Connection::~Connection() { close(); }

void Connection::close() {
  if (fd_ >= 0) ::close(fd_);
  fd_ = -1;
}

void Connection::send_frame(const std::string& header, const uint8_t* payload, uint64_t n, const std::string& key,
                            uint32_t chunk) {
  if (n > kMaxPayload) throw std::invalid_argument("payload larger than 16 GiB");
  if (chunk == 0) chunk = 16u << 20;
  const uint32_t flags = key.empty() ? 0u : 1u;
  uint8_t hdr[24];
  std::memcpy(hdr, kMagic, 4);
  const uint32_t hl = (uint32_t)header.size();
  std::memcpy(hdr + 4, &hl, 4);
  std::memcpy(hdr + 8, &n, 8);
  std::memcpy(hdr + 16, &chunk, 4);
  std::memcpy(hdr + 20, &flags, 4);
  send_all(fd_, hdr, sizeof(hdr));
  send_all(fd_, header.data(), header.size());
  uint64_t seq = 0;
  for (uint64_t off = 0; off < n; off += chunk, ++seq) {
    const size_t len = (size_t)std::min<uint64_t>(chunk, n - off);
    send_all(fd_, payload + off, len);
    if (flags & 1u) {
      uint8_t tag[32];
      chunk_tag(key, seq, payload + off, len, tag);
      send_all(fd_, tag, 32);
    }
  }
}

std::string Connection::recv_frame(const std::string& key, const std::function<uint8_t*(uint64_t)>& alloc,
                                   uint64_t* n_out) {
  uint8_t hdr[24];
  recv_all(fd_, hdr, sizeof(hdr));
  if (std::memcmp(hdr, kMagic, 4) != 0) throw std::runtime_error("bad frame magic");
  uint32_t hl, chunk, flags;
  uint64_t n;
  std::memcpy(&hl, hdr + 4, 4);
  std::memcpy(&n, hdr + 8, 8);
  std::memcpy(&chunk, hdr + 16, 4);
  std::memcpy(&flags, hdr + 20, 4);
  if (n > kMaxPayload || hl > (64u << 20) || chunk == 0) throw std::runtime_error("frame header out of range");
  if ((flags & 1u) && key.empty()) throw std::runtime_error("frame is signed but no key was given");
  if (!(flags & 1u) && !key.empty()) throw std::runtime_error("unsigned frame where a signature is required");
  std::string header(hl, '\0');
  recv_all(fd_, header.data(), hl);
  uint8_t* dst = alloc(n);
  uint64_t seq = 0;
  for (uint64_t off = 0; off < n; off += chunk, ++seq) {
    const size_t len = (size_t)std::min<uint64_t>(chunk, n - off);
    recv_all(fd_, dst + off, len);
    if (flags & 1u) {
      uint8_t tag[32], want[32];
      recv_all(fd_, tag, 32);
      chunk_tag(key, seq, dst + off, len, want);
      if (!ct_equal(tag, want, 32)) throw std::runtime_error("chunk signature mismatch");
    }
  }
  *n_out = n;
  return header;
}

Connection* tcp_connect(const std::string& host, int port, double timeout_s) {
  addrinfo hints{}, *res = nullptr;
  hints.ai_family = AF_UNSPEC;
  hints.ai_socktype = SOCK_STREAM;
  const std::string ps = std::to_string(port);
  if (::getaddrinfo(host.c_str(), ps.c_str(), &hints, &res) != 0 || !res)
    throw std::runtime_error("cannot resolve " + host);
  int fd = -1;
  std::string last = "no address";
  for (addrinfo* a = res; a; a = a->ai_next) {
    fd = ::socket(a->ai_family, a->ai_socktype, a->ai_protocol);
    if (fd < 0) continue;
    timeval tv{};
    tv.tv_sec = (long)timeout_s;
    tv.tv_usec = (long)((timeout_s - (long)timeout_s) * 1e6);
    ::setsockopt(fd, SOL_SOCKET, SO_SNDTIMEO, &tv, sizeof(tv));
    ::setsockopt(fd, SOL_SOCKET, SO_RCVTIMEO, &tv, sizeof(tv));
    if (::connect(fd, a->ai_addr, a->ai_addrlen) == 0) break;
    last = std::strerror(errno);
    ::close(fd);
    fd = -1;
  }
  ::freeaddrinfo(res);
  if (fd < 0) throw std::runtime_error("connect " + host + ":" + ps + ": " + last);
  tune(fd);
  return new Connection(fd);
}

Listener::Listener(const std::string& host, int port) {
  fd_ = ::socket(AF_INET, SOCK_STREAM, 0);
  if (fd_ < 0) throw std::runtime_error("socket failed");
  int one = 1;
  ::setsockopt(fd_, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
  sockaddr_in addr{};
  addr.sin_family = AF_INET;
  addr.sin_port = htons((uint16_t)port);
  if (::inet_pton(AF_INET, host.c_str(), &addr.sin_addr) != 1) throw std::runtime_error("bad IPv4 address " + host);
  if (::bind(fd_, reinterpret_cast<sockaddr*>(&addr), sizeof(addr)) != 0)
    throw std::runtime_error(std::string("bind: ") + std::strerror(errno));
  if (::listen(fd_, 16) != 0) throw std::runtime_error(std::string("listen: ") + std::strerror(errno));
  socklen_t len = sizeof(addr);
  ::getsockname(fd_, reinterpret_cast<sockaddr*>(&addr), &len);
  port_ = ntohs(addr.sin_port);
}

Listener::~Listener() { close(); }

void Listener::close() {
  if (fd_ >= 0) ::close(fd_);
  fd_ = -1;
}

Connection* Listener::accept(double timeout_s) {
  pollfd pfd{fd_, POLLIN, 0};
  const int r = ::poll(&pfd, 1, timeout_s < 0 ? -1 : (int)(timeout_s * 1000));
  if (r == 0) return nullptr;
  if (r < 0) throw std::runtime_error(std::string("poll: ") + std::strerror(errno));
  const int c = ::accept(fd_, nullptr, nullptr);
  if (c < 0) throw std::runtime_error(std::string("accept: ") + std::strerror(errno));
  tune(c);
  return new Connection(c);
}

}  // namespace vrt
