// Host runtime services (see vrm_host.h).
#include "vrm_host.h"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>

namespace vrm {

namespace {
constexpr int kMaxDevices = 64;
constexpr size_t kCounterCount = 1 << 16;

struct DeviceScratch {
  uint32_t* err = nullptr;
  void* ws = nullptr;
  size_t ws_bytes = 0;
  uint32_t* counters = nullptr;
  int sms = 0;
};

std::mutex g_mu;
DeviceScratch g_dev[kMaxDevices];
std::atomic<uint64_t> g_allocs{0};

// every device allocation of the host services goes through here (counted)
cudaError_t counted_malloc(void** p, size_t bytes) {
  g_allocs.fetch_add(1, std::memory_order_relaxed);
  return cudaMalloc(p, bytes);
}

int current_device() {
  int d = 0;
  VRM_CUDA_CHECK(cudaGetDevice(&d));
  VRM_REQUIRE(d < kMaxDevices, "device index out of range");
  return d;
}

bool capturing(cudaStream_t s) {
  cudaStreamCaptureStatus st = cudaStreamCaptureStatusNone;
  cudaStreamIsCapturing(s, &st);
  return st != cudaStreamCaptureStatusNone;
}
}  // namespace

EncodeTiledFn encode_tensor_map() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess) fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  VRM_REQUIRE(fn != nullptr, "could not resolve cuTensorMapEncodeTiled from the CUDA driver");
  return fn;
}

uint32_t* error_word() {
  const int d = current_device();
  std::lock_guard<std::mutex> g(g_mu);
  if (!g_dev[d].err) {
    VRM_CUDA_CHECK(counted_malloc(reinterpret_cast<void**>(&g_dev[d].err), sizeof(uint32_t)));
    VRM_CUDA_CHECK(cudaMemset(g_dev[d].err, 0, sizeof(uint32_t)));
  }
  return g_dev[d].err;
}

uint32_t read_and_clear_errors() {
  uint32_t* w = error_word();
  uint32_t v = 0;
  VRM_CUDA_CHECK(cudaDeviceSynchronize());
  VRM_CUDA_CHECK(cudaMemcpy(&v, w, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  VRM_CUDA_CHECK(cudaMemset(w, 0, sizeof(uint32_t)));
  return v;
}

void* workspace_get(size_t bytes, cudaStream_t stream) {
  const int d = current_device();
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& s = g_dev[d];
  if (bytes > s.ws_bytes) {
    VRM_REQUIRE(!capturing(stream),
                "workspace too small during CUDA graph capture; reserve_workspace() before capture");
    size_t sz = std::max(bytes, (size_t)32 << 20);
    void* p = nullptr;
    VRM_CUDA_CHECK(counted_malloc(&p, sz));
    // the old buffer is intentionally kept: captured graphs may still use it
    s.ws = p;
    s.ws_bytes = sz;
  }
  return s.ws;
}

void workspace_reserve(size_t bytes, cudaStream_t stream) {
  (void)workspace_get(bytes, stream);
  (void)tile_counters_get(stream);
  (void)error_word();
}

size_t workspace_size() {
  const int d = current_device();
  std::lock_guard<std::mutex> g(g_mu);
  return g_dev[d].ws_bytes;
}

uint32_t* tile_counters_get(cudaStream_t stream) {
  const int d = current_device();
  std::lock_guard<std::mutex> g(g_mu);
  DeviceScratch& s = g_dev[d];
  if (!s.counters) {
    VRM_REQUIRE(!capturing(stream), "tile counters must be created before CUDA graph capture");
    VRM_CUDA_CHECK(counted_malloc(reinterpret_cast<void**>(&s.counters), kCounterCount * sizeof(uint32_t)));
    VRM_CUDA_CHECK(cudaMemset(s.counters, 0, kCounterCount * sizeof(uint32_t)));
  }
  return s.counters;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VRM_PDL");
    return !(e && (e[0] == '0' || e[0] == 'n' || e[0] == 'N'));
  }();
  return on;
}

int device_sm_count() {
  const int d = current_device();
  std::lock_guard<std::mutex> g(g_mu);
  if (g_dev[d].sms == 0) VRM_CUDA_CHECK(cudaDeviceGetAttribute(&g_dev[d].sms, cudaDevAttrMultiProcessorCount, d));
  return g_dev[d].sms;
}

uint64_t device_allocations() { return g_allocs.load(std::memory_order_relaxed); }

}  // namespace vrm
