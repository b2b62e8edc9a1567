// Allocation-free variant of the split-KV paged decode attention launch (see
// vrm_noalloc.h for who needs it and its limits).  The split partials, the
// per-(sequence, kv head) merge counters and the error word that bounded waits and
// bounds checks report into live in the file-scope device arrays below instead of the
// per-device workspace and error word that the regular launcher allocates lazily.
//
// In host code the array names are host-side stand-ins, not device addresses; the
// device address is resolved once per device with cudaGetSymbolAddress (device
// current) and that pointer is what the kernel receives.
#include <cstring>
#include <mutex>
#include <string>

#include "vrm_host.h"
#include "vrm_kernels.h"
#include "vrm_noalloc.h"

namespace {

static __device__ __align__(256) float g_noalloc_scratch[VRM_NOALLOC_SCRATCH_BYTES / sizeof(float)];
static __device__ __align__(256) uint32_t g_noalloc_counters[VRM_NOALLOC_MAX_GROUPS];
static __device__ __align__(256) uint32_t g_noalloc_err[1];

constexpr int kMaxDevices = 64;

struct DeviceSlot {
  float* scratch = nullptr;
  uint32_t* counters = nullptr;
  uint32_t* err = nullptr;
  bool ready = false;
};

std::mutex g_mu;
DeviceSlot g_slots[kMaxDevices];
thread_local std::string g_last_error;

// Resolves the device addresses of the scratch arrays on `dev` (which is current).
cudaError_t resolve(int dev, DeviceSlot* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceSlot& s = g_slots[dev];
  if (!s.ready) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    void* c = nullptr;
    e = cudaGetSymbolAddress(&c, g_noalloc_counters);
    if (e != cudaSuccess) return e;
    void* w = nullptr;
    e = cudaGetSymbolAddress(&w, g_noalloc_err);
    if (e != cudaSuccess) return e;
    s.scratch = static_cast<float*>(p);
    s.counters = static_cast<uint32_t*>(c);
    s.err = static_cast<uint32_t*>(w);
    s.ready = true;
  }
  *out = s;
  return cudaSuccess;
}

int fail(const std::string& msg) {
  g_last_error = msg;
  return -1;
}

// Resolves the current device's slot; 0 or a failure code (message set).
int current_slot(DeviceSlot* slot) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail("device index out of range");
  e = resolve(dev, slot);
  if (e != cudaSuccess) return fail(std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
  return 0;
}

}  // namespace

extern "C" int vrm_paged_attention_decode_noalloc(const void* q, int64_t ld_q, const void* kv_cache,
                                                  int cache_is_fp8, int num_layers, int layer, int num_kv_heads,
                                                  int head_dim, int num_q_heads, const int* block_tables,
                                                  int block_table_stride, const int* context_lens,
                                                  const float* kv_scale, float sm_scale, void* out, int64_t ld_out,
                                                  int batch, int max_pages, int num_splits, cudaStream_t stream) {
  g_last_error.clear();
  try {
    DeviceSlot slot;
    if (current_slot(&slot) != 0) return -1;
    cudaError_t e = cudaSuccess;
    if (batch <= 0) return 0;
    if (num_kv_heads <= 0 || num_q_heads % num_kv_heads != 0 || num_q_heads / num_kv_heads > 8)
      return fail("GQA group (num_q_heads / num_kv_heads) must be a whole number <= 8");
    if (head_dim != 64 && head_dim != 128) return fail("head_dim must be 64 or 128");
    if (cache_is_fp8 && kv_scale == nullptr) return fail("fp8 cache needs kv_scale");

    const size_t cap = VRM_NOALLOC_SCRATCH_BYTES;
    int splits = num_splits;
    if (splits <= 0) {
      splits = vrm::decode_attention_choose_splits(batch, num_kv_heads, max_pages);
      while (splits > 1 && vrm::decode_attention_scratch_bytes(batch, num_q_heads, head_dim, splits) > cap) --splits;
    }
    if (splits > 128) return fail("num_splits must be <= 128 (got " + std::to_string(splits) + ")");
    const size_t need = vrm::decode_attention_scratch_bytes(batch, num_q_heads, head_dim, splits);
    if (need > cap)
      return fail("request needs " + std::to_string(need) + " bytes of split scratch (batch " + std::to_string(batch) +
                  ", splits " + std::to_string(splits) + "), the allocation-free entry point has " +
                  std::to_string(cap) + "; use fewer splits or a smaller batch");
    if (splits > 1 && (size_t)batch * num_kv_heads > VRM_NOALLOC_MAX_GROUPS)
      return fail("batch * num_kv_heads exceeds " + std::to_string(VRM_NOALLOC_MAX_GROUPS) +
                  " merge counters; use num_splits = 1");
    if (splits > 1) {
      // the merge counters must start at zero (a previous call that did not finish
      // could have left some set)
      e = cudaMemsetAsync(slot.counters, 0, sizeof(uint32_t) * (size_t)batch * num_kv_heads, stream);
      if (e != cudaSuccess) return fail(std::string("cudaMemsetAsync: ") + cudaGetErrorString(e));
    }

    vrm::DecodeAttnArgs a;
    a.q = q;
    a.ld_q = ld_q;
    a.cache = kv_cache;
    a.cache_fp8 = cache_is_fp8 != 0;
    a.num_layers = num_layers;
    a.layer = layer;
    a.KH = num_kv_heads;
    a.D = head_dim;
    a.Hq = num_q_heads;
    a.block_tables = block_tables;
    a.bt_stride = block_table_stride;
    a.context_lens = context_lens;
    a.kv_scale = kv_scale;
    a.sm_scale = sm_scale;
    a.out = out;
    a.ld_o = ld_out;
    a.B = batch;
    a.max_pages = max_pages;
    a.num_splits = splits;
    a.ws = slot.scratch;
    a.ws_bytes = cap;
    a.counters = slot.counters;
    a.err = slot.err;
    vrm::paged_attention_decode(a, stream);
    return 0;
  } catch (const std::exception& ex) {
    return fail(ex.what());
  }
}

extern "C" const char* vrm_noalloc_last_error(void) { return g_last_error.c_str(); }

extern "C" size_t vrm_noalloc_scratch_capacity(void) { return VRM_NOALLOC_SCRATCH_BYTES; }

extern "C" int vrm_noalloc_setup(void) {
  g_last_error.clear();
  DeviceSlot slot;
  return current_slot(&slot);
}

extern "C" int vrm_noalloc_read_and_clear_errors(uint32_t* flags) {
  g_last_error.clear();
  DeviceSlot slot;
  if (current_slot(&slot) != 0) return -1;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(std::string("cudaDeviceSynchronize: ") + cudaGetErrorString(e));
  uint32_t v = 0;
  e = cudaMemcpy(&v, slot.err, sizeof(uint32_t), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(std::string("cudaMemcpy: ") + cudaGetErrorString(e));
  e = cudaMemset(slot.err, 0, sizeof(uint32_t));
  if (e != cudaSuccess) return fail(std::string("cudaMemset: ") + cudaGetErrorString(e));
  if (flags) *flags = v;
  return 0;
}

extern "C" uint64_t vrm_host_device_allocations(void) { return vrm::device_allocations(); }
