// Virtual-memory regions whose chunks are backed by memory on chosen GPUs (CUDA VMM).
//
// A KV pool that may borrow pages from another GPU reserves one contiguous virtual
// range for all its pages; the local pages are backed by this GPU's HBM and borrowed
// chunks by physical memory created on the lender GPU and mapped into the tail of the
// same range, readable and writable from both GPUs.  Every kernel that indexes the
// pool from its base pointer (paged attention, KV writes, page copies) then reads a
// borrowed page in place over NVLink with ordinary loads; nothing else changes.
//
// Chunks can also be exported as POSIX file descriptors and mapped in another process
// (a lender rank on another GPU of the same node).  Driver entry points are resolved
// at run time (cudaGetDriverEntryPoint), so the library does not link libcuda.
#include <cuda.h>
#include <cuda_runtime.h>

#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

namespace {

struct Drv {
  decltype(&cuMemGetAllocationGranularity) granularity = nullptr;
  decltype(&cuMemAddressReserve) reserve = nullptr;
  decltype(&cuMemAddressFree) addr_free = nullptr;
  decltype(&cuMemCreate) create = nullptr;
  decltype(&cuMemRelease) release = nullptr;
  decltype(&cuMemMap) map = nullptr;
  decltype(&cuMemUnmap) unmap = nullptr;
  decltype(&cuMemSetAccess) set_access = nullptr;
  decltype(&cuMemExportToShareableHandle) export_handle = nullptr;
  decltype(&cuMemImportFromShareableHandle) import_handle = nullptr;
};

template <typename F>
void resolve(F* fn, const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q);
  VRM_REQUIRE(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p,
              std::string("could not resolve ") + name + " from the CUDA driver");
  *fn = reinterpret_cast<F>(p);
}

const Drv& drv() {
  static Drv d;
  static std::once_flag once;
  std::call_once(once, [] {
    resolve(&d.granularity, "cuMemGetAllocationGranularity");
    resolve(&d.reserve, "cuMemAddressReserve");
    resolve(&d.addr_free, "cuMemAddressFree");
    resolve(&d.create, "cuMemCreate");
    resolve(&d.release, "cuMemRelease");
    resolve(&d.map, "cuMemMap");
    resolve(&d.unmap, "cuMemUnmap");
    resolve(&d.set_access, "cuMemSetAccess");
    resolve(&d.export_handle, "cuMemExportToShareableHandle");
    resolve(&d.import_handle, "cuMemImportFromShareableHandle");
  });
  return d;
}

void check(CUresult r, const char* what) {
  VRM_REQUIRE(r == CUDA_SUCCESS, std::string(what) + " failed (CUresult " + std::to_string((int)r) + ")");
}

struct Region {
  size_t bytes = 0;
  std::map<size_t, std::pair<size_t, CUmemGenericAllocationHandle>> chunks;   // offset -> (bytes, handle)
};

std::mutex g_mu;
std::map<CUdeviceptr, Region> g_regions;

CUmemAllocationProp prop_for(int device, bool shareable) {
  CUmemAllocationProp prop = {};
  prop.type = CU_MEM_ALLOCATION_TYPE_PINNED;
  prop.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
  prop.location.id = device;
  prop.requestedHandleTypes = shareable ? CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR : CU_MEM_HANDLE_TYPE_NONE;
  return prop;
}

void grant(CUdeviceptr at, size_t bytes, const std::vector<int>& devices) {
  std::vector<CUmemAccessDesc> acc(devices.size());
  for (size_t i = 0; i < devices.size(); ++i) {
    acc[i].location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc[i].location.id = devices[i];
    acc[i].flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
  }
  check(drv().set_access(at, bytes, acc.data(), acc.size()), "cuMemSetAccess");
}

Region& region_of(uint64_t base) {
  auto it = g_regions.find((CUdeviceptr)base);
  VRM_REQUIRE(it != g_regions.end(), "vmm: unknown region");
  return it->second;
}

}  // namespace

size_t vmm_granularity(int device) {
  CUmemAllocationProp prop = prop_for(device, true);
  size_t g = 0;
  check(drv().granularity(&g, &prop, CU_MEM_ALLOC_GRANULARITY_MINIMUM), "cuMemGetAllocationGranularity");
  return g;
}

uint64_t vmm_reserve(size_t bytes, size_t alignment) {
  CUdeviceptr p = 0;
  check(drv().reserve(&p, bytes, alignment, 0, 0), "cuMemAddressReserve");
  std::lock_guard<std::mutex> lk(g_mu);
  g_regions[p].bytes = bytes;
  return (uint64_t)p;
}

void vmm_map(uint64_t base, size_t offset, size_t bytes, int location_device, const std::vector<int>& access,
             bool shareable) {
  std::lock_guard<std::mutex> lk(g_mu);
  Region& r = region_of(base);
  VRM_REQUIRE(offset + bytes <= r.bytes, "vmm: chunk outside the region");
  VRM_REQUIRE(!r.chunks.count(offset), "vmm: chunk already mapped");
  CUmemAllocationProp prop = prop_for(location_device, shareable);
  CUmemGenericAllocationHandle h;
  check(drv().create(&h, bytes, &prop, 0), "cuMemCreate");
  CUresult m = drv().map((CUdeviceptr)base + offset, bytes, 0, h, 0);
  if (m != CUDA_SUCCESS) {
    drv().release(h);
    check(m, "cuMemMap");
  }
  r.chunks[offset] = {bytes, h};
  grant((CUdeviceptr)base + offset, bytes, access);
}

int vmm_export_fd(uint64_t base, size_t offset) {
  std::lock_guard<std::mutex> lk(g_mu);
  Region& r = region_of(base);
  auto it = r.chunks.find(offset);
  VRM_REQUIRE(it != r.chunks.end(), "vmm: no chunk at that offset");
  int fd = -1;
  check(drv().export_handle(&fd, it->second.second, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
        "cuMemExportToShareableHandle");
  return fd;
}

void vmm_map_fd(uint64_t base, size_t offset, size_t bytes, int fd, const std::vector<int>& access) {
  std::lock_guard<std::mutex> lk(g_mu);
  Region& r = region_of(base);
  VRM_REQUIRE(offset + bytes <= r.bytes && !r.chunks.count(offset), "vmm: bad chunk for an imported handle");
  CUmemGenericAllocationHandle h;
  check(drv().import_handle(&h, (void*)(intptr_t)fd, CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
        "cuMemImportFromShareableHandle");
  CUresult m = drv().map((CUdeviceptr)base + offset, bytes, 0, h, 0);
  if (m != CUDA_SUCCESS) {
    drv().release(h);
    check(m, "cuMemMap");
  }
  r.chunks[offset] = {bytes, h};
  grant((CUdeviceptr)base + offset, bytes, access);
}

void vmm_unmap(uint64_t base, size_t offset) {
  std::lock_guard<std::mutex> lk(g_mu);
  Region& r = region_of(base);
  auto it = r.chunks.find(offset);
  VRM_REQUIRE(it != r.chunks.end(), "vmm: no chunk at that offset");
  VRM_CUDA_CHECK(cudaDeviceSynchronize());     // no kernel may still read the chunk
  check(drv().unmap((CUdeviceptr)base + offset, it->second.first), "cuMemUnmap");
  check(drv().release(it->second.second), "cuMemRelease");
  r.chunks.erase(it);
}

void vmm_free(uint64_t base) {
  std::lock_guard<std::mutex> lk(g_mu);
  Region& r = region_of(base);
  VRM_CUDA_CHECK(cudaDeviceSynchronize());
  for (auto& kv : r.chunks) {
    drv().unmap((CUdeviceptr)base + kv.first, kv.second.first);
    drv().release(kv.second.second);
  }
  drv().addr_free((CUdeviceptr)base, r.bytes);
  g_regions.erase((CUdeviceptr)base);
}

}  // namespace vrm
