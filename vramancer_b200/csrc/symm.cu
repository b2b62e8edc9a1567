// Symmetric device buffers for in-kernel collectives (one process per GPU).
//
// Each rank allocates its buffers with cudaMalloc, exports a CUDA IPC handle, and
// opens its peers' handles, so every kernel gets raw peer pointers it can load from
// or store to over NVLink / NVSwitch.  These allocations are made once at set-up
// (never during stream capture) and live until the process exits.
#include <cstring>
#include <vector>

#include "vrm_host.h"

namespace vrm {

void* symm_malloc(size_t bytes) {
  void* p = nullptr;
  VRM_CUDA_CHECK(cudaMalloc(&p, bytes));
  VRM_CUDA_CHECK(cudaMemset(p, 0, bytes));
  return p;
}

void symm_free(void* p) {
  if (p) cudaFree(p);
}

namespace {
__global__ void fill_u16_kernel(uint16_t* p, size_t n, uint16_t v) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}
}  // namespace

void symm_fill_u16(void* p, size_t count, uint16_t value) {
  if (count == 0) return;
  fill_u16_kernel<<<256, 256>>>(static_cast<uint16_t*>(p), count, value);
  VRM_CUDA_CHECK(cudaGetLastError());
  VRM_CUDA_CHECK(cudaDeviceSynchronize());
}

std::vector<uint8_t> ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  VRM_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  std::vector<uint8_t> out(sizeof(h));
  std::memcpy(out.data(), &h, sizeof(h));
  return out;
}

void* ipc_open(const std::vector<uint8_t>& bytes) {
  VRM_REQUIRE(bytes.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, bytes.data(), sizeof(h));
  void* p = nullptr;
  VRM_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return p;
}

void ipc_close(void* p) {
  if (p) cudaIpcCloseMemHandle(p);
}

}  // namespace vrm
