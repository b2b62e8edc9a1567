// Host-side runtime services shared by every kernel launcher (plain CUDA runtime,
// no framework dependency):
//   * the cuTensorMapEncodeTiled entry point (fetched from the driver at run time,
//     so the library does not link libcuda directly)
//   * a per-device error word that bounded device-side waits report into
//   * a per-device split-K / split-KV workspace and a zeroed tile-counter array
// Failures throw std::runtime_error.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>
#include <utility>

namespace vrm {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tensor_map();

#define VRM_CUDA_CHECK(expr)                                                                       \
  do {                                                                                             \
    cudaError_t _e = (expr);                                                                       \
    if (_e != cudaSuccess)                                                                         \
      throw std::runtime_error(std::string("CUDA error ") + cudaGetErrorString(_e) + " at " +      \
                               __FILE__ + ":" + std::to_string(__LINE__));                         \
  } while (0)

#define VRM_REQUIRE(cond, msg)                                                                     \
  do {                                                                                             \
    if (!(cond)) throw std::runtime_error(std::string("vramancer_b200: ") + (msg));                \
  } while (0)

// Device word (current device) that kernels atomically OR error codes into.
uint32_t* error_word();
// Reads and clears the current device's error word (synchronises the device).
uint32_t read_and_clear_errors();

// Persistent scratch of at least `bytes` on the current device.  Grows only when
// `stream` is not capturing; old buffers are never freed while the process lives
// (graphs captured earlier may still point at them).
void* workspace_get(size_t bytes, cudaStream_t stream);
void workspace_reserve(size_t bytes, cudaStream_t stream);
size_t workspace_size();
// Zero-initialised uint32 counters (65536 per device); every user resets the
// ones it touched before its kernel exits.
uint32_t* tile_counters_get(cudaStream_t stream);

int device_sm_count();

// Number of device allocations (cudaMalloc) this library's host services have made in
// this process, all devices together.
uint64_t device_allocations();

// Programmatic dependent launch on/off (env VRM_PDL, default on).
bool pdl_enabled();

// Launches `kern` with the programmatic-stream-serialization attribute when PDL is
// enabled, so its CTAs may start while the previous kernel drains; every kernel
// launched this way calls pdl_wait() before touching data the predecessor produced.
template <typename... KArgs, typename... Args>
void launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  VRM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

// launch_kernel with a thread-block cluster of `cluster` CTAs (grid.x, .y, .z each a
// multiple of the cluster's extent along that axis).
template <typename... KArgs, typename... Args>
void launch_kernel_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, dim3 cluster, size_t smem,
                           cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cluster.x;
  attr[0].val.clusterDim.y = cluster.y;
  attr[0].val.clusterDim.z = cluster.z;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  VRM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...));
}

}  // namespace vrm
