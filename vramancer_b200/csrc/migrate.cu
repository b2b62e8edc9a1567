// KV page migration between pools (same GPU or a peer GPU over NVLink/NVSwitch).
//
// page_copy_kernel copies whole pages  dst[dst_idx[i]] <- src[src_idx[i]]  where a page
// is `page_bytes` contiguous bytes (all layers of 16 tokens: 3 MiB for the
// Qwen2.5-14B shape).  The launch runs on the source GPU and pushes 16-byte vector
// stores into the destination pool (a peer pointer when the pools live on different
// GPUs: fire-and-forget NVLink writes, no CPU staging, no copy-engine round trips).
// Work is cut into 32 KiB chunks; each CTA loads 8 vectors per thread before storing
// them, so every thread keeps 128 B of reads in flight.
//
// Reference parity: the reference moves lending-pool pages through TransferManager ->
// Rust GpuPipeline, CPU-staged triple buffering on its PCIe box
// (rust_core/src/lib.rs:578-830, benchmarks/bench_kv_migration.py:70-117).
#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

constexpr int kCopyThreads = 256;
constexpr int kVecPerThread = 8;                                   // 8 x 16 B
constexpr int kChunkVecs = kCopyThreads * kVecPerThread;           // 2048 vectors = 32 KiB

__global__ void __launch_bounds__(kCopyThreads)
    page_copy_kernel(const uint4* __restrict__ src, uint4* __restrict__ dst, const int* __restrict__ src_idx,
                     const int* __restrict__ dst_idx, int n_pages, long long page_vecs, long long src_pages,
                     long long dst_pages, uint32_t* err) {
  pdl_launch();
  pdl_wait_for(src, src_idx, dst_idx);
  const long long chunks_per_page = (page_vecs + kChunkVecs - 1) / kChunkVecs;
  const long long total = (long long)n_pages * chunks_per_page;
  for (long long w = blockIdx.x; w < total; w += gridDim.x) {
    const int p = (int)(w / chunks_per_page);
    const long long c = w - (long long)p * chunks_per_page;
    if (!in_bounds(src_idx[p], src_pages, err) || !in_bounds(dst_idx[p], dst_pages, err)) continue;
    const uint4* s = src + (long long)src_idx[p] * page_vecs + c * kChunkVecs;
    uint4* d = dst + (long long)dst_idx[p] * page_vecs + c * kChunkVecs;
    const long long lim = min((long long)kChunkVecs, page_vecs - c * kChunkVecs);
    uint4 v[kVecPerThread];
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      const long long i = threadIdx.x + (long long)j * kCopyThreads;
      if (i < lim) v[j] = __ldcs(s + i);            // streamed once: do not keep in L2
    }
#pragma unroll
    for (int j = 0; j < kVecPerThread; ++j) {
      const long long i = threadIdx.x + (long long)j * kCopyThreads;
      if (i < lim) __stcs(d + i, v[j]);
    }
  }
}

void page_copy(const void* src_pool, void* dst_pool, const int* src_idx, const int* dst_idx, int n_pages,
               size_t page_bytes, cudaStream_t stream, int64_t src_pages, int64_t dst_pages) {
  if (n_pages <= 0) return;
  VRM_REQUIRE(page_bytes % 16 == 0, "page_copy: page size must be a multiple of 16 bytes");
  VRM_REQUIRE((reinterpret_cast<uintptr_t>(src_pool) & 15) == 0 && (reinterpret_cast<uintptr_t>(dst_pool) & 15) == 0,
              "page_copy: pools must be 16-byte aligned");
  const long long page_vecs = (long long)(page_bytes / 16);
  const long long chunks = (long long)n_pages * ((page_vecs + kChunkVecs - 1) / kChunkVecs);
  const int grid = (int)std::min<long long>(chunks, (long long)device_sm_count() * 4);
  launch_kernel(page_copy_kernel, dim3(grid), dim3(kCopyThreads), 0, stream, reinterpret_cast<const uint4*>(src_pool),
                reinterpret_cast<uint4*>(dst_pool), src_idx, dst_idx, n_pages, page_vecs, (long long)src_pages,
                (long long)dst_pages, error_word());
}

bool enable_peer_access(int device, int peer) {
  int can = 0;
  VRM_CUDA_CHECK(cudaDeviceCanAccessPeer(&can, device, peer));
  if (!can) return false;
  int prev = 0;
  VRM_CUDA_CHECK(cudaGetDevice(&prev));
  VRM_CUDA_CHECK(cudaSetDevice(device));
  cudaError_t e = cudaDeviceEnablePeerAccess(peer, 0);
  if (e == cudaErrorPeerAccessAlreadyEnabled) {
    cudaGetLastError();   // clear the sticky-free status of this benign error
    e = cudaSuccess;
  }
  cudaSetDevice(prev);
  VRM_CUDA_CHECK(e);
  return true;
}

}  // namespace vrm
