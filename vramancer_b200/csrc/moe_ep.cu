// Expert-parallel MoE exchange over peer memory (NVLink P2P stores into CUDA IPC
// buffers; no NCCL, no host round trip, graph-capturable).  One layer call is
//   counts   this rank's per-expert pair counts -> every rank (advances the epoch)
//   dispatch every routed row -> its expert owner's receive buffer, grouped by local
//            expert then source rank, with a (source rank, pair) tag
//   owner    block list over the local experts once every rank's rows have landed
//   gemms    grouped gate/up, then grouped down whose epilogue stores each row back
//            into the source rank's return buffer (gemm_tc.cu, moe_ep_grouped_return)
//   combine  weighted k-order sum of the returned rows (moe.cu, moe_ep_combine)
// Each phase flags every peer with the epoch (release at system scope after one
// system fence behind a CTA barrier); waits are acquire loads with a bounded spin that
// records kErrFlagTimeout and gives up.  Buffers alternate halves with the epoch's
// parity: a rank can be at most one call ahead of any peer, because each call waits
// for every peer's counts before writing into the peers' halves.
//
// Reference parity: the reference has no expert parallelism (MoE only through vLLM /
// llama.cpp; core/expert_pinning.py:281-640 mirrors cold experts onto a lender GPU).
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kPhaseCount = 0, kPhaseDispatch = 1, kPhaseReturn = 2;
constexpr int kEpMaxExperts = 2048;

// thread-0 wait for every rank's flag of `phase` to reach epoch; false on timeout
__device__ bool wait_all(const MoeEpBuffers& b, int phase, uint32_t epoch, uint32_t* err) {
  const uint32_t* f = b.flags[b.rank] + phase * b.world;
  for (int r = 0; r < b.world; ++r) {
    const unsigned long long t0 = clock64();
    while ((int)(ld_acquire_sys(f + r) - epoch) < 0) {
      if ((unsigned long long)(clock64() - t0) > VRM_SPIN_LIMIT_CYCLES) {
        report_error(err, kErrFlagTimeout);
        return false;
      }
    }
  }
  return true;
}

__device__ void flag_all(const MoeEpBuffers& b, int phase, uint32_t epoch) {
  asm volatile("fence.acq_rel.sys;" ::: "memory");
  for (int o = 0; o < b.world; ++o) st_release_sys(b.flags[o] + phase * b.world + b.rank, epoch);
}

__global__ void __launch_bounds__(256) ep_counts_kernel(MoeEpBuffers b, const int* counts, int T) {
  pdl_launch();
  pdl_wait_for(counts);
  __shared__ uint32_t s_epoch;
  if (threadIdx.x == 0) {
    s_epoch = *b.epoch + 1u;
    *b.epoch = s_epoch;
  }
  __syncthreads();
  const uint32_t ep = s_epoch;
  const int par = ep & 1u;
  for (int o = 0; o < b.world; ++o) {
    int* dst = b.cnt[o] + ((size_t)par * b.world + b.rank) * b.E;
    for (int e = threadIdx.x; e < b.E; e += blockDim.x) dst[e] = T > 0 ? counts[e] : 0;
  }
  __syncthreads();
  if (threadIdx.x == 0) flag_all(b, kPhaseCount, ep);
}

// 8 warps per CTA, one routed pair per warp at a time
__global__ void __launch_bounds__(256) ep_dispatch_kernel(MoeEpBuffers b, const __nv_bfloat16* x, const int* ids,
                                                          const int* row_of, const int* offsets, int P, int topk,
                                                          uint32_t* err) {
  pdl_launch();
  pdl_wait_for(x, ids, row_of, offsets);
  __shared__ int base[kEpMaxExperts];
  __shared__ int pre[kEpMaxExperts];
  __shared__ int ok;
  const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(b.epoch);
  const int par = ep & 1u;
  if (threadIdx.x == 0) ok = wait_all(b, kPhaseCount, ep, err) ? 1 : 0;
  __syncthreads();
  const int W = b.world, E = b.E;
  if (ok) {
    // every rank's counts: base row of (expert e, this rank) in e's owner's buffer
    const int* cnt = b.cnt[b.rank] + (size_t)par * W * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      int tot = 0, before = 0;
      for (int r = 0; r < W; ++r) {
        const int c = __ldcg(cnt + (size_t)r * E + e);
        tot += c;
        if (r < b.rank) before += c;
      }
      base[e] = tot;
      pre[e] = before;
    }
    __syncthreads();
    if (threadIdx.x < W) {
      int s = 0;
      for (int j = 0; j < b.E_local; ++j) {
        const int e = threadIdx.x * b.E_local + j;
        const int t = base[e];
        base[e] = s + pre[e];
        s += t;
      }
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nvec = b.H / 8;
    for (int p = blockIdx.x * 8 + warp; p < P; p += gridDim.x * 8) {
      const int e = ids[p];
      const int o = e / b.E_local;
      const int row = base[e] + (row_of[p] - offsets[e]);
      if (row < 0 || row >= b.r_rows) {
        if (lane == 0) report_error(err, kErrBadShape);
        continue;
      }
      const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)(p / topk) * b.H);
      uint4* dst = reinterpret_cast<uint4*>(b.xrecv[o] + ((size_t)par * b.r_rows + row) * b.H);
      for (int v = lane; v < nvec; v += 32) dst[v] = src[v];
      if (lane == 0) b.meta[o][(size_t)par * b.r_rows + row] = b.rank * b.p_cap + p;
    }
  }
  // the last CTA to finish flags every owner (its stores and ours ordered by the fences)
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(b.done) : "memory");
    if (prev == gridDim.x - 1) {
      *b.done = 0u;
      flag_all(b, kPhaseDispatch, ep);
    }
  }
}

__global__ void __launch_bounds__(128) ep_owner_plan_kernel(MoeEpBuffers b, int BN, MoeBlock* blocks, int* num_blocks,
                                                            int max_blocks, uint32_t* err) {
  pdl_launch();
  pdl_wait();
  const uint32_t ep = *reinterpret_cast<volatile uint32_t*>(b.epoch);
  const int par = ep & 1u;
  if (threadIdx.x != 0) return;
  const bool ok = wait_all(b, kPhaseDispatch, ep, err);
  // the peers' rows are read by the next kernels' TMA (async proxy)
  asm volatile("fence.proxy.async.global;" ::: "memory");
  const int* cnt = b.cnt[b.rank] + (size_t)par * b.world * b.E;
  int row = 0, nb = 0;
  for (int j = 0; ok && j < b.E_local; ++j) {
    const int e = b.rank * b.E_local + j;
    int n = 0;
    for (int r = 0; r < b.world; ++r) n += __ldcg(cnt + (size_t)r * b.E + e);
    for (int r0 = 0; r0 < n; r0 += BN) {
      if (nb < max_blocks) blocks[nb] = MoeBlock{j, par * b.r_rows + row + r0, min(BN, n - r0), 0};
      ++nb;
    }
    row += n;
  }
  if (nb > max_blocks) {
    report_error(err, kErrBadShape);
    nb = max_blocks;
  }
  *num_blocks = nb;
}

}  // namespace

void moe_ep_counts(const MoeEpBuffers& b, const int* counts, int T, cudaStream_t st) {
  VRM_REQUIRE(b.E > 0 && b.E <= kEpMaxExperts && b.world >= 1 && b.E == b.E_local * b.world, "moe_ep: bad sizes");
  launch_kernel(ep_counts_kernel, dim3(1), dim3(256), 0, st, b, counts, T);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_ep_dispatch(const MoeEpBuffers& b, const void* x, const int* ids32, const int* row_of, const int* offsets,
                     int T, int topk, cudaStream_t st) {
  VRM_REQUIRE(b.H % 8 == 0 && (long long)T * topk <= b.p_cap, "moe_ep_dispatch: H % 8 or pair capacity");
  const int P = T * topk;
  const int grid = std::max(1, std::min((P + 7) / 8, 4 * device_sm_count()));
  launch_kernel(ep_dispatch_kernel, dim3(grid), dim3(256), 0, st, b, reinterpret_cast<const __nv_bfloat16*>(x),
                ids32, row_of, offsets, P, topk, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_ep_owner_plan(const MoeEpBuffers& b, int BN, MoeBlock* blocks, int* num_blocks, int max_blocks,
                       cudaStream_t st) {
  launch_kernel(ep_owner_plan_kernel, dim3(1), dim3(128), 0, st, b, BN, blocks, num_blocks, max_blocks,
                error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
