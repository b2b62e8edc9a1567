// Mixture-of-experts routing on the device: plan (counts, grouped rows, token blocks),
// gather of the routed activations, and the weighted combine back to token order.  The
// expert GEMMs in between are the grouped tcgen05 kernel of gemm_tc.cu.  Nothing here
// reads back to the host, so a whole MoE layer can be captured in a CUDA graph.
//
// Grouped row order within an expert follows atomic arrival, which may vary between
// runs; every grouped row is computed independently and the combine sums each token's
// top-k rows in k order, so the layer output does not depend on it.
//
// Ordering under programmatic dependent launch: the plan is consumed up to four
// kernels later (gather, both grouped GEMMs, combine), by grids that the chain of
// early triggers may have launched before the plan kernel finished.  That is safe as
// long as no load of plan data is scheduled above griddepcontrol.wait, which is what
// pdl_wait_for() guarantees for the pointers it is given.
//
// Reference parity: the reference has no MoE kernels (it defers MoE to vLLM /
// llama.cpp); its expert placement hook is core/expert_pinning.py:115-642.
#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kPlanThreads = 1024;

__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(MoePlanArgs a, uint32_t* __restrict__ err) {
  pdl_launch();
  pdl_wait();
  for (int e = threadIdx.x; e < a.E; e += blockDim.x) a.counts[e] = 0;
  __syncthreads();
  // rank of each pair within its expert (arrival order)
  for (int p = threadIdx.x; p < a.P; p += blockDim.x) {
    int e = (int)a.ids[p];
    if (e < 0 || e >= a.E) {
      report_error(err, kErrBadShape);
      e = 0;
    }
    a.row_of[p] = atomicAdd(&a.counts[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0, nb = 0;
    for (int e = 0; e < a.E; ++e) {
      a.offsets[e] = off;
      const int n = a.counts[e];
      for (int r0 = 0; r0 < n; r0 += a.BN) {
        if (nb < a.max_blocks) a.blocks[nb] = MoeBlock{e, off + r0, min(a.BN, n - r0), 0};
        ++nb;
      }
      off += n;
    }
    a.offsets[a.E] = off;
    if (nb > a.max_blocks) {
      report_error(err, kErrBadShape);
      nb = a.max_blocks;
    }
    *a.num_blocks = nb;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < a.P; p += blockDim.x) {
    int e = (int)a.ids[p];
    if (e < 0 || e >= a.E) e = 0;
    const int row = a.offsets[e] + a.row_of[p];
    a.row_of[p] = row;
    a.tok_of_row[row] = p / a.topk;
  }
}

// one CTA per grouped row, 16-byte copies
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int* __restrict__ tok,
                                  int K, __nv_bfloat16* __restrict__ xp, int64_t ldp) {
  pdl_launch();
  pdl_wait_for(x, tok);
  const int r = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok[r] * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)r * ldp);
  for (int v = threadIdx.x; v < K / 8; v += blockDim.x) dst[v] = src[v];
}

// one CTA per token: fp32 sum of its top-k expert rows in k order (+ add), to bf16
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ yp, int64_t ldp, const int* __restrict__ row_of,
                                   const float* __restrict__ w, int topk, int H,
                                   const __nv_bfloat16* __restrict__ add, __nv_bfloat16* __restrict__ out,
                                   int64_t ldo) {
  pdl_launch();
  pdl_wait_for(yp, row_of, w, add);
  const int t = blockIdx.x;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < topk; ++k) {
      const float wk = w[t * topk + k];
      const uint4 u = *reinterpret_cast<const uint4*>(yp + (size_t)row_of[t * topk + k] * ldp + v * 8);
      const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += wk * bf16_lo(pu[j]);
        acc[2 * j + 1] += wk * bf16_hi(pu[j]);
      }
    }
    if (add) {
      const uint4 u = *reinterpret_cast<const uint4*>(add + (size_t)t * H + v * 8);
      const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] += bf16_lo(pu[j]);
        acc[2 * j + 1] += bf16_hi(pu[j]);
      }
    }
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) po[j] = pack_bf16x2(acc[2 * j], acc[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + (size_t)t * ldo + v * 8) = o;
  }
}

}  // namespace

void moe_plan(const MoePlanArgs& a, cudaStream_t st) {
  VRM_REQUIRE(a.E > 0 && a.E <= 4096 && a.P >= 0 && a.topk > 0 && a.BN > 0, "moe_plan: bad sizes");
  if (a.P == 0) return;
  launch_kernel(moe_plan_kernel, dim3(1), dim3(kPlanThreads), 0, st, a, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_gather(const void* x, int64_t ldx, const int* tok_of_row, int P, int K, void* x_perm, int64_t ld_perm,
                cudaStream_t st) {
  VRM_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ld_perm % 8 == 0, "moe_gather: rows must be 16-byte multiples");
  if (P <= 0) return;
  launch_kernel(moe_gather_kernel, dim3(P), dim3(std::min(256, std::max(32, K / 8))), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(x), ldx, tok_of_row, K,
                reinterpret_cast<__nv_bfloat16*>(x_perm), ld_perm);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_combine(const void* y_perm, int64_t ld_perm, const int* __restrict__ row_of, const float* weights, int T, int topk,
                 int H, const void* add, void* out, int64_t ldo, cudaStream_t st) {
  VRM_REQUIRE(H % 8 == 0 && ld_perm % 8 == 0 && ldo % 8 == 0, "moe_combine: rows must be 16-byte multiples");
  if (T <= 0) return;
  launch_kernel(moe_combine_kernel, dim3(T), dim3(std::min(256, std::max(32, H / 8))), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(y_perm), ld_perm, row_of, weights, topk, H,
                reinterpret_cast<const __nv_bfloat16*>(add), reinterpret_cast<__nv_bfloat16*>(out), ldo);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
