// Reduce half of the fused tensor-parallel all-reduce, fused with the residual update
// and the norm that follows the row-parallel projection (ARNormArgs in vrm_kernels.h).
//
// The row-parallel GEMM of every rank has pushed its bf16 partial into this rank's
// receive buffer over NVLink and flagged it (gemm_tc.cu, ARPush).  One CTA per token
// row waits for the peers' flags (bounded spin, kErrFlagTimeout on expiry), sums the
// world slots in rank order in fp32 from local HBM, adds bias and the bf16 residual, stores the
// new residual and writes the normalised row for the next GEMM.  So one decode layer at
// TP > 1 launches the same eight kernels as at TP = 1: the all-reduce costs one set of
// posted NVLink stores in the GEMM epilogue and a flag wait here, no extra launch.
//
// Reference parity: the reference all-reduces with torch.cuda.nccl.all_reduce and adds
// the residual in PyTorch (core/tensor_parallel.py:67-80, 393-445); no fused kernel.
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

namespace {

__device__ __forceinline__ float ar_block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

// VPT vectors of 8 features per thread; H <= 8 * blockDim * VPT.
template <int VPT>
__global__ void __launch_bounds__(256) ar_norm_kernel(ARNormArgs a, uint32_t* __restrict__ err) {
  pdl_launch();
  pdl_wait();
  __shared__ float red[33];
  const int row = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(a.epoch);
  if (threadIdx.x == 0) {
    // peers' flags for this rank; signed difference: the epoch wraps after 2^32 calls
    for (int p = 0; p < a.world; ++p) {
      if (p == a.rank) continue;
      const unsigned long long t0 = clock64();
      while ((int)(ld_acquire_sys(a.flags + p) - epoch) < 0) {
        if ((unsigned long long)(clock64() - t0) > VRM_SPIN_LIMIT_CYCLES) {
          report_error(err, kErrFlagTimeout);
          break;
        }
      }
    }
  }
  __syncthreads();
  const int H = a.H, nvec = H >> 3;
  const __nv_bfloat16* half = a.xbuf + (size_t)(epoch & 1u) * a.world * a.half_floats + (size_t)row * H;
  const auto* bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  auto* res = a.residual ? reinterpret_cast<__nv_bfloat16*>(a.residual) + (size_t)row * H : nullptr;
  float vals[VPT][8];
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
    if (v >= nvec) continue;
    for (int p = 0; p < a.world; ++p) {
      const uint4 x = __ldcg(reinterpret_cast<const uint4*>(half + (size_t)p * a.half_floats + v * 8));
      vals[i][0] += bf16_lo(x.x); vals[i][1] += bf16_hi(x.x); vals[i][2] += bf16_lo(x.y); vals[i][3] += bf16_hi(x.y);
      vals[i][4] += bf16_lo(x.z); vals[i][5] += bf16_hi(x.z); vals[i][6] += bf16_lo(x.w); vals[i][7] += bf16_hi(x.w);
    }
    if (bias) {
      const uint4 bb = *reinterpret_cast<const uint4*>(bias + v * 8);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&bb);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vals[i][2 * j] += bf16_lo(pb[j]);
        vals[i][2 * j + 1] += bf16_hi(pb[j]);
      }
    }
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
    if (res) {
      const uint4 rr = *reinterpret_cast<const uint4*>(res + v * 8);
      const uint32_t* pr = reinterpret_cast<const uint32_t*>(&rr);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vals[i][2 * j] += bf16_lo(pr[j]);
        vals[i][2 * j + 1] += bf16_hi(pr[j]);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      po[j] = pack_bf16x2(vals[i][2 * j], vals[i][2 * j + 1]);
      // the residual stream is bf16: normalise the rounded value
      vals[i][2 * j] = bf16_lo(po[j]);
      vals[i][2 * j + 1] = bf16_hi(po[j]);
      s1 += vals[i][2 * j] + vals[i][2 * j + 1];
    }
    if (res) *reinterpret_cast<uint4*>(res + v * 8) = o;
    if (a.mode == kArAdd && a.out && a.out != a.residual)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)row * a.ldo + v * 8) = o;
  }
  if (a.mode == kArAdd) return;
  float mean = 0.f;
  if (a.mode == kArLayerNorm) mean = ar_block_sum(s1, red) / (float)H;
  float s2 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = vals[i][j] - mean;
        s2 += d * d;
      }
    }
  }
  const float inv = rsqrtf(ar_block_sum(s2, red) / (float)H + a.eps);
  const auto* w = reinterpret_cast<const __nv_bfloat16*>(a.w);
  const auto* b = reinterpret_cast<const __nv_bfloat16*>(a.b);
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)row * a.ldo;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v >= nvec) continue;
    const uint4 g = *reinterpret_cast<const uint4*>(w + v * 8);
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
    float bb[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (a.mode == kArLayerNorm) {
      const uint4 q = *reinterpret_cast<const uint4*>(b + v * 8);
      const uint32_t* pq = reinterpret_cast<const uint32_t*>(&q);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        bb[2 * j] = bf16_lo(pq[j]);
        bb[2 * j + 1] = bf16_hi(pq[j]);
      }
    }
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      po[j] = pack_bf16x2((vals[i][2 * j] - mean) * inv * bf16_lo(pg[j]) + bb[2 * j],
                          (vals[i][2 * j + 1] - mean) * inv * bf16_hi(pg[j]) + bb[2 * j + 1]);
    *reinterpret_cast<uint4*>(orow + v * 8) = o;
  }
}

}  // namespace

void ar_norm(const ARNormArgs& a, cudaStream_t st) {
  if (a.T <= 0) return;
  VRM_REQUIRE(a.H % 8 == 0 && a.H <= 8 * 256 * 8, "ar_norm: hidden must be a multiple of 8 and <= 16384");
  VRM_REQUIRE((long long)a.T * a.H <= a.half_floats, "ar_norm: rows larger than the receive buffer");
  VRM_REQUIRE(a.mode == kArAdd || (a.w && a.out), "ar_norm: norm weight and output required");
  VRM_REQUIRE(a.mode != kArLayerNorm || a.b, "ar_norm: layernorm bias required");
  VRM_REQUIRE(a.mode != kArAdd || a.residual || a.out, "ar_norm: nothing to write");
  const int nvec = a.H / 8;
  const int threads = std::min(256, ((nvec + 31) / 32) * 32);
  const int vpt = (nvec + threads - 1) / threads;
  uint32_t* err = error_word();
  if (vpt <= 1) launch_kernel(ar_norm_kernel<1>, dim3(a.T), dim3(threads), 0, st, a, err);
  else if (vpt <= 2) launch_kernel(ar_norm_kernel<2>, dim3(a.T), dim3(threads), 0, st, a, err);
  else if (vpt <= 4) launch_kernel(ar_norm_kernel<4>, dim3(a.T), dim3(threads), 0, st, a, err);
  else launch_kernel(ar_norm_kernel<8>, dim3(a.T), dim3(threads), 0, st, a, err);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
