// FP8 (e4m3) W8A8 linear layers: per-row quantisation (weights: one scale per output
// channel; activations: one scale per token, the fused activation quantisation of a
// decode or prefill step) and the GEMM, which is the stream-K tcgen05 kernel of
// gemm_tc.cu instantiated for kind::f8f6f4 with the two scales applied in its epilogue.
//
//   scale[r] = amax(|x[r, :]|) / 448 (1 for an all-zero row)
//   q[r, k]  = e4m3_rn_sat(x[r, k] / scale[r])
//   y[m, n]  = sum_k q_x[m, k] q_w[n, k] * scale_x[m] * scale_w[n]
//
// Reference parity: the reference's 8-bit path is bitsandbytes LLM.int8 / vLLM fp8
// (core/backends.py quantisation switch); this is the Blackwell-native 8-bit format.
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

__device__ __forceinline__ uint16_t f32x2_to_e4m3x2_f8(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// one CTA per row; 8 elements (16 bytes of bf16 -> 8 bytes of e4m3) per thread step
__global__ void __launch_bounds__(256) fp8_rows_quant_kernel(const __nv_bfloat16* x, int64_t ldx, int K, uint8_t* q,
                                                             float* scale) {
  pdl_launch();
  pdl_wait_for(x);
  __shared__ float red[33];
  const int r = blockIdx.x;
  const __nv_bfloat16* xr = x + (size_t)r * ldx;
  const int nv = K / 8;
  float m = 0.f;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + v * 8);
    const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16_lo(pu[j])), fabsf(bf16_hi(pu[j]))));
  }
  m = warp_max(m);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_max(t);
    if (threadIdx.x == 0) red[32] = t;
  }
  __syncthreads();
  const float amax = red[32];
  const float s = amax > 0.f ? amax / 448.f : 1.f;
  if (threadIdx.x == 0) scale[r] = s;
  uint8_t* qr = q + (size_t)r * K;
  for (int v = threadIdx.x; v < nv; v += blockDim.x) {
    const uint4 u = *reinterpret_cast<const uint4*>(xr + v * 8);
    const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
    uint32_t o[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint16_t lo = f32x2_to_e4m3x2_f8(bf16_hi(pu[2 * h]) / s, bf16_lo(pu[2 * h]) / s);
      const uint16_t hi = f32x2_to_e4m3x2_f8(bf16_hi(pu[2 * h + 1]) / s, bf16_lo(pu[2 * h + 1]) / s);
      o[h] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    *reinterpret_cast<uint2*>(qr + v * 8) = make_uint2(o[0], o[1]);
  }
}

}  // namespace

void fp8_rows_quantize(const void* x, int64_t ldx, int rows, int K, uint8_t* q, float* scale, cudaStream_t st) {
  VRM_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              "fp8 rows: K and the row stride must be multiples of 8, rows 16-byte aligned");
  if (rows <= 0) return;
  launch_kernel(fp8_rows_quant_kernel, dim3(rows), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(x), ldx, K,
                q, scale);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
