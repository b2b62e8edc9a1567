// Reduce half of the fused tensor-parallel all-reduce, fused with the residual update
// and the norm that follows the row-parallel projection (ARNormArgs in vrm_kernels.h).
//
// The row-parallel GEMM of every rank has stored its bf16 partial into this rank's
// receive buffer over NVLink (gemm_tc.cu, ARPush) with no fence and no flag.  One CTA
// per token row loads every source rank's slot of the row at once and re-polls the
// vectors that still hold the empty pattern (bounded: kErrFlagTimeout on expiry, the
// missing values count as 0), sums the world slots in rank order in fp32 (bitwise the
// same on every rank), adds bias and the bf16 residual, stores the new residual and
// writes the normalised row for the next GEMM.  It then empties the slots it read (the
// same half is written again two calls later, only after this kernel has finished on
// this rank), and the last CTA advances the epoch that selects the half.
//
// So the all-reduce costs one set of posted NVLink stores in the GEMM epilogue and one
// NVLink write latency here; a decode layer at TP > 1 launches as many kernels as at
// TP = 1 with unfolded norms.
//
// Reference parity: the reference all-reduces with torch.cuda.nccl.all_reduce and adds
// the residual in PyTorch (core/tensor_parallel.py:67-80, 393-445); no fused kernel.
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

namespace {

constexpr int kArMaxWorld = 8;

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

__device__ __forceinline__ void add_bf16x8(float (&acc)[8], const uint4& x) {
  acc[0] += bf16_lo(x.x); acc[1] += bf16_hi(x.x); acc[2] += bf16_lo(x.y); acc[3] += bf16_hi(x.y);
  acc[4] += bf16_lo(x.z); acc[5] += bf16_hi(x.z); acc[6] += bf16_lo(x.w); acc[7] += bf16_hi(x.w);
}

// empty lanes of a vector read after the wait gave up count as 0
__device__ __forceinline__ uint4 zero_empty(uint4 x) {
  auto z = [](uint32_t w) {
    if ((w & 0xffffu) == kBf16Empty) w &= 0xffff0000u;
    if ((w >> 16) == kBf16Empty) w &= 0x0000ffffu;
    return w;
  };
  return make_uint4(z(x.x), z(x.y), z(x.z), z(x.w));
}

// VPT vectors of 8 features per thread; H <= 8 * blockDim * VPT.  WORLD source ranks.
// At most ar_threads(VPT) threads, so that every slot of the thread's vectors stays in
// registers (no spills up to VPT 2 at WORLD 8).
constexpr int ar_threads(int vpt) { return vpt == 1 ? 768 : 512; }

template <int VPT, int WORLD>
__global__ void __launch_bounds__(ar_threads(VPT)) ar_norm_kernel(ARNormArgs a, uint32_t* __restrict__ err) {
  pdl_launch();
  pdl_wait();
  __shared__ float red[33];
  const int row = blockIdx.x;
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(a.epoch);
  const int H = a.H, nvec = H >> 3;
  __nv_bfloat16* half = a.xbuf + (size_t)(epoch & 1u) * WORLD * a.half_floats + (size_t)row * H;
  const auto* bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  auto* res = a.residual ? reinterpret_cast<__nv_bfloat16*>(a.residual) + (size_t)row * H : nullptr;
  const unsigned long long limit = a.spin_limit ? a.spin_limit : VRM_SPIN_LIMIT_CYCLES;

  // every slot of every vector of this thread in flight at once, then re-poll the
  // vectors that have not fully arrived
  uint4 x[VPT][WORLD];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int p = 0; p < WORLD; ++p)
      x[i][p] = v < nvec ? ld_relaxed_sys_v4(half + (size_t)p * a.half_floats + v * 8) : make_uint4(0, 0, 0, 0);
  }
  bool timed_out = false;
  const unsigned long long t0 = clock64();
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v >= nvec) continue;
#pragma unroll
    for (int p = 0; p < WORLD; ++p) {
      while (bf16x8_has_empty(x[i][p])) {
        if (timed_out || (unsigned long long)(clock64() - t0) > limit) {
          if (!timed_out) report_error(err, kErrFlagTimeout);
          timed_out = true;
          x[i][p] = zero_empty(x[i][p]);
          break;
        }
        x[i][p] = ld_relaxed_sys_v4(half + (size_t)p * a.half_floats + v * 8);
      }
    }
  }

  float vals[VPT][8];
  float s1 = 0.f;
  const uint4 empty = make_uint4(kBf16EmptyX2, kBf16EmptyX2, kBf16EmptyX2, kBf16EmptyX2);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
#pragma unroll
    for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
    if (v >= nvec) continue;
#pragma unroll
    for (int p = 0; p < WORLD; ++p) {
      add_bf16x8(vals[i], x[i][p]);
      // the slot is empty again for the call two epochs on
      *reinterpret_cast<uint4*>(half + (size_t)p * a.half_floats + v * 8) = empty;
    }
    if (bias) {
      const uint4 bb = *reinterpret_cast<const uint4*>(bias + v * 8);
      add_bf16x8(vals[i], bb);
    }
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
    if (res) {
      const uint4 rr = *reinterpret_cast<const uint4*>(res + v * 8);
      add_bf16x8(vals[i], rr);
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

  if (a.mode != kArAdd) {
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

  // the last CTA to finish advances the epoch (read by the next push GEMM, which runs
  // at least one kernel later in stream order)
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.done) : "memory");
    if (prev == gridDim.x - 1) {
      *a.done = 0u;
      *reinterpret_cast<volatile uint32_t*>(a.epoch) = epoch + 1u;
    }
  }
}

template <int VPT>
void launch_ar(const ARNormArgs& a, int threads, cudaStream_t st, uint32_t* err) {
  switch (a.world) {
    case 1: launch_kernel(ar_norm_kernel<VPT, 1>, dim3(a.T), dim3(threads), 0, st, a, err); break;
    case 2: launch_kernel(ar_norm_kernel<VPT, 2>, dim3(a.T), dim3(threads), 0, st, a, err); break;
    case 4: launch_kernel(ar_norm_kernel<VPT, 4>, dim3(a.T), dim3(threads), 0, st, a, err); break;
    case 8: launch_kernel(ar_norm_kernel<VPT, 8>, dim3(a.T), dim3(threads), 0, st, a, err); break;
    default: VRM_REQUIRE(false, "ar_norm: world must be 1, 2, 4 or 8");
  }
}

}  // namespace

void ar_norm(const ARNormArgs& a, cudaStream_t st) {
  if (a.T <= 0) return;
  VRM_REQUIRE(a.world >= 1 && a.world <= kArMaxWorld, "ar_norm: world must be 1..8");
  VRM_REQUIRE(a.H % 8 == 0 && a.H <= 8 * 1024 * 2, "ar_norm: hidden must be a multiple of 8 and <= 16384");
  VRM_REQUIRE((long long)a.T * a.H <= a.half_floats, "ar_norm: rows larger than the receive buffer");
  VRM_REQUIRE(a.mode == kArAdd || (a.w && a.out), "ar_norm: norm weight and output required");
  VRM_REQUIRE(a.mode != kArLayerNorm || a.b, "ar_norm: layernorm bias required");
  VRM_REQUIRE(a.mode != kArAdd || a.residual || a.out, "ar_norm: nothing to write");
  VRM_REQUIRE(a.xbuf && a.epoch && a.done, "ar_norm: receive buffer, epoch and done counter required");
  const int nvec = a.H / 8;
  // every load of the row in flight at once: one vector per thread while that fits
  const int vpt = nvec <= ar_threads(1) ? 1 : nvec <= 2 * ar_threads(2) ? 2 : 4;
  const int threads = ((nvec + vpt - 1) / vpt + 31) / 32 * 32;
  uint32_t* err = a.err ? a.err : error_word();
  if (vpt == 1) launch_ar<1>(a, threads, st, err);
  else if (vpt == 2) launch_ar<2>(a, threads, st, err);
  else launch_ar<4>(a, threads, st, err);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
