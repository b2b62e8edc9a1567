// Normalisation, rotary embedding + paged-KV write, activations, embedding lookup.
//
// Reference parity:
//   fused residual+RMSNorm     core/triton_fused_rmsnorm.py:20-56 (Triton, no residual)
//   RoPE (rotate-half)         core/triton_fused_rope.py:24-57
//   paged KV write             core/paged_attention.py:568-621 (write_kv, Python)
//   KV fp8 e4m3 quantisation   (reference: only through vLLM kv_cache_dtype="fp8")
// RoPE, the KV page write and the fp8 quantisation are one kernel that runs straight
// after the QKV projection, so K/V never make a separate round trip.
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

// ---------------------------------------------------------------- RMSNorm / LayerNorm
__device__ __forceinline__ float block_reduce_sum(float v, float* red) {
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

// Loads VPT vectors of 8 bf16 of x (+ residual, stored back rounded to bf16).
template <int VPT>
__device__ __forceinline__ void load_row(const __nv_bfloat16* xr, __nv_bfloat16* rr, int nvec, float (&vals)[VPT][8]) {
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 a = *reinterpret_cast<const uint4*>(xr + v * 8);
      const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        vals[i][2 * j] = bf16_lo(pa[j]);
        vals[i][2 * j + 1] = bf16_hi(pa[j]);
      }
      if (rr) {
        uint4 b = *reinterpret_cast<const uint4*>(rr + v * 8);
        const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
        uint4 s;
        uint32_t* ps = reinterpret_cast<uint32_t*>(&s);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          ps[j] = pack_bf16x2(vals[i][2 * j] + bf16_lo(pb[j]), vals[i][2 * j + 1] + bf16_hi(pb[j]));
          // the residual stream is kept in bf16: normalise the rounded value
          vals[i][2 * j] = bf16_lo(ps[j]);
          vals[i][2 * j + 1] = bf16_hi(ps[j]);
        }
        *reinterpret_cast<uint4*>(rr + v * 8) = s;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) vals[i][j] = 0.f;
    }
  }
}

template <int VPT>
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                               const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ out, int H, int64_t ldx,
                               int64_t ldo, float eps) {
  pdl_launch();
  pdl_wait_for(x, w);
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  float vals[VPT][8];
  load_row<VPT>(x + (size_t)row * ldx, residual ? residual + (size_t)row * H : nullptr, nvec, vals);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) ss += vals[i][j] * vals[i][j];
  const float inv = rsqrtf(block_reduce_sum(ss, red) / (float)H + eps);
  __nv_bfloat16* orow = out + (size_t)row * ldo;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 g = *reinterpret_cast<const uint4*>(w + v * 8);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        po[j] = pack_bf16x2(vals[i][2 * j] * inv * bf16_lo(pg[j]), vals[i][2 * j + 1] * inv * bf16_hi(pg[j]));
      *reinterpret_cast<uint4*>(orow + v * 8) = o;
    }
  }
}

template <int VPT>
__global__ void layernorm_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ residual,
                                 const __nv_bfloat16* __restrict__ w, const __nv_bfloat16* __restrict__ b,
                                 __nv_bfloat16* __restrict__ out, int H, int64_t ldx, int64_t ldo, float eps) {
  pdl_launch();
  pdl_wait_for(x, w, b);
  __shared__ float red[33];
  const int row = blockIdx.x;
  const int nvec = H / 8;
  float vals[VPT][8];
  load_row<VPT>(x + (size_t)row * ldx, residual ? residual + (size_t)row * H : nullptr, nvec, vals);
  float s1 = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) s1 += vals[i][j];
  const float mean = block_reduce_sum(s1, red) / (float)H;
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
  const float inv = rsqrtf(block_reduce_sum(s2, red) / (float)H + eps);
  __nv_bfloat16* orow = out + (size_t)row * ldo;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < nvec) {
      uint4 g = *reinterpret_cast<const uint4*>(w + v * 8);
      uint4 bb = *reinterpret_cast<const uint4*>(b + v * 8);
      const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&bb);
      uint4 o;
      uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        po[j] = pack_bf16x2((vals[i][2 * j] - mean) * inv * bf16_lo(pg[j]) + bf16_lo(pb[j]),
                            (vals[i][2 * j + 1] - mean) * inv * bf16_hi(pg[j]) + bf16_hi(pb[j]));
      *reinterpret_cast<uint4*>(orow + v * 8) = o;
    }
  }
}

static void norm_shape(int H, int* threads, int* vpt) {
  VRM_REQUIRE(H % 8 == 0 && H <= 8 * 256 * 8, "norm: hidden must be a multiple of 8 and <= 16384");
  const int nvec = H / 8;
  *threads = std::min(256, ((nvec + 31) / 32) * 32);
  *vpt = (nvec + *threads - 1) / *threads;
}

void rmsnorm(const void* x, int64_t ldx, void* residual, const void* w, void* out, int64_t ldo, int T, int H,
             float eps, cudaStream_t st) {
  if (T <= 0) return;
  int threads, vpt;
  norm_shape(H, &threads, &vpt);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x);
  auto rp = reinterpret_cast<__nv_bfloat16*>(residual);
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w);
  auto op = reinterpret_cast<__nv_bfloat16*>(out);
  if (vpt <= 1) launch_kernel(rmsnorm_kernel<1>, dim3(T), dim3(threads), 0, st, xp, rp, wp, op, H, ldx, ldo, eps);
  else if (vpt <= 2) launch_kernel(rmsnorm_kernel<2>, dim3(T), dim3(threads), 0, st, xp, rp, wp, op, H, ldx, ldo, eps);
  else if (vpt <= 4) launch_kernel(rmsnorm_kernel<4>, dim3(T), dim3(threads), 0, st, xp, rp, wp, op, H, ldx, ldo, eps);
  else launch_kernel(rmsnorm_kernel<8>, dim3(T), dim3(threads), 0, st, xp, rp, wp, op, H, ldx, ldo, eps);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void layernorm(const void* x, int64_t ldx, void* residual, const void* w, const void* b, void* out, int64_t ldo,
               int T, int H, float eps, cudaStream_t st) {
  if (T <= 0) return;
  int threads, vpt;
  norm_shape(H, &threads, &vpt);
  auto xp = reinterpret_cast<const __nv_bfloat16*>(x);
  auto rp = reinterpret_cast<__nv_bfloat16*>(residual);
  auto wp = reinterpret_cast<const __nv_bfloat16*>(w);
  auto bp = reinterpret_cast<const __nv_bfloat16*>(b);
  auto op = reinterpret_cast<__nv_bfloat16*>(out);
  if (vpt <= 1) launch_kernel(layernorm_kernel<1>, dim3(T), dim3(threads), 0, st, xp, rp, wp, bp, op, H, ldx, ldo, eps);
  else if (vpt <= 2) launch_kernel(layernorm_kernel<2>, dim3(T), dim3(threads), 0, st, xp, rp, wp, bp, op, H, ldx, ldo, eps);
  else if (vpt <= 4) launch_kernel(layernorm_kernel<4>, dim3(T), dim3(threads), 0, st, xp, rp, wp, bp, op, H, ldx, ldo, eps);
  else launch_kernel(layernorm_kernel<8>, dim3(T), dim3(threads), 0, st, xp, rp, wp, bp, op, H, ldx, ldo, eps);
  VRM_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- RoPE + KV write
// qkv: [T, (Hq + 2*KH) * D] (q heads, then k heads, then v heads), rotated in place.
// K and V rows are stored into the paged cache
//   cache[page, layer, {0:k,1:v}, kv_head, slot_in_page, d]
// as bf16, as fp8 e4m3 of value / scale[layer, k|v, kv_head] (saturating), or as a
// four-bit row (per 32 dims: scale = (max - min) / 15 and min in fp16, codes
// round((x - min) / scale) in 0..15; D = 64 or 128).
// cos_sin: [max_pos, rot_dim] fp32 = [cos(0..rot/2) | sin(0..rot/2)]; rotate-half form
// (GPT-NeoX / Llama / Qwen2) over the first rot_dim dims.  rot_dim == 0: no rotation.
template <int FMT>
__global__ void rope_kv_write_kernel(RopeKvArgs a) {
  pdl_launch();
  pdl_wait();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  const int D = a.D;
  const int p = a.positions ? a.positions[t] : 0;
  const int slot = a.slot_mapping ? a.slot_mapping[t] : -1;
  __nv_bfloat16* row = reinterpret_cast<__nv_bfloat16*>(a.qkv) + (size_t)t * a.ld_qkv;
  const int half = a.rot_dim / 2;
  const float* cs = a.cos_sin ? a.cos_sin + (size_t)p * a.rot_dim : nullptr;
  for (int h = warp; h < a.Hq + 2 * a.KH; h += nwarps) {
    __nv_bfloat16* hv = row + (size_t)h * D;
    const bool is_v = h >= a.Hq + a.KH;
    if (!is_v && cs != nullptr && half > 0) {
      for (int i = lane; i < half; i += 32) {
        const float c = cs[i], s = cs[half + i];
        float o1, o2;
        rope_rotate(__bfloat162float(hv[i]), __bfloat162float(hv[i + half]), c, s, o1, o2);
        hv[i] = __float2bfloat16(o1);
        hv[i + half] = __float2bfloat16(o2);
      }
      __syncwarp();
    }
    if (h >= a.Hq && slot >= 0 && in_bounds(slot / a.page_size, a.num_pages, a.err)) {
      const int kvh = is_v ? h - a.Hq - a.KH : h - a.Hq;
      const int kv = is_v ? 1 : 0;
      const int page = slot / a.page_size, off = slot % a.page_size;
      if constexpr (FMT == kFmtQ4) {
        const size_t rb = (size_t)D / 2 + D / 8;
        uint8_t* dst = reinterpret_cast<uint8_t*>(a.cache) +
                       ((((size_t)page * a.num_layers + a.layer) * 2 + kv) * a.KH + kvh) * (size_t)a.page_size * rb +
                       (size_t)off * rb;
        if (D == 128) {
          float x[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) x[j] = __bfloat162float(hv[lane * 4 + j]);
          q4_store_row<128>(dst, x, lane);
        } else {
          float x[2];
#pragma unroll
          for (int j = 0; j < 2; ++j) x[j] = __bfloat162float(hv[lane * 2 + j]);
          q4_store_row<64>(dst, x, lane);
        }
        continue;
      }
      const size_t base =
          ((((size_t)page * a.num_layers + a.layer) * 2 + kv) * a.KH + kvh) * (size_t)a.page_size * D + (size_t)off * D;
      if (FMT == kFmtFp8) {
        const float inv = 1.f / a.kv_scale[(a.layer * 2 + kv) * a.KH + kvh];
        uint8_t* c8 = reinterpret_cast<uint8_t*>(a.cache) + base;
        for (int d = lane; d < D; d += 32) {
          const __nv_fp8_storage_t q = __nv_cvt_float_to_fp8(__bfloat162float(hv[d]) * inv, __NV_SATFINITE, __NV_E4M3);
          c8[d] = q;
        }
      } else {
        __nv_bfloat16* cb = reinterpret_cast<__nv_bfloat16*>(a.cache) + base;
        for (int d = lane; d < D; d += 32) cb[d] = hv[d];
      }
    }
  }
}

void rope_kv_write(const RopeKvArgs& a_in, cudaStream_t st) {
  if (a_in.T <= 0) return;
  RopeKvArgs a = a_in;
  a.err = error_word();
  VRM_REQUIRE(!a.cache_fp8 || a.kv_scale != nullptr, "rope_kv_write: fp8 cache needs kv_scale");
  VRM_REQUIRE(!a.cache_q4 || a.D == 64 || a.D == 128, "rope_kv_write: four-bit pages need head_dim 64 or 128");
  const int threads = 32 * std::min(16, a.Hq + 2 * a.KH);
  if (a.cache_q4) launch_kernel(rope_kv_write_kernel<kFmtQ4>, dim3(a.T), dim3(threads), 0, st, a);
  else if (a.cache_fp8) launch_kernel(rope_kv_write_kernel<kFmtFp8>, dim3(a.T), dim3(threads), 0, st, a);
  else launch_kernel(rope_kv_write_kernel<kFmtBf16>, dim3(a.T), dim3(threads), 0, st, a);
  VRM_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- per-head q / k RMSNorm
// Qwen3's q_norm / k_norm: every q head and k head row of qkv [T, (Hq + 2 KH) * D] is
// normalised in place, x[d] = x[d] * rsqrt(mean(x^2) + eps) * w[d] (fp32 math, one bf16
// rounding), w = wq [D] for q heads and wk [D] for k heads; v heads are untouched.  One
// warp per head row, lane j holding dims j, j + 32, ... (coalesced); runs between the
// QKV projection and RoPE.
template <int kPer>
__global__ void qk_rmsnorm_kernel(__nv_bfloat16* __restrict__ qkv, int64_t ld, const __nv_bfloat16* __restrict__ wq,
                                  const __nv_bfloat16* __restrict__ wk, int Hq, int KH, float eps) {
  pdl_launch();
  pdl_wait_for(qkv, wq, wk);
  constexpr int D = kPer * 32;
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nwarps = blockDim.x >> 5;
  for (int h = warp; h < Hq + KH; h += nwarps) {
    __nv_bfloat16* row = qkv + (size_t)t * ld + (size_t)h * D;
    const __nv_bfloat16* w = h < Hq ? wq : wk;
    float v[kPer];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      v[j] = __bfloat162float(row[lane + 32 * j]);
      ss += v[j] * v[j];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss * (1.f / D) + eps);
#pragma unroll
    for (int j = 0; j < kPer; ++j) row[lane + 32 * j] = __float2bfloat16(v[j] * r * __bfloat162float(w[lane + 32 * j]));
  }
}

void qk_rmsnorm(void* qkv, int64_t ld, const void* wq, const void* wk, int T, int Hq, int KH, int D, float eps,
                cudaStream_t st) {
  if (T <= 0) return;
  VRM_REQUIRE(D == 64 || D == 128 || D == 256, "qk_rmsnorm: head_dim must be 64, 128 or 256");
  auto q = static_cast<__nv_bfloat16*>(qkv);
  auto a = static_cast<const __nv_bfloat16*>(wq);
  auto b = static_cast<const __nv_bfloat16*>(wk);
  const int threads = 32 * std::min(16, Hq + KH);
  if (D == 64) launch_kernel(qk_rmsnorm_kernel<2>, dim3(T), dim3(threads), 0, st, q, ld, a, b, Hq, KH, eps);
  else if (D == 128) launch_kernel(qk_rmsnorm_kernel<4>, dim3(T), dim3(threads), 0, st, q, ld, a, b, Hq, KH, eps);
  else launch_kernel(qk_rmsnorm_kernel<8>, dim3(T), dim3(threads), 0, st, q, ld, a, b, Hq, KH, eps);
  VRM_CUDA_CHECK(cudaGetLastError());
}

// ---------------------------------------------------------------- activations
// out[t, i] = silu(x[t, i]) * x[t, I + i]   (gate | up concatenated)
__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ x, __nv_bfloat16* __restrict__ out, int I,
                                int64_t ldx, int64_t ldo) {
  pdl_launch();
  pdl_wait_for(x);
  const int t = blockIdx.y;
  const int v = blockIdx.x * blockDim.x + threadIdx.x;   // vector of 8
  if (v * 8 >= I) return;
  const __nv_bfloat16* g = x + (size_t)t * ldx + v * 8;
  uint4 a = *reinterpret_cast<const uint4*>(g);
  uint4 b = *reinterpret_cast<const uint4*>(g + I);
  const uint32_t* pa = reinterpret_cast<const uint32_t*>(&a);
  const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
  uint4 o;
  uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float g0 = bf16_lo(pa[j]), g1 = bf16_hi(pa[j]);
    const float s0 = g0 / (1.f + __expf(-g0)), s1 = g1 / (1.f + __expf(-g1));
    po[j] = pack_bf16x2(s0 * bf16_lo(pb[j]), s1 * bf16_hi(pb[j]));
  }
  *reinterpret_cast<uint4*>(out + (size_t)t * ldo + v * 8) = o;
}

void silu_mul(const void* x, int64_t ldx, void* out, int64_t ldo, int T, int I, cudaStream_t st) {
  if (T <= 0) return;
  VRM_REQUIRE(I % 8 == 0 && ldx % 8 == 0 && ldo % 8 == 0, "silu_mul: sizes must be multiples of 8");
  dim3 grid((I / 8 + 127) / 128, T);
  launch_kernel(silu_mul_kernel, grid, dim3(128), 0, st, reinterpret_cast<const __nv_bfloat16*>(x),
                reinterpret_cast<__nv_bfloat16*>(out), I, ldx, ldo);
  VRM_CUDA_CHECK(cudaGetLastError());
}

// GELU, tanh approximation (GPT-2 "gelu_new"), in place.
__global__ void gelu_tanh_kernel(__nv_bfloat16* __restrict__ x, size_t n) {
  pdl_launch();
  pdl_wait();
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = __bfloat162float(x[i]);
  const float u = 0.7978845608028654f * (v + 0.044715f * v * v * v);
  x[i] = __float2bfloat16(0.5f * v * (1.f + tanhf(u)));
}

void gelu_tanh(void* x, size_t n, cudaStream_t st) {
  if (n == 0) return;
  launch_kernel(gelu_tanh_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st,
                reinterpret_cast<__nv_bfloat16*>(x), n);
  VRM_CUDA_CHECK(cudaGetLastError());
}

// out[t] = table[ids[t]] (+ pos_table[pos[t]])
__global__ void embedding_kernel(const int* __restrict__ ids, const __nv_bfloat16* __restrict__ table,
                                 const int* __restrict__ pos, const __nv_bfloat16* __restrict__ pos_table,
                                 __nv_bfloat16* __restrict__ out, int H) {
  pdl_launch();
  pdl_wait_for(ids, table, pos, pos_table);
  const int t = blockIdx.x;
  const __nv_bfloat16* src = table + (size_t)ids[t] * H;
  const __nv_bfloat16* psrc = pos_table ? pos_table + (size_t)pos[t] * H : nullptr;
  for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
    uint4 a = *reinterpret_cast<const uint4*>(src + v * 8);
    if (psrc) {
      uint4 b = *reinterpret_cast<const uint4*>(psrc + v * 8);
      uint32_t* pa = reinterpret_cast<uint32_t*>(&a);
      const uint32_t* pb = reinterpret_cast<const uint32_t*>(&b);
#pragma unroll
      for (int j = 0; j < 4; ++j) pa[j] = pack_bf16x2(bf16_lo(pa[j]) + bf16_lo(pb[j]), bf16_hi(pa[j]) + bf16_hi(pb[j]));
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * H + v * 8) = a;
  }
}

void embedding(const int* ids, const void* table, const int* pos, const void* pos_table, void* out, int T, int H,
               cudaStream_t st) {
  if (T <= 0) return;
  VRM_REQUIRE(H % 8 == 0, "embedding: hidden must be a multiple of 8");
  launch_kernel(embedding_kernel, dim3(T), dim3(128), 0, st, ids, reinterpret_cast<const __nv_bfloat16*>(table), pos,
                reinterpret_cast<const __nv_bfloat16*>(pos_table), reinterpret_cast<__nv_bfloat16*>(out), H);
  VRM_CUDA_CHECK(cudaGetLastError());
}

__global__ void add_inplace_kernel(__nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ b, size_t n) {
  pdl_launch();
  pdl_wait_for(b);
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[i] = __float2bfloat16(__bfloat162float(a[i]) + __bfloat162float(b[i]));
}

void add_inplace(void* a, const void* b, size_t n, cudaStream_t st) {
  if (n == 0) return;
  launch_kernel(add_inplace_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, st,
                reinterpret_cast<__nv_bfloat16*>(a), reinterpret_cast<const __nv_bfloat16*>(b), n);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
