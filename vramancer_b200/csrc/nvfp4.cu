// NVFP4 weights: e2m1 values, one e4m3 scale per 16 consecutive K elements of a row,
// one fp32 scale per tensor.  Quantisation, dequantisation, and the W4A16 decode GEMM.
//
// Convention (fixed, tested against a CPU restatement):
//   gs      = amax(|W|) / (6 * 448)                      (per tensor, fp32, on device)
//   s[n,b]  = e4m3_rn_sat(amax(|W[n, 16b:16b+16]|) / 6 / gs)
//   q[n,k]  = e2m1_rn_sat(W[n,k] / (float(s[n,k/16]) * gs))
//   W'[n,k] = float(q) * float(s) * gs
// float(q) * float(s) is exact in f16 (|value| <= 6 * 448, at most 5 significant
// bits), so the GEMM dequantises with the hardware e2m1 -> f16 conversion and one f16
// multiply and applies gs to the fp32 accumulator.
//
// Storage ("fragment order"), chosen so that one 16-byte load per lane is that lane's
// A fragments of mma.m16n8k16 for four k16 steps:
//   q: [N/16 strips][K/64 tiles][32 lanes][16 B]; lane l, byte 4*j + i (k-step j) holds
//      i = 0: rows r, cols c, c+1   i = 1: rows r+8, cols c, c+1
//      i = 2: rows r, cols c+8, c+9 i = 3: rows r+8, cols c+8, c+9
//      with r = l / 4, c = 16 j + 2 (l % 4); the even column in the low nibble.
//   s: [N/16][K/64][8 row groups r][4 k-steps][2 B]: (s[r, block], s[r+8, block]).
// Reference parity: core/nvfp4_direct.py (DirectFP4Linear: w_qdata [N, K/2] with the
// low nibble = even k, e4m3 block scales in cuBLAS's blocked layout, fp32 per-tensor
// scale) and csrc/fp4_gemv.cu:36-116 (M = 1 GEMV, warp per row, LUT dequant).  The
// layout here is different on purpose (tensor-core fragments, any M <= 32).
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kNvThreads = 256;   // 8 warps, one 16-row strip each: 128 rows per CTA
constexpr int kNvRows = 128;
constexpr int kSld = 132;          // fp32 accumulator tile row stride (conflict-free stores)

__device__ __forceinline__ uint16_t f32x2_to_e4m3x2(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
__device__ __forceinline__ float e4m3_to_f32(uint8_t v) {
  const uint32_t h = e4m3x2_to_f16x2(v);
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}
// 8 floats -> 8 e2m1 nibbles; element 2i in the low nibble of byte i.
__device__ __forceinline__ uint32_t f32x8_to_e2m1x8(const float (&v)[8]) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]));
  return r;
}
// byte i of w (two e2m1, low nibble first) -> f16x2 h[i] (low nibble in the low half)
__device__ __forceinline__ void e2m1x8_to_f16x8(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}
__device__ __forceinline__ uint32_t hmul2_u32(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t f32x2_to_f16x2_sat(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t& r0, uint32_t& r1) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}
__device__ __forceinline__ uint4 ld_stream_u4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint2 ld_stream_u2(const uint2* p) {
  uint2 v;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// (strip, tile, lane, byte 4j+i) -> the two (row, col) it holds
__device__ __forceinline__ void frag_coords(int strip, int tile, int lane, int j, int i, int* row, int* col) {
  *row = strip * 16 + (lane >> 2) + ((i & 1) ? 8 : 0);
  *col = tile * 64 + j * 16 + (lane & 3) * 2 + ((i & 2) ? 8 : 0);
}

// ---------------------------------------------------------------- quantisation
// one thread per (row, 16-block): row-major e4m3 block scales
__global__ void nvfp4_block_scales_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int N, int K,
                                          const float* __restrict__ gsp, uint8_t* __restrict__ sc) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int nb = K / 16;
  if (idx >= (int64_t)N * nb) return;
  const int n = (int)(idx / nb), b = (int)(idx % nb);
  const uint4* p = reinterpret_cast<const uint4*>(w + (size_t)n * ldw + b * 16);
  float m = 0.f;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const uint4 v = p[h];
    const uint32_t* pv = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16_lo(pv[j])), fabsf(bf16_hi(pv[j]))));
  }
  const float gs = *gsp;
  sc[idx] = (uint8_t)(f32x2_to_e4m3x2(0.f, m / 6.f / gs) & 0xFFu);
}

// one thread per (strip, tile, lane): 32 e2m1 values (16 B) + the lane group's scales
__global__ void nvfp4_pack_kernel(const __nv_bfloat16* __restrict__ w, int64_t ldw, int N, int K,
                                  const float* __restrict__ gsp, const uint8_t* __restrict__ sc,
                                  uint8_t* __restrict__ q, uint8_t* __restrict__ s) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int tiles = K / 64;
  if (idx >= (int64_t)(N / 16) * tiles * 32) return;
  const int lane = (int)(idx & 31);
  const int64_t st = idx >> 5;
  const int strip = (int)(st / tiles), tile = (int)(st % tiles);
  const float gs = *gsp;
  const int nb = K / 16;
  uint32_t out[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float v[8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int row, col;
      frag_coords(strip, tile, lane, j, i, &row, &col);
      const float sf = e4m3_to_f32(sc[(size_t)row * nb + col / 16]);
      const float denom = sf * gs;
      const uint32_t pr = *reinterpret_cast<const uint32_t*>(w + (size_t)row * ldw + col);
      v[2 * i] = denom > 0.f ? bf16_lo(pr) / denom : 0.f;
      v[2 * i + 1] = denom > 0.f ? bf16_hi(pr) / denom : 0.f;
    }
    out[j] = f32x8_to_e2m1x8(v);
  }
  reinterpret_cast<uint4*>(q)[idx] = make_uint4(out[0], out[1], out[2], out[3]);
  if ((lane & 3) == 0) {
    const int r = lane >> 2;
    uint8_t b[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int blk = tile * 4 + j;
      b[2 * j] = sc[(size_t)(strip * 16 + r) * nb + blk];
      b[2 * j + 1] = sc[(size_t)(strip * 16 + r + 8) * nb + blk];
    }
    uint2 o;
    o.x = b[0] | (b[1] << 8) | (b[2] << 16) | ((uint32_t)b[3] << 24);
    o.y = b[4] | (b[5] << 8) | (b[6] << 16) | ((uint32_t)b[7] << 24);
    reinterpret_cast<uint2*>(s)[st * 8 + r] = o;
  }
}

// ---------------------------------------------------------------- dequantisation
// one warp per (strip, tile): decode in registers, transpose through shared memory,
// store 16 rows x 64 bf16 with 128-byte row segments.
__global__ void __launch_bounds__(256) nvfp4_dequant_kernel(const uint8_t* __restrict__ q,
                                                            const uint8_t* __restrict__ s,
                                                            const float* __restrict__ gsp, int N, int K,
                                                            __nv_bfloat16* __restrict__ out) {
  __shared__ __align__(16) __nv_bfloat16 tile_s[8][16][64 + 8];
  pdl_launch();
  pdl_wait_for(q, s, gsp);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles = K / 64;
  const int64_t st = (int64_t)blockIdx.x * 8 + warp;
  if (st >= (int64_t)(N / 16) * tiles) return;
  const int strip = (int)(st / tiles), tile = (int)(st % tiles);
  const float gs = *gsp;
  const uint4 qv = reinterpret_cast<const uint4*>(q)[st * 32 + lane];
  const uint2 sv = reinterpret_cast<const uint2*>(s)[st * 8 + (lane >> 2)];
  const uint32_t qw[4] = {qv.x, qv.y, qv.z, qv.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint16_t s2 = (uint16_t)(((j < 2 ? sv.x : sv.y) >> ((j & 1) * 16)) & 0xFFFFu);
    const uint32_t sf = e4m3x2_to_f16x2(s2);
    const float s_r = __half2float(__ushort_as_half((unsigned short)(sf & 0xFFFFu)));
    const float s_r8 = __half2float(__ushort_as_half((unsigned short)(sf >> 16)));
    uint32_t h[4];
    e2m1x8_to_f16x8(qw[j], h);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float sc = ((i & 1) ? s_r8 : s_r) * gs;
      const float lo = __half2float(__ushort_as_half((unsigned short)(h[i] & 0xFFFFu))) * sc;
      const float hi = __half2float(__ushort_as_half((unsigned short)(h[i] >> 16))) * sc;
      const int r = (lane >> 2) + ((i & 1) ? 8 : 0);
      const int c = j * 16 + (lane & 3) * 2 + ((i & 2) ? 8 : 0);
      *reinterpret_cast<uint32_t*>(&tile_s[warp][r][c]) = pack_bf16x2(lo, hi);
    }
  }
  __syncwarp();
  // 16 rows x 128 B: lane covers 8 bytes of two rows per step
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 4 + (lane >> 3), c = (lane & 7) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(&tile_s[warp][r][c]);
    *reinterpret_cast<uint4*>(out + (size_t)(strip * 16 + r) * K + tile * 64 + c) = v;
  }
}

// ---------------------------------------------------------------- W4A16 GEMM (decode)
// grid (N/128 row blocks, splits); 8 warps, warp w owns rows [16w, 16w+16) of the block
// over the split's K range.  NT n8 tiles of tokens (M <= 8 NT).  The CTA stages its K
// range of X as f16 (saturating) in shared memory; weights stream from HBM into
// registers four tiles (4 x 64 K) at a time, double buffered, the first group issued
// before the programmatic-launch wait.  Splits > 1: fp32 partials to the workspace,
// the last CTA of a row block reduces them in split order (deterministic).
template <int NT>
__global__ void __launch_bounds__(kNvThreads, 2)
    nvfp4_gemm_kernel(Nvfp4GemmArgs a, int kc, int splits, float* __restrict__ ws,
                      uint32_t* __restrict__ counters) {
  extern __shared__ __align__(16) uint8_t smem[];
  constexpr int MT = NT * 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rb = blockIdx.x, sp = blockIdx.y;
  const int kbeg = sp * kc, kend = min(a.K, kbeg + kc);
  const int tiles = (kend - kbeg) >> 6;
  const int ktiles = a.K >> 6;
  const int strip = rb * 8 + warp;
  const bool active = strip < (a.N >> 4);
  const size_t tile0 = (size_t)strip * ktiles + (kbeg >> 6);
  const uint4* wq = reinterpret_cast<const uint4*>(a.q) + tile0 * 32 + lane;
  const uint2* wsc = reinterpret_cast<const uint2*>(a.s) + tile0 * 8 + (lane >> 2);

  uint4 qa[4], qb[4];
  uint2 sa[4], sb[4];
  auto load = [&](uint4 (&qq)[4], uint2 (&ss)[4], int g) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int tile = g * 4 + t;
      if (active && tile < tiles) {
        qq[t] = ld_stream_u4(wq + (size_t)tile * 32);
        ss[t] = ld_stream_u2(wsc + (size_t)tile * 8);
      } else {
        qq[t] = make_uint4(0u, 0u, 0u, 0u);
        ss[t] = make_uint2(0u, 0u);
      }
    }
  };
  load(qa, sa, 0);   // weights do not depend on the previous kernel
  pdl_launch();
  pdl_wait();

  // stage X[:, kbeg:kend] as f16, row stride kc + 8 (conflict-free ldmatrix rows)
  const int xs = kc + 8;
  __half* xsm = reinterpret_cast<__half*>(smem);
  const auto* x = reinterpret_cast<const __nv_bfloat16*>(a.x);
  const int vpr = kc / 8;
  // eight independent 16-byte loads in flight per thread, then convert and store
  constexpr int kB = 8;
  for (int base = threadIdx.x; base < MT * vpr; base += kNvThreads * kB) {
    uint4 raw[kB];
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int idx = base + b * kNvThreads;
      const int m = idx / vpr, k = kbeg + (idx % vpr) * 8;
      raw[b] = make_uint4(0u, 0u, 0u, 0u);
      if (idx < MT * vpr && m < a.M && k < kend) raw[b] = *reinterpret_cast<const uint4*>(x + (size_t)m * a.ldx + k);
    }
#pragma unroll
    for (int b = 0; b < kB; ++b) {
      const int idx = base + b * kNvThreads;
      if (idx >= MT * vpr) break;
      const int m = idx / vpr, v = idx % vpr;
      uint4 o;
      o.x = f32x2_to_f16x2_sat(bf16_lo(raw[b].x), bf16_hi(raw[b].x));
      o.y = f32x2_to_f16x2_sat(bf16_lo(raw[b].y), bf16_hi(raw[b].y));
      o.z = f32x2_to_f16x2_sat(bf16_lo(raw[b].z), bf16_hi(raw[b].z));
      o.w = f32x2_to_f16x2_sat(bf16_lo(raw[b].w), bf16_hi(raw[b].w));
      *reinterpret_cast<uint4*>(xsm + (size_t)m * xs + v * 8) = o;
    }
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[nt][j] = 0.f;
  const uint32_t xbase = smem_u32(xsm) + (uint32_t)(((lane & 7) * xs + ((lane >> 3) & 1) * 8) * 2);

  auto compute = [&](const uint4 (&qq)[4], const uint2 (&ss)[4], int g) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int tile = g * 4 + t;
      if (tile >= tiles) break;
      const uint32_t qw[4] = {qq[t].x, qq[t].y, qq[t].z, qq[t].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint16_t s2 = (uint16_t)(((j < 2 ? ss[t].x : ss[t].y) >> ((j & 1) * 16)) & 0xFFFFu);
        const uint32_t sf = e4m3x2_to_f16x2(s2);
        const uint32_t s_r = __byte_perm(sf, sf, 0x1010), s_r8 = __byte_perm(sf, sf, 0x3232);
        uint32_t h[4];
        e2m1x8_to_f16x8(qw[j], h);
        const uint32_t a0 = hmul2_u32(h[0], s_r), a1 = hmul2_u32(h[1], s_r8);
        const uint32_t a2 = hmul2_u32(h[2], s_r), a3 = hmul2_u32(h[3], s_r8);
        const uint32_t koff = (uint32_t)((tile * 64 + j * 16) * 2);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          uint32_t b0, b1;
          ldsm_x2(xbase + koff + (uint32_t)(nt * 8 * xs * 2), b0, b1);
          mma_f16_16816(acc[nt], a0, a1, a2, a3, b0, b1);
        }
      }
    }
  };
  const int groups = (tiles + 3) / 4;
  for (int g = 0; g < groups; g += 2) {
    load(qb, sb, g + 1);
    compute(qa, sa, g);
    load(qa, sa, g + 2);
    compute(qb, sb, g + 1);
  }

  // accumulators -> S[token][row of block] (fp32), reusing the X staging area
  __syncthreads();
  float* S = reinterpret_cast<float*>(smem);
  {
    const int gr = lane >> 2, tig = lane & 3;
    const int r = warp * 16 + gr;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int m = nt * 8 + tig * 2;
      S[m * kSld + r] = acc[nt][0];
      S[(m + 1) * kSld + r] = acc[nt][1];
      S[m * kSld + r + 8] = acc[nt][2];
      S[(m + 1) * kSld + r + 8] = acc[nt][3];
    }
  }
  __syncthreads();
  const int M = a.M, N = a.N;
  const int n0 = rb * kNvRows;
  if (splits > 1) {
    __shared__ int last;
    float* part = ws + (size_t)sp * M * N;
    for (int idx = threadIdx.x; idx < M * kNvRows; idx += kNvThreads) {
      const int m = idx / kNvRows, r = idx % kNvRows;
      if (n0 + r < N) __stcg(part + (size_t)m * N + n0 + r, S[m * kSld + r]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(counters + rb, 1u) == (uint32_t)(splits - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int idx = threadIdx.x; idx < M * kNvRows; idx += kNvThreads) {
      const int m = idx / kNvRows, r = idx % kNvRows;
      if (n0 + r >= N) continue;
      // the partials' loads are independent: issue them together, add in split order
      const float* src = ws + (size_t)m * N + n0 + r;
      const size_t stride = (size_t)M * N;
      float v = 0.f;
      int p = 0;
      for (; p + 8 <= splits; p += 8) {
        float t[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) t[u] = __ldcg(src + (size_t)(p + u) * stride);
#pragma unroll
        for (int u = 0; u < 8; ++u) v += t[u];
      }
      float t[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) t[u] = p + u < splits ? __ldcg(src + (size_t)(p + u) * stride) : 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) v += t[u];
      S[m * kSld + r] = v;
    }
    if (threadIdx.x == 0) counters[rb] = 0u;
    __syncthreads();
  }
  const float gs = *a.gs;
  const auto* bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  const auto* res = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  auto* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  if (a.epilogue == kEpiSiluMul) {
    // rows 2j / 2j+1 are gate / up of output column j
    for (int idx = threadIdx.x; idx < M * (kNvRows / 2); idx += kNvThreads) {
      const int m = idx / (kNvRows / 2), j = idx % (kNvRows / 2);
      const int n = n0 + 2 * j;
      if (n >= N) continue;
      float gt = S[m * kSld + 2 * j] * gs, up = S[m * kSld + 2 * j + 1] * gs;
      if (bias) {
        gt += __bfloat162float(bias[n]);
        up += __bfloat162float(bias[n + 1]);
      }
      out[(size_t)m * a.ldo + n / 2] = __float2bfloat16(gt / (1.f + __expf(-gt)) * up);
    }
  } else if (a.push) {
    // fused all-reduce: posted stores of the partial into this rank's slot on every rank
    const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(a.ar.epoch);
    const size_t slot = ((size_t)(epoch & 1u) * a.ar.world + a.ar.rank) * (size_t)a.ar.half_floats;
    for (int idx = threadIdx.x; idx < M * kNvRows; idx += kNvThreads) {
      const int m = idx / kNvRows, r = idx % kNvRows;
      const int n = n0 + r;
      if (n >= N) continue;
      const uint16_t bits = bf16_bits_nonempty(S[m * kSld + r] * gs);
      for (int p = 0; p < a.ar.world; ++p) st_relaxed_sys_u16(a.ar.xbuf[p] + slot + (size_t)m * N + n, bits);
    }
  } else {
    for (int idx = threadIdx.x; idx < M * kNvRows; idx += kNvThreads) {
      const int m = idx / kNvRows, r = idx % kNvRows;
      const int n = n0 + r;
      if (n >= N) continue;
      float y = S[m * kSld + r] * gs;
      if (bias) y += __bfloat162float(bias[n]);
      if (res) y += __bfloat162float(res[(size_t)m * a.ldo + n]);
      out[(size_t)m * a.ldo + n] = __float2bfloat16(y);
    }
  }
}

constexpr int kNvSmemCap = 100 * 1024;

}  // namespace

void nvfp4_quantize(const void* w, int64_t ldw, int N, int K, const float* gs, uint8_t* q, uint8_t* s,
                    cudaStream_t st) {
  VRM_REQUIRE(N % 16 == 0 && K % 64 == 0, "nvfp4: N must be a multiple of 16 and K of 64");
  VRM_REQUIRE(ldw % 8 == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0, "nvfp4: weight rows 16-byte aligned");
  const size_t nsc = (size_t)N * (K / 16);
  auto* sc = static_cast<uint8_t*>(workspace_get(nsc, st));
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  nvfp4_block_scales_kernel<<<(unsigned)((nsc + 255) / 256), 256, 0, st>>>(wp, ldw, N, K, gs, sc);
  VRM_CUDA_CHECK(cudaGetLastError());
  const size_t threads = (size_t)(N / 16) * (K / 64) * 32;
  nvfp4_pack_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(wp, ldw, N, K, gs, sc, q, s);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void nvfp4_dequantize(const uint8_t* q, const uint8_t* s, const float* gs, int N, int K, void* out,
                      cudaStream_t st) {
  VRM_REQUIRE(N % 16 == 0 && K % 64 == 0, "nvfp4: N must be a multiple of 16 and K of 64");
  const int64_t warps = (int64_t)(N / 16) * (K / 64);
  launch_kernel(nvfp4_dequant_kernel, dim3((unsigned)((warps + 7) / 8)), dim3(256), 0, st, q, s, gs, N, K,
                reinterpret_cast<__nv_bfloat16*>(out));
  VRM_CUDA_CHECK(cudaGetLastError());
}

int nvfp4_gemm_max_m() { return 32; }

void nvfp4_gemm(const Nvfp4GemmArgs& a, cudaStream_t st) {
  VRM_REQUIRE(a.N % 16 == 0 && a.K % 64 == 0, "nvfp4 gemm: N must be a multiple of 16 and K of 64");
  VRM_REQUIRE(a.M >= 1 && a.M <= 32, "nvfp4 gemm: M must be in [1, 32] (dequantise for larger M)");
  VRM_REQUIRE(a.ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0, "nvfp4 gemm: x rows 16-byte aligned");
  VRM_REQUIRE(a.epilogue != kEpiSiluMul || a.residual == nullptr, "nvfp4 gemm: silu_mul takes no residual");
  VRM_REQUIRE(!a.push || (a.epilogue == kEpiNone && !a.bias && !a.residual && a.ar.xbuf && a.ar.epoch &&
                          (long long)a.M * a.N <= a.ar.half_floats),
              "nvfp4 gemm: the all-reduce push stores the raw partial into the receive buffer");
  const int NT = (a.M + 7) / 8;
  const int rbs = (a.N + kNvRows - 1) / kNvRows;
  const int ktiles = a.K / 64;
  // fill the 2 CTAs per SM of one wave without spilling into a second one, and keep the
  // staged X slice within the shared-memory cap
  const int slots = 2 * device_sm_count();
  int splits = std::max(1, std::min(ktiles, slots / rbs));
  auto smem_for = [&](int sp) {
    const int kc = ((ktiles + sp - 1) / sp) * 64;
    return std::max((size_t)NT * 8 * (kc + 8) * 2, (size_t)NT * 8 * kSld * 4);
  };
  while (smem_for(splits) > (size_t)kNvSmemCap && splits < ktiles) ++splits;
  const int tps = (ktiles + splits - 1) / splits;
  splits = (ktiles + tps - 1) / tps;
  const int kc = tps * 64;
  const size_t smem = smem_for(splits);
  float* ws = nullptr;
  uint32_t* counters = nullptr;
  if (splits > 1) {
    ws = static_cast<float*>(workspace_get((size_t)splits * a.M * a.N * sizeof(float), st));
    counters = tile_counters_get(st);
    VRM_REQUIRE(rbs <= 32768, "nvfp4 gemm: too many row blocks");
  }
  dim3 grid(rbs, splits);
  switch (NT) {
#define VRM_NV_CASE(T)                                                                                        \
  case T: {                                                                                                    \
    static int attr_mask = 0;                                                                                  \
    int dev = 0;                                                                                               \
    cudaGetDevice(&dev);                                                                                       \
    if (!(attr_mask & (1 << (dev & 31)))) {                                                                    \
      VRM_CUDA_CHECK(cudaFuncSetAttribute(nvfp4_gemm_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,  \
                                          kNvSmemCap));                                                        \
      attr_mask |= 1 << (dev & 31);                                                                            \
    }                                                                                                          \
    launch_kernel(nvfp4_gemm_kernel<T>, grid, dim3(kNvThreads), smem, st, a, kc, splits, ws, counters);        \
  } break;
    VRM_NV_CASE(1)
    VRM_NV_CASE(2)
    VRM_NV_CASE(3)
    default: VRM_NV_CASE(4)
#undef VRM_NV_CASE
  }
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
