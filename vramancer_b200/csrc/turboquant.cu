// TurboQuant KV records (64 bytes per 128-dim vector): randomized Hadamard rotation,
// PolarQuant angles (3 bits), 1-bit QJL sketch of the residual.  Record layout and
// math: vramancer_b200/kv/turboquant.py (the torch oracle of these kernels).
//
// One warp per vector; lane l holds elements 4l..4l+3.  The Walsh-Hadamard butterflies
// run in registers for h = 1, 2 and across lanes with shfl_xor for h = 4..64, in the
// oracle's stage order (identical fp32 results).  The polar tree pairs elements in
// registers for levels 0-1 and lanes for levels 2-6; the 64 JL projections of the
// residual are two per lane over the CTA's shared copy of P, and their signs come out
// of two ballots already bit-packed.
//
// Reference parity: csrc/turboquant_kernel.cu:36-405 (Hadamard + polar encode/decode +
// QJL in fused compress / decompress kernels).
#include <cooperative_groups.h>
#include <cuda_fp16.h>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kTqD = 128, kTqM = 64, kTqBits = 3, kTqRec = 64;
constexpr int kTqWarps = 8;
constexpr float kPi = 3.14159265358979323846f;

// angle-slot base of each polar level (64 + 32 + ... + 1 = 127 slots)
__device__ __forceinline__ int level_base(int k) { return kTqD - (kTqD >> k); }

__device__ __forceinline__ void fwht4(float (&v)[4], int lane) {
  // h = 1, 2 inside the lane
  float a = v[0], b = v[1], c = v[2], d = v[3];
  v[0] = a + b; v[1] = a - b; v[2] = c + d; v[3] = c - d;
  a = v[0]; b = v[1]; c = v[2]; d = v[3];
  v[0] = a + c; v[1] = b + d; v[2] = a - c; v[3] = b - d;
  // h = 4 .. 64: partner lane differs in bit (h / 4)
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = lane & m;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float p = __shfl_xor_sync(0xffffffffu, v[j], m);
      v[j] = upper ? p - v[j] : v[j] + p;
    }
  }
  // divide (not multiply by the reciprocal): bit-identical to the oracle's x / sqrt(128)
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] = v[j] / 11.313708498984761f;
}

__device__ __forceinline__ int quant_angle(float ang, int level) {
  const float lo = level == 0 ? -kPi : 0.f;
  const float span = level == 0 ? 2.f * kPi : 0.5f * kPi;
  const float q = floorf((ang - lo) / span * (float)(1 << kTqBits));
  return (int)fminf(fmaxf(q, 0.f), (float)((1 << kTqBits) - 1));
}

__device__ __forceinline__ float angle_centre(int q, int level) {
  const float lo = level == 0 ? -kPi : 0.f;
  const float span = level == 0 ? 2.f * kPi : 0.5f * kPi;
  return lo + ((float)q + 0.5f) * span / (float)(1 << kTqBits);
}

// polar decode of the rotated vector from angle slots (shared) and the radius
__device__ __forceinline__ void polar_decode(const uint8_t* idx, float radius, int lane, float (&v)[4]) {
  float R = radius;
  // levels 6 .. 2: lanes paired across bit (k - 2)
#pragma unroll
  for (int k = 6; k >= 2; --k) {
    const int span = 1 << (k - 1);                 // lanes under one angle
    const float th = angle_centre(idx[level_base(k) + lane / span], k);
    R = (lane & (1 << (k - 2))) ? R * sinf(th) : R * cosf(th);
  }
  const float t1 = angle_centre(idx[level_base(1) + lane], 1);
  const float r0 = R * cosf(t1), r1 = R * sinf(t1);
  const float a0 = angle_centre(idx[2 * lane], 0), a1 = angle_centre(idx[2 * lane + 1], 0);
  v[0] = r0 * cosf(a0);
  v[1] = r0 * sinf(a0);
  v[2] = r1 * cosf(a1);
  v[3] = r1 * sinf(a1);
}

template <typename T>
__device__ __forceinline__ void load4(const T* p, float (&v)[4]);
template <>
__device__ __forceinline__ void load4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  v[0] = bf16_lo(u.x); v[1] = bf16_hi(u.x); v[2] = bf16_lo(u.y); v[3] = bf16_hi(u.y);
}
template <>
__device__ __forceinline__ void load4<float>(const float* p, float (&v)[4]) {
  const float4 u = *reinterpret_cast<const float4*>(p);
  v[0] = u.x; v[1] = u.y; v[2] = u.z; v[3] = u.w;
}

// One warp encodes one vector: v[4] = the lane's dims 4l..4l+3 (not yet sign-flipped);
// the 64-byte record goes to out (16 lanes store 4 bytes each).  idx / r / rec are the
// warp's scratch in shared memory; jl is the CTA's padded copy of P.
__device__ __forceinline__ void tq_encode(float (&v)[4], int lane, const float* s_sign, const float (*s_jl)[kTqD + 1],
                                          float* s_r, uint8_t* idx, uint8_t* rec, uint8_t* out) {
#pragma unroll
  for (int j = 0; j < 4; ++j) v[j] *= s_sign[4 * lane + j];
  fwht4(v, lane);
  // ---- polar encode
  const float ra = sqrtf(v[0] * v[0] + v[1] * v[1]), rb = sqrtf(v[2] * v[2] + v[3] * v[3]);
  idx[2 * lane] = (uint8_t)quant_angle(atan2f(v[1], v[0]), 0);
  idx[2 * lane + 1] = (uint8_t)quant_angle(atan2f(v[3], v[2]), 0);
  idx[level_base(1) + lane] = (uint8_t)quant_angle(atan2f(rb, ra), 1);
  float R = sqrtf(ra * ra + rb * rb);
#pragma unroll
  for (int k = 2; k <= 6; ++k) {
    const int m = 1 << (k - 2);
    const float p = __shfl_xor_sync(0xffffffffu, R, m);
    const bool lower = !(lane & m);
    const float a = lower ? R : p, b = lower ? p : R;
    if ((lane & ((m << 1) - 1)) == 0) idx[level_base(k) + lane / (m << 1)] = (uint8_t)quant_angle(atan2f(b, a), k);
    R = sqrtf(a * a + b * b);
  }
  if (lane == 0) idx[kTqD - 1] = 0;
  const __half r16 = __float2half_rn(R);
  __syncwarp();
  // ---- residual against the decoded vector (fp16 radius, as stored)
  float d[4];
  polar_decode(idx, __half2float(r16), lane, d);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float r = v[j] - d[j];
    s_r[4 * lane + j] = r;
    ss += r * r;
  }
  const float nrm = sqrtf(warp_sum(ss));
  __syncwarp();
  // ---- QJL: projections lane and lane + 32, signs by ballot
  float p0 = 0.f, p1 = 0.f;
#pragma unroll 8
  for (int i = 0; i < kTqD; ++i) {
    const float r = s_r[i];
    p0 += s_jl[lane][i] * r;
    p1 += s_jl[lane + 32][i] * r;
  }
  const uint32_t b0 = __ballot_sync(0xffffffffu, p0 > 0.f), b1 = __ballot_sync(0xffffffffu, p1 > 0.f);
  // ---- record: angles (3 bytes per 8 slots), radius, signs, residual norm
  if (lane < 16) {
    uint32_t bits = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) bits |= (uint32_t)idx[8 * lane + j] << (3 * j);
    rec[3 * lane] = (uint8_t)bits;
    rec[3 * lane + 1] = (uint8_t)(bits >> 8);
    rec[3 * lane + 2] = (uint8_t)(bits >> 16);
  } else if (lane == 16) {
    const unsigned short rb16 = __half_as_ushort(r16);
    const unsigned short nb16 = __half_as_ushort(__float2half_rn(nrm));
    rec[48] = (uint8_t)rb16;
    rec[49] = (uint8_t)(rb16 >> 8);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      rec[50 + j] = (uint8_t)(b0 >> (8 * j));
      rec[54 + j] = (uint8_t)(b1 >> (8 * j));
    }
    rec[58] = (uint8_t)nb16;
    rec[59] = (uint8_t)(nb16 >> 8);
    rec[60] = rec[61] = rec[62] = rec[63] = 0;
  }
  __syncwarp();
  if (lane < 16) reinterpret_cast<uint32_t*>(out)[lane] = reinterpret_cast<const uint32_t*>(rec)[lane];
  __syncwarp();
}

template <typename T>
__global__ void __launch_bounds__(kTqWarps * 32) tq_compress_kernel(const T* __restrict__ x, int64_t n,
                                                                    const float* __restrict__ signs,
                                                                    const float* __restrict__ jl,
                                                                    uint8_t* __restrict__ out) {
  // rows padded to 129 floats: lane l reads row l (and l + 32) at the same column, so
  // an unpadded 128-float stride puts all 32 lanes in one bank (32-way conflicts)
  __shared__ float s_jl[kTqM][kTqD + 1];
  __shared__ float s_sign[kTqD];
  __shared__ float s_r[kTqWarps][kTqD];
  __shared__ uint8_t s_idx[kTqWarps][kTqD];
  __shared__ __align__(16) uint8_t s_rec[kTqWarps][kTqRec];
  pdl_launch();
  for (int i = threadIdx.x; i < kTqM * kTqD; i += blockDim.x) s_jl[i / kTqD][i % kTqD] = jl[i];
  for (int i = threadIdx.x; i < kTqD; i += blockDim.x) s_sign[i] = signs[i];
  pdl_wait_for(x, signs, jl);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int64_t vec = (int64_t)blockIdx.x * kTqWarps + warp; vec < n; vec += (int64_t)gridDim.x * kTqWarps) {
    float v[4];
    load4<T>(x + vec * kTqD + 4 * lane, v);
    tq_encode(v, lane, s_sign, s_jl, s_r[warp], s_idx[warp], s_rec[warp], out + vec * kTqRec);
  }
}

// TurboQuant KV pages: the (already rotated) k and v rows of each token of a qkv buffer
// [T, (Hq + 2 KH) * 128] become records in pool[page, layer, k|v, kv_head, slot] (64 B).
__global__ void __launch_bounds__(kTqWarps * 32) tq_kv_write_kernel(const __nv_bfloat16* __restrict__ qkv, int64_t ld,
                                                                    int T, int Hq, int KH,
                                                                    const int* __restrict__ slot_mapping,
                                                                    uint8_t* __restrict__ pool, int num_layers,
                                                                    int layer, long long num_pages,
                                                                    const float* __restrict__ signs,
                                                                    const float* __restrict__ jl,
                                                                    uint32_t* __restrict__ err) {
  __shared__ float s_jl[kTqM][kTqD + 1];
  __shared__ float s_sign[kTqD];
  __shared__ float s_r[kTqWarps][kTqD];
  __shared__ uint8_t s_idx[kTqWarps][kTqD];
  __shared__ __align__(16) uint8_t s_rec[kTqWarps][kTqRec];
  pdl_launch();
  for (int i = threadIdx.x; i < kTqM * kTqD; i += blockDim.x) s_jl[i / kTqD][i % kTqD] = jl[i];
  for (int i = threadIdx.x; i < kTqD; i += blockDim.x) s_sign[i] = signs[i];
  pdl_wait_for(qkv, slot_mapping);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = (int64_t)T * 2 * KH;
  for (int64_t vec = (int64_t)blockIdx.x * kTqWarps + warp; vec < n; vec += (int64_t)gridDim.x * kTqWarps) {
    const int t = (int)(vec / (2 * KH));
    const int hv = (int)(vec % (2 * KH));      // kv * KH + head
    const int slot = slot_mapping[t];
    if (slot < 0 || !in_bounds(slot / 16, num_pages, err)) continue;
    float v[4];
    load4<__nv_bfloat16>(qkv + (size_t)t * ld + (size_t)(Hq + hv) * kTqD + 4 * lane, v);
    const int page = slot / 16, off = slot % 16;
    uint8_t* dst = pool + ((((size_t)page * num_layers + layer) * 2 * KH + hv) * 16 + off) * kTqRec;
    tq_encode(v, lane, s_sign, s_jl, s_r[warp], s_idx[warp], s_rec[warp], dst);
  }
}

__global__ void __launch_bounds__(kTqWarps * 32) tq_decompress_kernel(const uint8_t* __restrict__ rec_in, int64_t n,
                                                                      const float* __restrict__ signs,
                                                                      __nv_bfloat16* __restrict__ out) {
  __shared__ __align__(16) uint8_t s_rec[kTqWarps][kTqRec];
  __shared__ uint8_t s_idx[kTqWarps][kTqD];
  pdl_launch();
  pdl_wait_for(rec_in, signs);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* rec = s_rec[warp];
  uint8_t* idx = s_idx[warp];
  float sg[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) sg[j] = signs[4 * lane + j];
  for (int64_t vec = (int64_t)blockIdx.x * kTqWarps + warp; vec < n; vec += (int64_t)gridDim.x * kTqWarps) {
    if (lane < 16)
      reinterpret_cast<uint32_t*>(rec)[lane] = reinterpret_cast<const uint32_t*>(rec_in + vec * kTqRec)[lane];
    __syncwarp();
    if (lane < 16) {
      const uint32_t bits = rec[3 * lane] | (uint32_t)rec[3 * lane + 1] << 8 | (uint32_t)rec[3 * lane + 2] << 16;
#pragma unroll
      for (int j = 0; j < 8; ++j) idx[8 * lane + j] = (uint8_t)((bits >> (3 * j)) & 7u);
    }
    const float radius = __half2float(__ushort_as_half((unsigned short)(rec[48] | (rec[49] << 8))));
    __syncwarp();
    float v[4];
    polar_decode(idx, radius, lane, v);
    fwht4(v, lane);
    uint2 o;
    o.x = pack_bf16x2(v[0] * sg[0], v[1] * sg[1]);
    o.y = pack_bf16x2(v[2] * sg[2], v[3] * sg[3]);
    *reinterpret_cast<uint2*>(out + vec * kTqD + 4 * lane) = o;
    __syncwarp();
  }
}

// ---------------------------------------------------------------- attention over records
// Decode attention straight from TurboQuant K / V pages (one query token per sequence).
// grid (kv_heads, batch), 8 warps; the warps take the tokens round-robin, one token per
// warp step, lanes holding dims 4l..4l+3 of the rotated domain:
//   score_h = <q_rot_h, k_hat_rot> + sqrt(pi/2) / m * ||r|| * <P q_rot_h, sign(P r)>
// (q_rot and P q_rot are computed once per CTA for the group's query heads), online
// softmax per warp and head, values accumulated as their rotated polar decodes; the
// warps merge in shared memory and the sum is unrotated once per head (the rotation
// is linear, so no value is unrotated on its own).  cos / sin of the 8 bin centres of
// both angle ranges come from a table filled with the same sinf / cosf as the encoder.
constexpr int kTqAttnWarps = 8;

struct TqTables {
  float c[2][8], s[2][8];
};

__device__ __forceinline__ void polar_decode_tab(const uint8_t* idx, float radius, int lane, const TqTables& T,
                                                 float (&v)[4]) {
  float R = radius;
#pragma unroll
  for (int k = 6; k >= 2; --k) {
    const int span = 1 << (k - 1);
    const int q = idx[level_base(k) + lane / span];
    R = (lane & (1 << (k - 2))) ? R * T.s[1][q] : R * T.c[1][q];
  }
  const int q1 = idx[level_base(1) + lane];
  const float r0 = R * T.c[1][q1], r1 = R * T.s[1][q1];
  const int a0 = idx[2 * lane], a1 = idx[2 * lane + 1];
  v[0] = r0 * T.c[0][a0];
  v[1] = r0 * T.s[0][a0];
  v[2] = r1 * T.c[0][a1];
  v[3] = r1 * T.s[0][a1];
}

// the warp's record (already in rec) -> angle slots in idx; returns the radius
__device__ __forceinline__ float unpack_record(const uint8_t* rec, uint8_t* idx, int lane) {
  if (lane < 16) {
    const uint32_t bits = rec[3 * lane] | (uint32_t)rec[3 * lane + 1] << 8 | (uint32_t)rec[3 * lane + 2] << 16;
#pragma unroll
    for (int j = 0; j < 8; ++j) idx[8 * lane + j] = (uint8_t)((bits >> (3 * j)) & 7u);
  }
  __syncwarp();
  return __half2float(__ushort_as_half((unsigned short)(rec[48] | (rec[49] << 8))));
}

template <bool kCluster>
__global__ void __launch_bounds__(kTqAttnWarps * 32) tq_paged_decode_kernel(
    const __nv_bfloat16* __restrict__ q, int64_t ld_q, const uint8_t* __restrict__ pool, int num_layers, int layer,
    int KH, int G, const int* __restrict__ block_tables, int bt_stride, const int* __restrict__ context_lens,
    const float* __restrict__ signs, const float* __restrict__ jl, float sm_scale, __nv_bfloat16* __restrict__ out,
    int64_t ld_o, long long num_pages, uint32_t* __restrict__ err) {
  __shared__ TqTables T;
  __shared__ float s_sign[kTqD];
  __shared__ float s_q[8][kTqD];                  // rotated queries of the group
  __shared__ float s_pq[8][kTqM];                 // P q_rot
  __shared__ __align__(16) uint8_t s_rec[kTqAttnWarps][2][kTqRec];
  __shared__ uint8_t s_idx[kTqAttnWarps][2][kTqD];
  __shared__ float s_m[kTqAttnWarps][8], s_l[kTqAttnWarps][8];
  __shared__ float s_acc[kTqAttnWarps][8][kTqD];
  __shared__ float s_fm[8], s_fl[8];              // this CTA's merged (max, sum) per head
  __shared__ float s_fo[8][kTqD];                 // and its rotated output (unnormalised)
  pdl_launch();
  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, nsplit = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x < 16) {
    const int lv = threadIdx.x >> 3, qb = threadIdx.x & 7;
    const float th = angle_centre(qb, lv);
    T.c[lv][qb] = cosf(th);
    T.s[lv][qb] = sinf(th);
  }
  for (int i = threadIdx.x; i < kTqD; i += blockDim.x) s_sign[i] = signs[i];
  pdl_wait_for(q, pool, block_tables, context_lens);
  __syncthreads();
  // rotated queries and their JL projections (warp h < G)
  if (warp < G) {
    const __nv_bfloat16* qr = q + (size_t)b * ld_q + (size_t)(kvh * G + warp) * kTqD + 4 * lane;
    float v[4];
    load4<__nv_bfloat16>(qr, v);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] *= s_sign[4 * lane + j];
    fwht4(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) s_q[warp][4 * lane + j] = v[j];
    __syncwarp();
    float p0 = 0.f, p1 = 0.f;
    for (int i = 0; i < kTqD; ++i) {
      const float x = s_q[warp][i];
      p0 += __ldg(jl + (size_t)lane * kTqD + i) * x;
      p1 += __ldg(jl + (size_t)(lane + 32) * kTqD + i) * x;
    }
    s_pq[warp][lane] = p0;
    s_pq[warp][lane + 32] = p1;
  }
  __syncthreads();
  const int ctx = context_lens[b];
  const int per = (ctx + nsplit - 1) / nsplit;
  const int t_begin = split * per, t_end = min(ctx, t_begin + per);
  const int* bt = block_tables + (size_t)b * bt_stride;
  const float qjl_c = 1.2533141373155003f / (float)kTqM;   // sqrt(pi / 2) / m
  const float sl2 = sm_scale * 1.4426950408889634f;
  float qv[8][4], pqa[8], pqb[8];
#pragma unroll
  for (int h = 0; h < 8; ++h) {
#pragma unroll
    for (int j = 0; j < 4; ++j) qv[h][j] = h < G ? s_q[h][4 * lane + j] : 0.f;
    pqa[h] = h < G ? s_pq[h][lane] : 0.f;
    pqb[h] = h < G ? s_pq[h][lane + 32] : 0.f;
  }
  float m_run[8], l_run[8], acc[8][4];
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[h][j] = 0.f;
  }
  uint8_t* krec = s_rec[warp][0];
  uint8_t* vrec = s_rec[warp][1];
  const size_t vofs = (size_t)KH * 16 * kTqRec;
  // records of this warp's next kPre tokens in flight in registers (lanes 0-15: 4 bytes
  // of the K record and 4 of the V record each): the loads of token i + kPre overlap
  // the arithmetic of token i
  constexpr int kPre = 4;
  uint32_t pk[kPre], pv[kPre];
  auto fetch = [&](int t, uint32_t& kw, uint32_t& vw) {
    kw = vw = 0u;
    if (t < t_end && lane < 16) {
      int page = bt[t >> 4];
      if (!in_bounds(page, num_pages, err)) page = 0;
      const uint8_t* base = pool + ((((size_t)page * num_layers + layer) * 2 * KH + kvh) * 16 + (t & 15)) * kTqRec;
      kw = __ldg(reinterpret_cast<const uint32_t*>(base) + lane);
      vw = __ldg(reinterpret_cast<const uint32_t*>(base + vofs) + lane);
    }
  };
#pragma unroll
  for (int i = 0; i < kPre; ++i) fetch(t_begin + warp + i * kTqAttnWarps, pk[i], pv[i]);
  for (int t = t_begin + warp; t < t_end; t += kTqAttnWarps) {
    // this token's words -> shared; refill the slot with the token kPre steps ahead
    uint32_t kw = pk[0], vw = pv[0];
#pragma unroll
    for (int i = 0; i < kPre - 1; ++i) {
      pk[i] = pk[i + 1];
      pv[i] = pv[i + 1];
    }
    fetch(t + kPre * kTqAttnWarps, pk[kPre - 1], pv[kPre - 1]);
    if (lane < 16) {
      reinterpret_cast<uint32_t*>(krec)[lane] = kw;
      reinterpret_cast<uint32_t*>(vrec)[lane] = vw;
    }
    __syncwarp();
    const float kr = unpack_record(krec, s_idx[warp][0], lane);
    const float vr = unpack_record(vrec, s_idx[warp][1], lane);
    float kv4[4], vv4[4];
    polar_decode_tab(s_idx[warp][0], kr, lane, T, kv4);
    polar_decode_tab(s_idx[warp][1], vr, lane, T, vv4);
    // sign words at record bytes 50..53 and 54..57: not 4-byte aligned, assembled bytewise
    const uint32_t sg0 = (uint32_t)krec[50] | (uint32_t)krec[51] << 8 | (uint32_t)krec[52] << 16 |
                         (uint32_t)krec[53] << 24;
    const uint32_t sg1 = (uint32_t)krec[54] | (uint32_t)krec[55] << 8 | (uint32_t)krec[56] << 16 |
                         (uint32_t)krec[57] << 24;
    const float nrm = __half2float(__ushort_as_half((unsigned short)(krec[58] | (krec[59] << 8))));
    const float sa = (sg0 >> lane) & 1u ? 1.f : -1.f, sb = (sg1 >> lane) & 1u ? 1.f : -1.f;
    float sc[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      float x = kv4[0] * qv[h][0] + kv4[1] * qv[h][1] + kv4[2] * qv[h][2] + kv4[3] * qv[h][3];
      x += qjl_c * nrm * (sa * pqa[h] + sb * pqb[h]);
      sc[h] = x;
    }
#pragma unroll
    for (int h = 0; h < 8; ++h) sc[h] = warp_sum(sc[h]);
#pragma unroll
    for (int h = 0; h < 8; ++h) {
      if (h >= G) continue;
      const float x = sc[h] * sl2;
      const float mn = fmaxf(m_run[h], x);
      const float alpha = exp2f(m_run[h] - mn);    // 0 on the first token
      const float p = exp2f(x - mn);
      l_run[h] = l_run[h] * alpha + p;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[h][j] = acc[h][j] * alpha + p * vv4[j];
      m_run[h] = mn;
    }
    __syncwarp();
  }
  // ---- merge this CTA's warps (rotated domain, unnormalised)
#pragma unroll
  for (int h = 0; h < 8; ++h) {
    if (h >= G) continue;
    if (lane == 0) {
      s_m[warp][h] = m_run[h];
      s_l[warp][h] = l_run[h];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_acc[warp][h][4 * lane + j] = acc[h][j];
  }
  __syncthreads();
  if (warp < G) {
    const int h = warp;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTqAttnWarps; ++w) M = fmaxf(M, s_m[w][h]);
    float L = 0.f, v[4] = {0.f, 0.f, 0.f, 0.f};
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTqAttnWarps; ++w) {
        const float f = exp2f(s_m[w][h] - M);
        L += s_l[w][h] * f;
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] += s_acc[w][h][4 * lane + j] * f;
      }
    }
    if (lane == 0) {
      s_fm[h] = M;
      s_fl[h] = L;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) s_fo[h][4 * lane + j] = v[j];
  }
  // ---- merge the splits of the cluster (DSMEM): CTA rank r finishes heads r, r + S, ...
  if constexpr (kCluster) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = (int)cluster.block_rank();
    for (int h = rank + warp * nsplit; h < G; h += kTqAttnWarps * nsplit) {
      float M = -INFINITY;
      for (int r = 0; r < nsplit; ++r) M = fmaxf(M, cluster.map_shared_rank(s_fm, r)[h]);
      float L = 0.f, v[4] = {0.f, 0.f, 0.f, 0.f};
      if (M != -INFINITY) {
        for (int r = 0; r < nsplit; ++r) {
          const float f = exp2f(cluster.map_shared_rank(s_fm, r)[h] - M);
          L += cluster.map_shared_rank(s_fl, r)[h] * f;
          const float* o = cluster.map_shared_rank(&s_fo[0][0], r) + h * kTqD + 4 * lane;
#pragma unroll
          for (int j = 0; j < 4; ++j) v[j] += o[j] * f;
        }
      }
      const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] *= inv;
      fwht4(v, lane);                            // H / sqrt(D): its own inverse
      uint2 o2;
      o2.x = pack_bf16x2(v[0] * s_sign[4 * lane], v[1] * s_sign[4 * lane + 1]);
      o2.y = pack_bf16x2(v[2] * s_sign[4 * lane + 2], v[3] * s_sign[4 * lane + 3]);
      *reinterpret_cast<uint2*>(out + (size_t)b * ld_o + (size_t)(kvh * G + h) * kTqD + 4 * lane) = o2;
    }
    cluster.sync();     // peers' shared memory stays valid until every CTA has read it
  } else {
    __syncthreads();
    if (warp < G) {
      const int h = warp;
      const float L = s_fl[h];
      const float inv = L > 0.f ? 1.f / L : 0.f;
      float v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) v[j] = s_fo[h][4 * lane + j] * inv;
      fwht4(v, lane);
      uint2 o2;
      o2.x = pack_bf16x2(v[0] * s_sign[4 * lane], v[1] * s_sign[4 * lane + 1]);
      o2.y = pack_bf16x2(v[2] * s_sign[4 * lane + 2], v[3] * s_sign[4 * lane + 3]);
      *reinterpret_cast<uint2*>(out + (size_t)b * ld_o + (size_t)(kvh * G + h) * kTqD + 4 * lane) = o2;
    }
  }
}

int tq_grid(int64_t n) {
  const int64_t need = (n + kTqWarps - 1) / kTqWarps;
  return (int)std::max<int64_t>(1, std::min<int64_t>(need, 4ll * device_sm_count()));
}

}  // namespace

void tq_compress(const void* x, bool x_bf16, int64_t n, const float* signs, const float* jl, uint8_t* out,
                 cudaStream_t st) {
  if (n <= 0) return;
  if (x_bf16)
    launch_kernel(tq_compress_kernel<__nv_bfloat16>, dim3(tq_grid(n)), dim3(kTqWarps * 32), 0, st,
                  reinterpret_cast<const __nv_bfloat16*>(x), n, signs, jl, out);
  else
    launch_kernel(tq_compress_kernel<float>, dim3(tq_grid(n)), dim3(kTqWarps * 32), 0, st,
                  reinterpret_cast<const float*>(x), n, signs, jl, out);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void tq_kv_write(const void* qkv, int64_t ld, int T, int Hq, int KH, const int* slot_mapping, uint8_t* pool,
                 int num_layers, int layer, int64_t num_pages, const float* signs, const float* jl, cudaStream_t st) {
  if (T <= 0) return;
  launch_kernel(tq_kv_write_kernel, dim3(tq_grid((int64_t)T * 2 * KH)), dim3(kTqWarps * 32), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(qkv), ld, T, Hq, KH, slot_mapping, pool, num_layers, layer,
                (long long)num_pages, signs, jl, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void tq_paged_decode(const void* q, int64_t ld_q, const uint8_t* pool, int num_layers, int layer, int KH, int Hq,
                     const int* block_tables, int bt_stride, const int* context_lens, int B, const float* signs,
                     const float* jl, float sm_scale, void* out, int64_t ld_o, int64_t num_pages, cudaStream_t st) {
  VRM_REQUIRE(KH > 0 && Hq % KH == 0 && Hq / KH <= 8, "turboquant decode: GQA group <= 8 heads");
  if (B <= 0) return;
  // splits of the context over the CTAs of a cluster (merged over DSMEM) when the
  // (sequence, KV head) groups alone leave SMs idle
  const int groups = B * KH;
  int splits = 1;
  while (splits < 8 && groups * splits * 2 <= device_sm_count()) splits *= 2;
  const dim3 grid(KH, B, splits);
  if (splits > 1)
    launch_kernel_cluster(tq_paged_decode_kernel<true>, grid, dim3(kTqAttnWarps * 32), dim3(1, 1, splits), 0, st,
                          reinterpret_cast<const __nv_bfloat16*>(q), ld_q, pool, num_layers, layer, KH, Hq / KH,
                          block_tables, bt_stride, context_lens, signs, jl, sm_scale,
                          reinterpret_cast<__nv_bfloat16*>(out), ld_o, (long long)num_pages, error_word());
  else
    launch_kernel(tq_paged_decode_kernel<false>, grid, dim3(kTqAttnWarps * 32), 0, st,
                  reinterpret_cast<const __nv_bfloat16*>(q), ld_q, pool, num_layers, layer, KH, Hq / KH, block_tables,
                  bt_stride, context_lens, signs, jl, sm_scale, reinterpret_cast<__nv_bfloat16*>(out), ld_o,
                  (long long)num_pages, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void tq_decompress(const uint8_t* rec, int64_t n, const float* signs, void* out, cudaStream_t st) {
  if (n <= 0) return;
  launch_kernel(tq_decompress_kernel, dim3(tq_grid(n)), dim3(kTqWarps * 32), 0, st, rec, n, signs,
                reinterpret_cast<__nv_bfloat16*>(out));
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
