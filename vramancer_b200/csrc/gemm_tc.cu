// bf16 GEMM on the 5th-generation tensor cores (tcgen05 + TMEM), sm_100a.
//
//   Y[M, N] = X[M, K] @ W[N, K]^T (+ bias[N]) (+ residual[M, N])   (nn.Linear layout)
//
// One CTA = 6 warps, warp-specialised:
//   warp 0      TMA producer: streams K-major 128B-swizzled tiles of both operands
//               into a STAGES-deep shared-memory ring (mbarrier complete_tx).
//   warp 1      allocates the TMEM accumulator and issues tcgen05.mma (one thread),
//               releasing each smem stage with tcgen05.commit -> empty barrier.
//   warps 2..5  epilogue: tcgen05.ld from TMEM, bias / SiLU*up / residual, bf16 store.
//
// Two operand orientations share the kernel:
//   * kSwapAB = false (prefill, M > 128): MMA-M = tokens, MMA-N = features.
//   * kSwapAB = true  (decode, M <= 128): MMA-M = 128 weight rows, MMA-N = the few
//     tokens padded to 16/32/64/128 (TMA zero-fills rows past M).  The 128-lane tensor
//     core then works on the weight stream, which is what bounds decode.
// Split-K: when there are too few output tiles to cover the SMs, K is split over
// gridDim.y.  Each split writes an fp32 partial; the last CTA to finish a tile (tile
// counter, reset after use) sums the partials in split order (deterministic) and runs
// the epilogue.  Workspace and counters are persistent per-device scratch.
//
// Reference parity: replaces the reference's cuBLAS linear layers on its HF/accelerate
// path (core/backends.py:1390) and its SIMT NVFP4 GEMV (csrc/fp4_gemv.cu:36-116) for
// the bf16 case.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>
#include <unordered_map>

#include <cooperative_groups.h>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

constexpr int kBM = 128;        // MMA M (TMEM lanes)
constexpr int kBK = 64;         // K elements per stage (128 B of bf16 = one swizzle row)
constexpr int kUmmaK = 16;      // K per tcgen05.mma kind::f16
constexpr int kGemmThreads = 192;

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kBM * kBK * 2;   // 16 KB
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[STAGES], empty[STAGES], tmem_full, then tmem slot + flag
  static constexpr int kTotal = kBarOffset + (2 * STAGES + 1) * 8 + 16;
  static constexpr int kAlloc = kTotal + 1024;   // slack for 1024-B alignment
};

struct EpiParams {
  __nv_bfloat16* out;
  int ldo;
  const __nv_bfloat16* bias;
  const __nv_bfloat16* residual;
  int M, N;       // logical output rows (tokens) and GEMM columns (weight rows)
  int epilogue;
  // FP8 operands: the accumulator is scaled by scale_w[weight row] * scale_x[token] first
  const float* scale_w;
  const float* scale_x;
  // RMSNorm folded into the decode GEMMs (swap-AB stream-K kernel only; GemmArgs):
  // a producer (residual epilogue) stores per (weight tile, token) the sum over the
  // tile's 128 features of bf16(out)^2 at ssq_out[tile * ssq_ld + token]; a consumer
  // scales its accumulator by rstd[m] = rsqrt(sum_p ssq_in[p * ssq_ld + m] / norm_dim
  // + eps) before bias and SiLU (its weight columns carry the norm weight).
  float* ssq_out = nullptr;
  const float* ssq_in = nullptr;
  int ssq_ld = 0, ssq_parts = 0, norm_dim = 0;
  float norm_eps = 0.f;
};

// Sum over the warp's 32 lanes of each of 16 per-lane values, reduce-scatter style
// (16 shuffles instead of 16 x 5): every lane returns the total of value index
// (lane >> 1) & 15.  Partners add the same two numbers, so both lanes of a pair agree.
__device__ __forceinline__ float warp_sum16_scatter(float (&q)[16], int lane) {
  {
    const bool up = lane & 16;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float send = up ? q[i] : q[i + 8], keep = up ? q[i + 8] : q[i];
      q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
  }
  {
    const bool up = lane & 8;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float send = up ? q[i] : q[i + 4], keep = up ? q[i + 4] : q[i];
      q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
  }
  {
    const bool up = lane & 4;
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float send = up ? q[i] : q[i + 2], keep = up ? q[i + 2] : q[i];
      q[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
    }
  }
  {
    const bool up = lane & 2;
    const float send = up ? q[0] : q[1], keep = up ? q[1] : q[0];
    q[0] = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return q[0] + __shfl_xor_sync(0xffffffffu, q[0], 1);
}

// Stream-K fixup: out[j] = sum over contributors 1 .. nc-1 (in order) of their fp32
// partial of this thread's row, columns c0 .. c0+15 (`base` = contributor 0's slot at
// this row; slots are kBM x BN apart, column-major with kBM rows).  Two contributors'
// loads are in flight at once.
template <int BN>
__device__ __forceinline__ void sum_partials16_t(const float* base, int nc, int c0, float (&out)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = 0.f;
  for (int q0 = 1; q0 < nc; q0 += 2) {
    float x[2][16];
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int j = 0; j < 16; ++j)
        x[u][j] = q0 + u < nc ? __ldcg(base + (size_t)(q0 + u) * (kBM * BN) + (size_t)(c0 + j) * kBM) : 0.f;
#pragma unroll
    for (int u = 0; u < 2; ++u)
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] += x[u][j];
  }
}

// Cluster barrier halves (non-aligned: threads of divergent roles call them on their own).
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }

// Cluster fixup of a split tile: the owner (cluster rank 0) sums the 16-column chunk c0
// of contributors 1 .. nc-1, read from their shared memory ([column][row] fp32), four
// peers' loads in flight at once, in contributor order.
template <int BN>
__device__ __forceinline__ void sum_peers16(const float* s_part, int nc, int c0, int row, float (&out)[16]) {
  namespace cg = cooperative_groups;
  cg::cluster_group cluster = cg::this_cluster();
#pragma unroll
  for (int j = 0; j < 16; ++j) out[j] = 0.f;
  for (int q0 = 1; q0 < nc; q0 += 4) {
    float x[4][16];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (q0 + u < nc) {
        const float* src = cluster.map_shared_rank(s_part, q0 + u) + row;
#pragma unroll
        for (int j = 0; j < 16; ++j) x[u][j] = src[(c0 + j) * kBM];
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) x[u][j] = 0.f;
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int j = 0; j < 16; ++j) out[j] += x[u][j];
  }
}

// Store one accumulator row segment.  `tok` / `feat0` are output coordinates of the
// first value; in swap mode the 16 values run over tokens (fixed feature), otherwise
// over features (fixed token).
template <bool kSwapAB>
__device__ __forceinline__ void epi_store(const EpiParams& p, int row_glob, int col0, const float (&v_in)[16],
                                          float* rounded = nullptr) {
  float v[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = v_in[j];
  if (p.scale_w) {
    // FP8: per weight row x per token scales (out-of-range rows / tokens are never stored)
    if (kSwapAB) {
      const float sw = row_glob < p.N ? p.scale_w[row_glob] : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] *= sw * (col0 + j < p.M ? p.scale_x[col0 + j] : 0.f);
    } else {
      const float sx = row_glob < p.M ? p.scale_x[row_glob] : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] *= sx * (col0 + j < p.N ? p.scale_w[col0 + j] : 0.f);
    }
  }
  if (p.epilogue == kEpiSiluMul) {
    // pairs (gate, up) of adjacent weight rows -> one output column
    if (!kSwapAB) {
      const int m = row_glob;
      if (m >= p.M) return;
#pragma unroll
      for (int j = 0; j < 16; j += 2) {
        const int n = col0 + j;
        if (n + 1 < p.N) {
          float g = v[j], u = v[j + 1];
          if (p.bias) {
            g += __bfloat162float(p.bias[n]);
            u += __bfloat162float(p.bias[n + 1]);
          }
          const float s = g / (1.f + __expf(-g));
          p.out[(size_t)m * p.ldo + (n >> 1)] = __float2bfloat16(s * u);
        }
      }
    } else {
      // feature pairs live in adjacent lanes: exchange with the neighbour
      const int n = row_glob;
      const float bn = (p.bias && n < p.N) ? __bfloat162float(p.bias[n]) : 0.f;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float mine = v[j] + bn;
        const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
        const int m = col0 + j;
        if ((n & 1) == 0 && n + 1 < p.N && m < p.M) {
          const float s = mine / (1.f + __expf(-mine));
          p.out[(size_t)m * p.ldo + (n >> 1)] = __float2bfloat16(s * other);
        }
      }
    }
    return;
  }
  if (!kSwapAB) {
    const int m = row_glob;
    if (m >= p.M) return;
    const int n0 = col0;
    if (n0 + 16 <= p.N && (p.ldo & 7) == 0) {
      float t[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) t[j] = v[j];
      if (p.bias) {
        const uint4 b0 = *reinterpret_cast<const uint4*>(p.bias + n0);
        const uint4 b1 = *reinterpret_cast<const uint4*>(p.bias + n0 + 8);
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&b0);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&b1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          t[2 * j] += bf16_lo(q0[j]);
          t[2 * j + 1] += bf16_hi(q0[j]);
          t[8 + 2 * j] += bf16_lo(q1[j]);
          t[8 + 2 * j + 1] += bf16_hi(q1[j]);
        }
      }
      if (p.residual) {
        const uint4 r0 = *reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.ldo + n0);
        const uint4 r1 = *reinterpret_cast<const uint4*>(p.residual + (size_t)m * p.ldo + n0 + 8);
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&r0);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&r1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          t[2 * j] += bf16_lo(q0[j]);
          t[2 * j + 1] += bf16_hi(q0[j]);
          t[8 + 2 * j] += bf16_lo(q1[j]);
          t[8 + 2 * j + 1] += bf16_hi(q1[j]);
        }
      }
      uint4 w0, w1;
      uint32_t* p0 = reinterpret_cast<uint32_t*>(&w0);
      uint32_t* p1 = reinterpret_cast<uint32_t*>(&w1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p0[j] = pack_bf16x2(t[2 * j], t[2 * j + 1]);
        p1[j] = pack_bf16x2(t[8 + 2 * j], t[8 + 2 * j + 1]);
      }
      *reinterpret_cast<uint4*>(p.out + (size_t)m * p.ldo + n0) = w0;
      *reinterpret_cast<uint4*>(p.out + (size_t)m * p.ldo + n0 + 8) = w1;
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int n = n0 + j;
        if (n < p.N) {
          float t = v[j];
          if (p.bias) t += __bfloat162float(p.bias[n]);
          if (p.residual) t += __bfloat162float(p.residual[(size_t)m * p.ldo + n]);
          p.out[(size_t)m * p.ldo + n] = __float2bfloat16(t);
        }
      }
    }
  } else {
    const int n = row_glob;
    if (n >= p.N) return;
    const float bn = p.bias ? __bfloat162float(p.bias[n]) : 0.f;
    // out may alias residual (in-place update): read every residual value before the
    // first store, so the 16 loads are in flight together instead of one per store
    float rv[16];
#pragma unroll
    for (int j = 0; j < 16; ++j)
      rv[j] = (p.residual && col0 + j < p.M) ? __bfloat162float(p.residual[(size_t)(col0 + j) * p.ldo + n]) : 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int m = col0 + j;
      const __nv_bfloat16 o = __float2bfloat16(v[j] + bn + rv[j]);
      if (m < p.M) p.out[(size_t)m * p.ldo + n] = o;
      if (rounded) rounded[j] = m < p.M ? __bfloat162float(o) : 0.f;   // (caller zero-fills)
    }
  }
}

template <int BN, int STAGES, bool kSwapAB>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tc_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        EpiParams ep, float* __restrict__ workspace, uint32_t* __restrict__ tile_counters, int K,
                        int num_a_tiles, int full_tiles, int tail_splits, uint32_t* __restrict__ err) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tmem_full = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  uint32_t* flag_slot = tmem_slot + 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // CTAs [0, full_tiles) compute whole tiles; every later tile is cut into tail_splits
  // K ranges (one CTA each) whose fp32 partials the tile's last CTA sums.  Whole-tile
  // rounds fill the SMs, the split tail fills the last partial round.
  int tile, split, num_splits;
  if ((int)blockIdx.x < full_tiles) {
    tile = blockIdx.x;
    split = 0;
    num_splits = 1;
  } else {
    const int j = blockIdx.x - full_tiles;
    tile = full_tiles + j / tail_splits;
    split = j % tail_splits;
    num_splits = tail_splits;
  }
  const int a_tile = tile % num_a_tiles;
  const int b_tile = tile / num_a_tiles;
  const int total_k_tiles = (K + kBK - 1) / kBK;
  const int k_per_split = (total_k_tiles + num_splits - 1) / num_splits;
  const int kt_begin = split * k_per_split;
  const int kt_end = min(total_k_tiles, kt_begin + k_per_split);
  const int num_k = max(0, kt_end - kt_begin);

  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer
    const uint64_t pol_a = kSwapAB ? policy_evict_first() : policy_evict_last();
    const uint64_t pol_b = kSwapAB ? policy_evict_last() : policy_evict_first();
    pdl_wait();
    int issued = 0;
    for (int i = 0; i < num_k; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      if (!mbar_wait(&empty_bar[s], ph ^ 1, err)) break;
      uint8_t* sa = smem + s * L::kStageBytes;
      uint8_t* sb = sa + L::kABytes;
      const int kc = (kt_begin + i) * kBK;
      mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
      tma_load_2d(sa, &map_a, &full_bar[s], kc, a_tile * kBM, pol_a);
      tma_load_2d(sb, &map_b, &full_bar[s], kc, b_tile * BN, pol_b);
      ++issued;
    }
    // Drain: none of our bulk copies may still be in flight when the CTA exits.
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int j = first; j < issued; ++j) mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(kBM, BN);
    for (int i = 0; i < num_k; ++i) {
      const int s = i % STAGES;
      const uint32_t ph = (i / STAGES) & 1;
      if (!mbar_wait(&full_bar[s], ph, err)) break;
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
      const uint32_t sb = sa + L::kABytes;
      const uint64_t da = make_sw128_desc(sa);
      const uint64_t db = make_sw128_desc(sb);
#pragma unroll
      for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
        // advance 32 B (16 bf16) along K inside the 128 B swizzle row
        umma_f16(tmem_base, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&empty_bar[s]);
    }
    umma_commit(tmem_full);   // always: tells the epilogue every MMA has retired
  } else if (warp >= 2) {
    // ---------------- epilogue (128 threads, one TMEM lane each)
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;   // TMEM lane == MMA row
    pdl_wait();
    const bool ok = mbar_wait(tmem_full, 0, err);
    tc_fence_after();

    // !swap: row -> token, columns -> features;  swap: row -> feature, columns -> tokens
    const int r_glob = a_tile * kBM + row;
    const int c_base = b_tile * BN;
    const uint32_t t_row = tmem_base + ((uint32_t)lane_base << 16);
    const bool direct = (num_splits == 1);
    // partial slots of split tiles: [tile - full_tiles][split][row][BN] fp32, each thread's
    // row contiguous, so the reducing CTA reads 16-byte vectors
    const size_t tail_tile = (size_t)(tile - full_tiles);
    auto slot = [&](int sp) {
      return workspace + ((tail_tile * num_splits + sp) * kBM + row) * (size_t)BN;
    };

#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_row + c0, r);
      tmem_wait_ld();
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (ok && num_k > 0) ? __uint_as_float(r[j]) : 0.f;
      if (direct) {
        epi_store<kSwapAB>(ep, r_glob, c_base + c0, v);
      } else {
        float4* dst = reinterpret_cast<float4*>(slot(split) + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) __stcg(dst + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
      }
    }

    if (!direct) {
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const uint32_t prev = atomicAdd(&tile_counters[tile], 1u);
        *flag_slot = (prev == (uint32_t)(num_splits - 1)) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*flag_slot) {
        __threadfence();
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          // four splits' 64-byte row segments in flight at once, summed in split order
          for (int s0 = 0; s0 < num_splits; s0 += 4) {
            float4 x[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float4* src = reinterpret_cast<const float4*>(slot(s0 + u) + c0);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                x[u][q] = s0 + u < num_splits ? __ldcg(src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                v[4 * q] += x[u][q].x;
                v[4 * q + 1] += x[u][q].y;
                v[4 * q + 2] += x[u][q].z;
                v[4 * q + 3] += x[u][q].w;
              }
          }
          epi_store<kSwapAB>(ep, r_glob, c_base + c0, v);
        }
        if (threadIdx.x == 64) tile_counters[tile] = 0u;   // ready for the next launch
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// =====================================================================================
// Persistent prefill GEMM: one CTA per SM.  CTA c first takes whole 128 x BN output
// tiles in data-parallel rounds (tiles c, c + G, ... below dp_tiles; token block fastest,
// so the CTAs in flight share each weight tile through L2), then its stream-K share of
// the remaining tiles: their k-iterations laid end to end (S = sk_tiles x k_tiles), CTA c
// takes [c S / G, (c + 1) S / G), cut at tile boundaries into segments.  Every CTA has
// the same number of k-iterations (G' <= G CTAs take part, each at least 8 and a
// quarter of a tile's k-iterations, so no tile collects more than a few partials), and a
// GEMM of fewer tiles than SMs (short prompts) still keeps every SM busy.  A tile covered by several segments writes one fp32 partial
// per segment; the last to arrive sums them in segment order (deterministic).  Warp 0
// streams A/B tiles through a STAGES-deep TMA ring that runs across unit boundaries;
// warp 1 issues the MMAs into one of two TMEM accumulators (2 x BN columns); warps 2-5
// drain the other accumulator, so a tile's epilogue overlaps the next one's main loop.
template <int BN, int STAGES>
struct PersistSmem {
  static constexpr int kABytes = kBM * kBK * 2;
  static constexpr int kBBytes = BN * kBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarOffset = STAGES * kStageBytes;
  // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], then tmem slot + flag
  static constexpr int kTotal = kBarOffset + (2 * STAGES + 4) * 8 + 16;
  static constexpr int kAlloc = kTotal + 1024;
};

struct WorkMap {
  int dp_tiles, grid, k_tiles, sk_tiles, sk_grid, max_seg;
  long long sk_work;   // sk_tiles * k_tiles; >= sk_grid whenever sk_tiles > 0 (no empty range)
  // split schedule instead of stream-K (tail_splits > 0): units u = c, c + G, ... below
  // num_units; units past dp_tiles are tail_splits equal K pieces of the remaining tiles
  int tail_splits, num_units;
  __device__ __forceinline__ int n_dp(int c) const { return c < dp_tiles ? (dp_tiles - 1 - c) / grid + 1 : 0; }
  // the CTA whose stream-K range holds k-iteration x: the largest c with c S / G' <= x
  // (G' = sk_grid: CTAs c < G' share the stream-K work)
  __device__ __forceinline__ int owner(long long x) const { return (int)(((x + 1) * sk_grid - 1) / sk_work); }
  // unit i of CTA c: tile, k-range [kb, ke), its segment index / count on the tile and
  // its workspace slot; false past the CTA's last unit
  __device__ __forceinline__ bool get(int c, int i, int& tile, int& kb, int& ke, int& seg, int& nseg,
                                      int& slot) const {
    if (tail_splits > 0) {
      const int u = c + i * grid;
      if (u >= num_units) return false;
      if (u < dp_tiles) {
        tile = u;
        seg = 0;
        nseg = 1;
      } else {
        const int j = u - dp_tiles;
        tile = dp_tiles + j / tail_splits;
        seg = j % tail_splits;
        nseg = tail_splits;
      }
      const int per = (k_tiles + nseg - 1) / nseg;
      kb = seg * per;
      ke = min(k_tiles, kb + per);
      if (ke < kb) ke = kb;
      slot = (tile - dp_tiles) * tail_splits;
      return true;
    }
    const int nd = n_dp(c);
    if (i < nd) {
      tile = c + i * grid;
      kb = 0;
      ke = k_tiles;
      seg = 0;
      nseg = 1;
      slot = 0;
      return true;
    }
    if (sk_tiles <= 0 || c >= sk_grid) return false;
    const long long b = (long long)c * sk_work / sk_grid, e = (long long)(c + 1) * sk_work / sk_grid;
    const long long t0 = b / k_tiles;
    const long long ts = t0 + (i - nd);
    if (ts >= sk_tiles || ts * k_tiles >= e) return false;
    kb = ts == t0 ? (int)(b - t0 * k_tiles) : 0;
    ke = (int)min((long long)k_tiles, e - ts * k_tiles);
    if (kb >= ke) return false;
    tile = dp_tiles + (int)ts;
    const int first = owner(ts * k_tiles), last = owner((ts + 1) * k_tiles - 1);
    seg = c - first;
    nseg = last - first + 1;
    slot = (int)ts * max_seg;
    return true;
  }
};

template <int BN, int STAGES>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_persistent_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                           EpiParams ep, float* __restrict__ workspace, uint32_t* __restrict__ tile_counters, int K,
                           int num_a_tiles, WorkMap wm, uint32_t* __restrict__ err) {
  using L = PersistSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L::kBarOffset);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* acc_full = empty_bar + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  uint32_t* flag_slot = tmem_slot + 1;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = 2 * BN;   // two accumulators

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);   // every epilogue thread arrives after its TMEM reads
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- TMA producer: one ring position per k-tile, across units
    const uint64_t pol_a = policy_evict_last();    // activations: re-read by every weight tile
    const uint64_t pol_b = policy_evict_normal();  // weights: shared by the token blocks in flight
    pdl_wait();
    int it = 0;
    bool failed = false;
    int tile, kb, ke, seg, nseg, slot;
    for (int i = 0; !failed && wm.get(blockIdx.x, i, tile, kb, ke, seg, nseg, slot); ++i) {
      const int a_tile = tile % num_a_tiles, b_tile = tile / num_a_tiles;
      for (int kt = kb; kt < ke; ++kt, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&empty_bar[s], ph ^ 1, err)) {
          failed = true;
          break;
        }
        uint8_t* sa = smem + s * L::kStageBytes;
        mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
        tma_load_2d(sa, &map_a, &full_bar[s], kt * kBK, a_tile * kBM, pol_a);
        tma_load_2d(sa + L::kABytes, &map_b, &full_bar[s], kt * kBK, b_tile * BN, pol_b);
      }
    }
    // none of our bulk copies may still be in flight when the CTA exits
    const int first = it > STAGES ? it - STAGES : 0;
    for (int j = first; j < it; ++j) mbar_wait(&full_bar[j % STAGES], (j / STAGES) & 1, err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(kBM, BN);
    int it = 0, n = 0;
    bool failed = false;
    int tile, kb, ke, seg, nseg, slot;
    for (int i = 0; wm.get(blockIdx.x, i, tile, kb, ke, seg, nseg, slot); ++i, ++n) {
      const int acc = n & 1;
      // the epilogue has read this accumulator's previous tile (first use passes)
      if (!failed && !mbar_wait(&acc_empty[acc], ((n >> 1) & 1) ^ 1, err)) failed = true;
      tc_fence_after();
      const uint32_t d = tmem_base + (uint32_t)(acc * BN);
      for (int kt = kb; kt < ke && !failed; ++kt, ++it) {
        const int s = it % STAGES;
        const uint32_t ph = (it / STAGES) & 1;
        if (!mbar_wait(&full_bar[s], ph, err)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
        const uint64_t da = make_sw128_desc(sa);
        const uint64_t db = make_sw128_desc(sa + L::kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / kUmmaK; ++kk)
          umma_f16(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (kt > kb || kk > 0) ? 1u : 0u);
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&acc_full[acc]);   // always: the epilogue waits for every unit
    }
  } else if (warp >= 2) {
    // ---------------- epilogue (128 threads, one TMEM lane each)
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    pdl_wait();
    int n = 0;
    int tile, kb, ke, seg, nseg, slot;
    for (int i = 0; wm.get(blockIdx.x, i, tile, kb, ke, seg, nseg, slot); ++i, ++n) {
      const int acc = n & 1;
      const bool ok = mbar_wait(&acc_full[acc], (n >> 1) & 1, err);
      tc_fence_after();
      const int a_tile = tile % num_a_tiles, b_tile = tile / num_a_tiles;
      const int r_glob = a_tile * kBM + row;
      const int c_base = b_tile * BN;
      const uint32_t t_row = tmem_base + ((uint32_t)lane_base << 16) + (uint32_t)(acc * BN);
      const bool direct = nseg == 1;
      const bool have = ok && ke > kb;
      float* slot0 = direct ? nullptr : workspace + ((size_t)slot * kBM + row) * (size_t)BN;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r0[16], r1[16];
        tmem_ld_32x32b_x16(t_row + c0, r0);
        tmem_ld_32x32b_x16(t_row + c0 + 16, r1);
        tmem_wait_ld();
        float v0[16], v1[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          v0[j] = have ? __uint_as_float(r0[j]) : 0.f;
          v1[j] = have ? __uint_as_float(r1[j]) : 0.f;
        }
        if (c0 + 32 >= BN) {
          // the accumulator is read: the MMA warp may start the unit after next on it
          tc_fence_before();
          mbar_arrive(&acc_empty[acc]);
        }
        if (direct) {
          epi_store<false>(ep, r_glob, c_base + c0, v0);
          epi_store<false>(ep, r_glob, c_base + c0 + 16, v1);
        } else {
          float4* dst = reinterpret_cast<float4*>(slot0 + (size_t)seg * kBM * BN + c0);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            __stcg(dst + q, make_float4(v0[4 * q], v0[4 * q + 1], v0[4 * q + 2], v0[4 * q + 3]));
            __stcg(dst + 4 + q, make_float4(v1[4 * q], v1[4 * q + 1], v1[4 * q + 2], v1[4 * q + 3]));
          }
        }
      }
      if (!direct) {
        // the tile's last segment to arrive sums every segment's partial in segment order
        __threadfence();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          const uint32_t prev = atomicAdd(&tile_counters[tile], 1u);
          *flag_slot = (prev == (uint32_t)(nseg - 1)) ? 1u : 0u;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const bool last = *flag_slot != 0u;
        asm volatile("bar.sync 1, 128;" ::: "memory");   // flag read before the next unit sets it
        if (last) {
          __threadfence();
#pragma unroll 1
          for (int c0 = 0; c0 < BN; c0 += 16) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) v[j] = 0.f;
            for (int s0 = 0; s0 < nseg; s0 += 4) {
              float4 x[4][4];
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const float4* src = reinterpret_cast<const float4*>(slot0 + (size_t)(s0 + w) * kBM * BN + c0);
#pragma unroll
                for (int q = 0; q < 4; ++q)
                  x[w][q] = s0 + w < nseg ? __ldcg(src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int w = 0; w < 4; ++w)
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                  v[4 * q] += x[w][q].x;
                  v[4 * q + 1] += x[w][q].y;
                  v[4 * q + 2] += x[w][q].z;
                  v[4 * q + 3] += x[w][q].w;
                }
            }
            epi_store<false>(ep, r_glob, c_base + c0, v);
          }
          if (threadIdx.x == 64) tile_counters[tile] = 0u;   // ready for the next launch
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// =====================================================================================
// NVFP4 W4A16 decode GEMM on tcgen05 (swap-AB: 128 weight rows = MMA M, the M <= 128
// tokens = MMA N).  Weights stay 4-bit in HBM: per 128-K stage the producer brings the
// tile's e2m1 codes (row-major [N, K/2] bytes, TMA, 8 KB), its two 512-byte e4m3 scale
// atoms (128 rows x 4 blocks each, bulk copy) and the activation tile (bf16, 128-byte
// swizzle).  Warps 2-5 turn each stage into MMA operands: codes x block scale -> f16
// (exact: an e2m1 value times an e4m3 scale has at most 6 significant bits and lies in
// f16's normal range) into a 128-byte-swizzled K-major tile, and the activations to f16
// in place (saturating, like the warp-MMA W4A16 kernel); warp 1 issues kind::f16 MMAs
// from it.  The 4-bit stream keeps 8-9 KB of weights per stage, so a deep ring (3-8
// stages) keeps HBM busy; two converted tiles let conversion run one stage ahead of the
// MMAs.  Grid = weight tiles x K-splits; the last split of a tile sums the partials in
// split order (deterministic); the per-tensor scale multiplies the sum.
constexpr int kW4KT = 128;                          // K per stage
constexpr int kW4Atom = 512;                        // one scale atom: 128 rows x 4 blocks of 16
template <int BN, int RS>
struct W4Smem {
  static constexpr int kXBytes = BN * kW4KT * 2;    // activations: two 128-byte-swizzled halves
  static constexpr int kQBytes = kBM * kW4KT / 2;   // 8 KB of codes
  static constexpr int kSfBytes = 2 * kW4Atom;
  static constexpr int kStage = kXBytes + kQBytes + kSfBytes;   // a multiple of 1024
  static constexpr int kConv = kBM * kW4KT * 2;     // 32 KB f16 weight tile (two halves)
  static constexpr int kConvOff = RS * kStage;
  static constexpr int kBarOff = kConvOff + 2 * kConv;
  // raw_full[RS], raw_empty[RS], conv_full[2], conv_empty[2], tmem_full; tmem slot, flag
  static constexpr int kTotal = kBarOff + (2 * RS + 5) * 8 + 16;
  static constexpr int kAlloc = kTotal + 1024;
  static_assert(kStage % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
};

__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
  return (1u << 4)                       // D format f32 (A, B format 0 = f16)
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// 4 bytes of e2m1 codes (8 values, low nibble first) -> 4 x f16x2
__device__ __forceinline__ void w4_e2m1x8_to_f16(uint32_t w, uint32_t (&h)[4]) {
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "r"(w));
}
__device__ __forceinline__ uint32_t w4_hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t w4_e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}
__device__ __forceinline__ uint32_t w4_bf16x2_to_f16x2_sat(uint32_t v) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(bf16_hi(v)), "f"(bf16_lo(v)));
  return r;
}
__device__ __forceinline__ void fence_proxy_async_cta() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <int BN, int RS>
__global__ void __launch_bounds__(kGemmThreads, 1)
    nvfp4_tc_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_x,
                    const uint8_t* __restrict__ sf_atoms, const float* __restrict__ gs, EpiParams ep,
                    float* __restrict__ workspace, uint32_t* __restrict__ tile_counters, int k_tiles, int splits,
                    uint32_t* __restrict__ err) {
  using L = W4Smem<BN, RS>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* raw_full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* raw_empty = raw_full + RS;
  uint64_t* conv_full = raw_empty + RS;
  uint64_t* conv_empty = conv_full + 2;
  uint64_t* tmem_full = conv_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_full + 1);
  uint32_t* flag_slot = tmem_slot + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x / splits, split = blockIdx.x % splits;
  const int per = (k_tiles + splits - 1) / splits;
  const int kb = split * per, ke = min(k_tiles, kb + per);
  const int n = max(0, ke - kb);
  constexpr uint32_t kTmemCols = BN < 32 ? 32 : BN;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_x);
    for (int s = 0; s < RS; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 128 + 1);   // the converters read it, the MMAs read its activations
    }
    for (int c = 0; c < 2; ++c) {
      mbar_init(&conv_full[c], 128);
      mbar_init(&conv_empty[c], 1);
    }
    mbar_init(tmem_full, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0 && lane == 0) {
    // ---------------- producer: weights first (they do not depend on the previous kernel)
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int pre = n < RS ? n : RS;
    const uint8_t* sf_tile = sf_atoms + (size_t)tile * (size_t)(k_tiles * 2) * kW4Atom;
    for (int g = 0; g < pre; ++g) {
      uint8_t* st = smem + g * L::kStage;
      const int kt = kb + g;
      mbar_arrive_expect_tx(&raw_full[g], L::kStage);
      tma_load_2d(st + L::kXBytes, &map_q, &raw_full[g], kt * (kW4KT / 2), tile * kBM, pol_w);
      bulk_g2s(st + L::kXBytes + L::kQBytes, sf_tile + (size_t)kt * 2 * kW4Atom, 2 * kW4Atom, &raw_full[g]);
    }
    pdl_wait();
    for (int g = 0; g < pre; ++g) {
      uint8_t* st = smem + g * L::kStage;
      const int kt = kb + g;
      tma_load_2d(st, &map_x, &raw_full[g], kt * kW4KT, 0, pol_x);
      tma_load_2d(st + BN * 128, &map_x, &raw_full[g], kt * kW4KT + 64, 0, pol_x);
    }
    int issued = pre;
    for (int g = pre; g < n; ++g) {
      const int s = g % RS;
      if (!mbar_wait(&raw_empty[s], ((g / RS) & 1) ^ 1, err)) break;
      uint8_t* st = smem + s * L::kStage;
      const int kt = kb + g;
      mbar_arrive_expect_tx(&raw_full[s], L::kStage);
      tma_load_2d(st + L::kXBytes, &map_q, &raw_full[s], kt * (kW4KT / 2), tile * kBM, pol_w);
      bulk_g2s(st + L::kXBytes + L::kQBytes, sf_tile + (size_t)kt * 2 * kW4Atom, 2 * kW4Atom, &raw_full[s]);
      tma_load_2d(st, &map_x, &raw_full[s], kt * kW4KT, 0, pol_x);
      tma_load_2d(st + BN * 128, &map_x, &raw_full[s], kt * kW4KT + 64, 0, pol_x);
      issued = g + 1;
    }
    const int first = issued > RS ? issued - RS : 0;
    for (int j = first; j < issued; ++j) mbar_wait(&raw_full[j % RS], (j / RS) & 1, err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc_f16(kBM, BN);
    for (int i = 0; i < n; ++i) {
      const int s = i % RS, c = i & 1;
      if (!mbar_wait(&conv_full[c], (i >> 1) & 1, err)) break;
      tc_fence_after();
      const uint32_t xa = smem_u32(smem + s * L::kStage);
      const uint32_t ca = smem_u32(smem + L::kConvOff + c * L::kConv);
#pragma unroll
      for (int kk = 0; kk < kW4KT / kUmmaK; ++kk) {
        const int h = kk >> 2;   // 64-K half: its own 128-byte swizzle atom
        const uint64_t da = make_sw128_desc(ca + h * (kBM * 128)) + (uint64_t)((kk & 3) * 2);
        const uint64_t db = make_sw128_desc(xa + h * (BN * 128)) + (uint64_t)((kk & 3) * 2);
        umma_f16(tmem_base, da, db, idesc, (i > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(&raw_empty[s]);
      umma_commit(&conv_empty[c]);
    }
    umma_commit(tmem_full);
  } else if (warp >= 2) {
    const int ct = threadIdx.x - 64;   // 0..127
    // ---------------- converters
    for (int i = 0; i < n; ++i) {
      const int s = i % RS, c = i & 1;
      const bool ok = mbar_wait(&raw_full[s], (i / RS) & 1, err) &&
                      mbar_wait(&conv_empty[c], ((i >> 1) & 1) ^ 1, err);
      uint8_t* st = smem + s * L::kStage;
      uint8_t* cv = smem + L::kConvOff + c * L::kConv;
      if (ok) {
        // activations -> f16 in place (position-independent: the swizzle is unchanged)
        for (int ch = ct; ch < BN * 16; ch += 128) {
          uint4 v = *reinterpret_cast<const uint4*>(st + ch * 16);
          v.x = w4_bf16x2_to_f16x2_sat(v.x);
          v.y = w4_bf16x2_to_f16x2_sat(v.y);
          v.z = w4_bf16x2_to_f16x2_sat(v.z);
          v.w = w4_bf16x2_to_f16x2_sat(v.w);
          *reinterpret_cast<uint4*>(st + ch * 16) = v;
        }
        // weights: item (row r, 16-byte code chunk qc) = 32 values of blocks 2 qc, 2 qc + 1;
        // a warp's 32 items are 8 whole rows (512 contiguous bytes)
        const uint8_t* q = st + L::kXBytes;
        const uint8_t* sf = q + L::kQBytes;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int item = ct + 128 * j;
          const int r = item >> 2, qc = item & 3;
          const uint4 codes = *reinterpret_cast<const uint4*>(q + r * 64 + qc * 16);
          const int h = qc >> 1;
          const uint16_t sc2 =
              *reinterpret_cast<const uint16_t*>(sf + h * kW4Atom + (r & 31) * 16 + ((r >> 5) & 3) * 4 + (qc & 1) * 2);
          const uint32_t sh = w4_e4m3x2_to_f16x2(sc2);          // (scale of block 2 qc, of 2 qc + 1)
          const uint32_t s_lo = __byte_perm(sh, 0, 0x1010), s_hi = __byte_perm(sh, 0, 0x3232);
          const uint32_t words[4] = {codes.x, codes.y, codes.z, codes.w};
          uint8_t* rowbase = cv + h * (kBM * 128) + (r >> 3) * 1024 + (r & 7) * 128;
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            uint32_t hh[4];
            w4_e2m1x8_to_f16(words[u], hh);
            const uint32_t sc = u < 2 ? s_lo : s_hi;
            uint4 o;
            o.x = w4_hmul2(hh[0], sc);
            o.y = w4_hmul2(hh[1], sc);
            o.z = w4_hmul2(hh[2], sc);
            o.w = w4_hmul2(hh[3], sc);
            const int c8 = (qc & 1) * 4 + u;   // 16-byte chunk (8 K) of the 128-byte row
            *reinterpret_cast<uint4*>(rowbase + ((c8 ^ (r & 7)) << 4)) = o;
          }
        }
      }
      fence_proxy_async_cta();   // generic-proxy writes -> visible to the tensor core / TMA
      mbar_arrive(&conv_full[c]);
      mbar_arrive(&raw_empty[s]);
      if (!ok) break;
    }
    // ---------------- epilogue (one TMEM lane = one weight row each)
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    pdl_wait();
    const bool ok = mbar_wait(tmem_full, 0, err);
    tc_fence_after();
    const float g = gs ? *gs : 1.f;
    const int r_glob = tile * kBM + row;
    const uint32_t t_row = tmem_base + ((uint32_t)lane_base << 16);
    const bool direct = splits == 1;
    auto slot = [&](int sp) { return workspace + (((size_t)tile * splits + sp) * kBM + row) * (size_t)BN; };
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_row + c0, r);
      tmem_wait_ld();
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = (ok && n > 0) ? __uint_as_float(r[j]) : 0.f;
      if (direct) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] *= g;
        epi_store<true>(ep, r_glob, c0, v);
      } else {
        float4* dst = reinterpret_cast<float4*>(slot(split) + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) __stcg(dst + q, make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
      }
    }
    if (!direct) {
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        const uint32_t prev = atomicAdd(&tile_counters[tile], 1u);
        *flag_slot = (prev == (uint32_t)(splits - 1)) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*flag_slot) {
        __threadfence();
#pragma unroll 1
        for (int c0 = 0; c0 < BN; c0 += 16) {
          float v[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = 0.f;
          for (int s0 = 0; s0 < splits; s0 += 4) {
            float4 x[4][4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const float4* src = reinterpret_cast<const float4*>(slot(s0 + u) + c0);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                x[u][q] = s0 + u < splits ? __ldcg(src + q) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
            for (int u = 0; u < 4; ++u)
#pragma unroll
              for (int q = 0; q < 4; ++q) {
                v[4 * q] += x[u][q].x;
                v[4 * q + 1] += x[u][q].y;
                v[4 * q + 2] += x[u][q].z;
                v[4 * q + 3] += x[u][q].w;
              }
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] *= g;
          epi_store<true>(ep, r_glob, c0, v);
        }
        if (threadIdx.x == 64) tile_counters[tile] = 0u;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// =====================================================================================
// Stream-K decode GEMM (swap-AB): one persistent CTA per SM.  The iteration space
// tiles x k_tiles (tile = 128 weight rows, k_tile = 64 K elements) is cut into equal
// contiguous ranges, one per CTA, so every SM streams the same number of weight bytes
// whatever the tile count.  A CTA walks its range tile by tile ("segments"); a segment
// that covers a whole tile is stored directly, otherwise its fp32 partial goes to the
// workspace and the last contributor of the tile (tile counter) sums the partials in
// contributor order (deterministic) and runs the epilogue.  Two TMEM accumulators let
// the epilogue of one segment overlap the MMAs of the next.  With programmatic
// dependent launch the producer streams the first STAGES weight tiles before waiting
// for the kernel that produces the activations.
struct StreamK {
  int64_t iters;   // tiles * k_tiles
  int ctas;
  int tiles_x;     // token blocks of BN tokens; tile t = (weight block t / tiles_x, token block t % tiles_x)
  // > 1: ctas == tiles * cluster, each tile's CTAs are one thread-block cluster and the
  // split-tile fixup goes through distributed shared memory (no global partials)
  int cluster;
  __device__ __forceinline__ int64_t start(int c) const { return (int64_t)c * iters / ctas; }
  __device__ __forceinline__ int owner(int64_t i) const {
    int c = (int)(((i + 1) * ctas - 1) / iters);
    if (c >= ctas) c = ctas - 1;
    while (c > 0 && start(c) > i) --c;
    while (c + 1 < ctas && start(c + 1) <= i) ++c;
    return c;
  }
};

// Fused all-reduce, push half (ARPush in vrm_kernels.h): the owner of each finished
// output tile stores the partial (pre-bias, rounded to bf16 like the input of a bf16
// NCCL all-reduce) into this rank's slot on every rank (posted NVLink stores; its own
// slot is local) and never waits.  No fence and no flag: ar_norm.cu polls the values
// themselves (empty pattern 0x8000), so the transfer costs one NVLink write latency.
using ARParams = ARPush;

// Fused reduce of the all-reduce (ARPush::reduce), run by every warp of the push GEMM
// after its own stores: item (token m, 128-feature chunk t); lane l takes 4 features.
__device__ __forceinline__ void ar_reduce_tail(const ARParams& ar, int M, int N, uint32_t* __restrict__ err) {
  const uint32_t epoch = *reinterpret_cast<const volatile uint32_t*>(ar.epoch);
  __nv_bfloat16* half = ar.xbuf[ar.rank] + (size_t)(epoch & 1u) * ar.world * (size_t)ar.half_floats;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  const int parts = (N + 127) / 128;
  const unsigned long long limit = ar.spin_limit ? ar.spin_limit : VRM_SPIN_LIMIT_CYCLES;
  const auto* bias = reinterpret_cast<const __nv_bfloat16*>(ar.bias);
  auto* res = reinterpret_cast<__nv_bfloat16*>(ar.residual);
  const uint2 empty = make_uint2(kBf16EmptyX2, kBf16EmptyX2);
  bool timed_out = false;
  for (int item = blockIdx.x * nw + warp; item < M * parts; item += gridDim.x * nw) {
    const int m = item / parts, t = item - m * parts;
    const int f = t * 128 + lane * 4;
    float q = 0.f;
    if (f < N) {
      __nv_bfloat16* src = half + (size_t)m * N + f;
      uint2 x[8];
#pragma unroll
      for (int p = 0; p < 8; ++p)
        if (p < ar.world) x[p] = ld_relaxed_sys_v2(src + (size_t)p * ar.half_floats);
      const unsigned long long t0 = clock64();
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        if (p >= ar.world) continue;
        while (bf16x4_has_empty(x[p])) {
          if (timed_out || (unsigned long long)(clock64() - t0) > limit) {
            if (!timed_out) report_error(err, kErrFlagTimeout);
            timed_out = true;
            auto z = [](uint32_t w) {
              if ((w & 0xffffu) == kBf16Empty) w &= 0xffff0000u;
              if ((w >> 16) == kBf16Empty) w &= 0x0000ffffu;
              return w;
            };
            x[p] = make_uint2(z(x[p].x), z(x[p].y));
            break;
          }
          x[p] = ld_relaxed_sys_v2(src + (size_t)p * ar.half_floats);
        }
      }
      float v[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        if (p >= ar.world) continue;
        v[0] += bf16_lo(x[p].x); v[1] += bf16_hi(x[p].x); v[2] += bf16_lo(x[p].y); v[3] += bf16_hi(x[p].y);
        *reinterpret_cast<uint2*>(src + (size_t)p * ar.half_floats) = empty;   // free for two calls on
      }
      if (bias) {
        const uint2 b = *reinterpret_cast<const uint2*>(bias + f);
        v[0] += bf16_lo(b.x); v[1] += bf16_hi(b.x); v[2] += bf16_lo(b.y); v[3] += bf16_hi(b.y);
      }
      __nv_bfloat16* rrow = res + (size_t)m * N + f;
      const uint2 r = *reinterpret_cast<const uint2*>(rrow);
      v[0] += bf16_lo(r.x); v[1] += bf16_hi(r.x); v[2] += bf16_lo(r.y); v[3] += bf16_hi(r.y);
      uint2 o;
      o.x = pack_bf16x2(v[0], v[1]);
      o.y = pack_bf16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(rrow) = o;
      // the residual stream is bf16: the norm sums are over the rounded values
      const float a0 = bf16_lo(o.x), a1 = bf16_hi(o.x), a2 = bf16_lo(o.y), a3 = bf16_hi(o.y);
      q = a0 * a0 + a1 * a1 + a2 * a2 + a3 * a3;
    }
    q = warp_sum(q);
    if (lane == 0 && ar.ssq_out != nullptr) ar.ssq_out[(size_t)t * ar.ssq_ld + m] = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t prev;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ar.done) : "memory");
    if (prev == gridDim.x - 1) {
      *ar.done = 0u;
      *reinterpret_cast<volatile uint32_t*>(const_cast<uint32_t*>(ar.epoch)) = epoch + 1u;
    }
  }
}

template <int BN, int STAGES, bool kAR, bool kF8 = false>
__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_streamk_swap_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                             EpiParams ep, float* __restrict__ workspace, uint32_t* __restrict__ tile_counters,
                             int k_tiles, StreamK sk, uint32_t* __restrict__ err,
                             unsigned long long* __restrict__ trace, ARParams ar) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  // barriers: full[STAGES], empty[STAGES], tmem_full[2], tmem_empty[2], drain
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull = empty_bar + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  float* s_ssq = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(tmem_slot) + 16);   // [2][4 warps][16]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x;
  const int64_t it_begin = sk.start(c), it_end = sk.start(c + 1);
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;
  // optional timeline (ns, %globaltimer): [0] entry [1] after setup [2] after pdl_wait
  // [3] first stage ready [4] last MMA issued [5] epilogue done
  unsigned long long* tr = trace ? trace + (size_t)blockIdx.x * 8 : nullptr;
  if (tr && threadIdx.x == 0) tr[0] = globaltimer();

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  if (tr && threadIdx.x == 0) tr[1] = globaltimer();

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    // decode reads every weight tile once (evict first); with several token blocks the
    // next blocks re-read it from L2 (evict normal)
    const uint64_t pol_w = sk.tiles_x > 1 ? policy_evict_normal() : policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    const int total = (int)(it_end - it_begin);
    const int pre = total < STAGES ? total : STAGES;
    // (k, weight block, token block) of the next load, advanced without divisions: the
    // producer is one thread whose per-iteration latency is on the critical path
    const int t0 = (int)(it_begin / k_tiles), k0 = (int)(it_begin - (int64_t)t0 * k_tiles);
    const int tw0 = t0 / sk.tiles_x, tb0 = t0 - tw0 * sk.tiles_x;
    int k = k0, tw = tw0, tb = tb0;
    auto advance = [&](int& kk, int& w, int& b) {
      if (++kk == k_tiles) {
        kk = 0;
        if (++b == sk.tiles_x) {
          b = 0;
          ++w;
        }
      }
    };
    // weights do not depend on the previous kernel: start streaming them first
    for (int g = 0; g < pre; ++g) {
      uint8_t* sa = smem + g * L::kStageBytes;
      mbar_arrive_expect_tx(&full_bar[g], L::kStageBytes);
      tma_load_2d(sa, &map_w, &full_bar[g], k * kBK, tw * kBM, pol_w);
      advance(k, tw, tb);
    }
    pdl_wait();
    if (tr) tr[2] = globaltimer();
    {
      int kx = k0, wx = tw0, bx = tb0;
      for (int g = 0; g < pre; ++g) {
        uint8_t* sb = smem + g * L::kStageBytes + L::kABytes;
        tma_load_2d(sb, &map_x, &full_bar[g], kx * kBK, bx * BN, pol_x);
        advance(kx, wx, bx);
      }
    }
    int issued = pre;
    int s = pre % STAGES;
    uint32_t ph = pre == STAGES ? 1u : 0u;   // phase of stage s's next use
    for (int g = pre; g < total; ++g) {
      if (!mbar_wait(&empty_bar[s], ph ^ 1, err)) break;
      uint8_t* sa = smem + s * L::kStageBytes;
      mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
      tma_load_2d(sa, &map_w, &full_bar[s], k * kBK, tw * kBM, pol_w);
      tma_load_2d(sa + L::kABytes, &map_x, &full_bar[s], k * kBK, tb * BN, pol_x);
      advance(k, tw, tb);
      issued = g + 1;
      if (++s == STAGES) {
        s = 0;
        ph ^= 1u;
      }
    }
    const int first = issued > STAGES ? issued - STAGES : 0;
    for (int j = first; j < issued; ++j) mbar_wait(&full_bar[j % STAGES], (uint32_t)((j / STAGES) & 1), err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = kF8 ? make_idesc_e4m3(kBM, BN) : make_idesc_bf16(kBM, BN);
    int64_t g = 0;
    int ms = 0;              // stage of the next full barrier, and its phase
    uint32_t mphase = 0u;
    int seg = 0;
    bool failed = false;
    for (int64_t it = it_begin; it < it_end && !failed; ++seg) {
      const int k0 = (int)(it % k_tiles);
      const int64_t n = min((int64_t)(k_tiles - k0), it_end - it);
      const int acc = seg & 1;
      if (!mbar_wait(&tempty[acc], (uint32_t)(((seg >> 1) & 1) ^ 1), err)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + (uint32_t)(acc * BN);
      for (int64_t j = 0; j < n; ++j, ++g) {
        const int s = ms;
        const uint32_t mph = mphase;
        if (++ms == STAGES) {
          ms = 0;
          mphase ^= 1u;
        }
        if (!mbar_wait(&full_bar[s], mph, err)) {
          failed = true;
          break;
        }
        if (tr && g == 0) tr[3] = globaltimer();
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
        const uint64_t da = make_sw128_desc(sa);
        const uint64_t db = make_sw128_desc(sa + L::kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
          // bf16: K 16 per MMA; e4m3: K 32 per MMA -- 32 bytes of the swizzle row either way
          if (kF8)
            umma_f8(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (j > 0 || kk > 0) ? 1u : 0u);
          else
            umma_f16(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&empty_bar[s]);
      }
      umma_commit(&tfull[acc]);
      it += n;
    }
    if (tr) tr[4] = globaltimer();
    // every MMA this thread issued must retire before TMEM is freed
    umma_commit(drain);
    mbar_wait(drain, 0, err);
  } else if (warp >= 2) {
    // ---------------- epilogue (16-column chunks: no full accumulator row in registers)
    // Split tiles use a fixed owner: the CTA holding the tile's first k-iteration (the
    // tile is its last segment).  Other contributors (for whom the tile is the first
    // segment) publish fp32 partials; the owner waits for them, so every CTA's waits
    // follow its own segment order, identically on every tensor-parallel rank.
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)lane_base << 16);
    pdl_wait();
    uint32_t epoch = 0;
    if (kAR) epoch = *reinterpret_cast<const volatile uint32_t*>(ar.epoch);
    // folded RMSNorm (consumer): rstd of token lane + 32 i in rs[i] of every epilogue warp
    float rs[4] = {1.f, 1.f, 1.f, 1.f};
    if (ep.ssq_in != nullptr) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int m = lane + 32 * i;
        if (m < ep.M) {
          // eight independent loads per round: a few L2 round trips, not one per part
          float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          int q = 0;
          for (; q + 8 <= ep.ssq_parts; q += 8) {
#pragma unroll
            for (int u = 0; u < 8; ++u) a[u] += ep.ssq_in[(size_t)(q + u) * ep.ssq_ld + m];
          }
          for (; q < ep.ssq_parts; ++q) a[0] += ep.ssq_in[(size_t)q * ep.ssq_ld + m];
          const float sq = ((a[0] + a[1]) + (a[2] + a[3])) + ((a[4] + a[5]) + (a[6] + a[7]));
          rs[i] = rsqrtf(sq / (float)ep.norm_dim + ep.norm_eps);
        }
      }
    }
    int chunk_no = 0;   // parity selects the s_ssq half (one barrier per chunk)
    const bool clm = sk.cluster > 1;
    bool phase1 = false;
    // cluster mode: a contributor's partial, [column][row] fp32, in its (drained) stages
    float* s_part = reinterpret_cast<float*>(smem);
    int seg = 0;
    for (int64_t it = it_begin; it < it_end; ++seg) {
      const int t = (int)(it / k_tiles);
      const int k0 = (int)(it % k_tiles);
      const int64_t n = min((int64_t)(k_tiles - k0), it_end - it);
      const bool whole = (k0 == 0 && n == k_tiles);
      const int acc = seg & 1;
      const int tw = t / sk.tiles_x, tb = t - tw * sk.tiles_x;
      const int r_glob = tw * kBM + row;   // weight row == output feature
      const int tok0 = tb * BN;            // first token of the tile
      int first_owner = c, nc = 1;
      if (!whole) {
        first_owner = sk.owner((int64_t)t * k_tiles);
        nc = sk.owner((int64_t)t * k_tiles + k_tiles - 1) - first_owner + 1;
      }
      const bool is_owner = whole || (c == first_owner);
      // one partial slot per CTA: only a CTA's first segment can be a non-owner partial
      const float* base = workspace + (size_t)first_owner * (size_t)(kBM * BN) + row;
      // this rank's slot in the current half; element (token m, feature n) at m * N + n
      const size_t xoff = kAR ? (((size_t)(epoch & 1u) * ar.world + ar.rank) * ar.half_floats + (size_t)r_glob) : 0;
      // The owner's fixup input does not depend on its own accumulator: wait for the
      // other contributors' partials (published in their first segment) and sum the
      // first 16-column chunk of them while this segment's MMAs are still running, so
      // the tail after the last MMA is the TMEM read, one add and the epilogue.
      float others0[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) others0[j] = 0.f;
      if (is_owner && !whole) {
        if (clm) {
          // phase 1: every contributor of the cluster has its partial in shared memory
          cluster_arrive();
          cluster_wait();
          phase1 = true;
          sum_peers16<BN>(s_part, nc, 0, row, others0);
        } else {
          if (threadIdx.x == 64) {
            const unsigned long long t0 = clock64();
            while (ld_acquire_gpu(tile_counters + t) < (uint32_t)(nc - 1)) {
              if ((unsigned long long)(clock64() - t0) > VRM_SPIN_LIMIT_CYCLES) {
                report_error(err, kErrFlagTimeout);
                break;
              }
            }
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");
          sum_partials16_t<BN>(base, nc, 0, others0);
        }
      }
      const bool ok = mbar_wait(&tfull[acc], (uint32_t)((seg >> 1) & 1), err);
      tc_fence_after();
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_lane + (uint32_t)(acc * BN + c0), r);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = ok ? __uint_as_float(r[j]) : 0.f;
        if (!is_owner) {
          if (clm) {
#pragma unroll
            for (int j = 0; j < 16; ++j) s_part[(c0 + j) * kBM + row] = v[j];
          } else {
            float* slot = workspace + (size_t)c * (size_t)(kBM * BN);
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(slot + (size_t)(c0 + j) * kBM + row, v[j]);
          }
          continue;
        }
        if (!whole) {
          // own contribution + (sum of the others in contributor order)
          float o[16];
          if (c0 == 0) {
#pragma unroll
            for (int j = 0; j < 16; ++j) o[j] = others0[j];
          } else if (clm) {
            sum_peers16<BN>(s_part, nc, c0, row, o);
          } else {
            sum_partials16_t<BN>(base, nc, c0, o);
          }
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += o[j];
        }
        if (kAR) {
          // push the partial into this rank's slot on every rank (own slot is local);
          // e4m3 operands: per weight row x per token scales first
          if (r_glob < ep.N) {
            if (kF8) {
              const float sw = ep.scale_w[r_glob];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] *= sw * (tok0 + c0 + j < ep.M ? ep.scale_x[tok0 + c0 + j] : 0.f);
            }
            uint16_t bits[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) bits[j] = bf16_bits_nonempty(v[j]);
            for (int p = 0; p < ar.world; ++p) {
              __nv_bfloat16* dst = ar.xbuf[p] + xoff;
#pragma unroll
              for (int j = 0; j < 16; ++j)
                if (tok0 + c0 + j < ep.M) st_relaxed_sys_u16(dst + (size_t)(tok0 + c0 + j) * ep.N, bits[j]);
            }
          }
        } else {
          if (ep.ssq_in != nullptr) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = tok0 + c0 + j;   // the same for every lane
              const int i = (m >> 5) & 3;
              const float sel = i == 0 ? rs[0] : i == 1 ? rs[1] : i == 2 ? rs[2] : rs[3];
              v[j] *= __shfl_sync(0xffffffffu, sel, m & 31);
            }
          }
          if (ep.ssq_out == nullptr) {
            epi_store<true>(ep, r_glob, tok0 + c0, v);
          } else {
            // folded RMSNorm (producer): per-token sum of squares of the stored values
            float q[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) q[j] = 0.f;
            epi_store<true>(ep, r_glob, tok0 + c0, v, q);
#pragma unroll
            for (int j = 0; j < 16; ++j) q[j] *= q[j];
            const float part = warp_sum16_scatter(q, lane);
            float* buf = s_ssq + (chunk_no & 1) * 64;
            if ((lane & 1) == 0) buf[(warp & 3) * 16 + ((lane >> 1) & 15)] = part;
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (threadIdx.x >= 64 && threadIdx.x < 80) {
              const int j = threadIdx.x - 64;
              const int m = tok0 + c0 + j;
              const float tot = buf[j] + buf[16 + j] + buf[32 + j] + buf[48 + j];
              if (m < ep.M) ep.ssq_out[(size_t)tw * ep.ssq_ld + m] = tot;
            }
            ++chunk_no;
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (clm) {
        // cluster mode: one segment per CTA, handed over through shared memory
      } else if (!is_owner) {
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          uint32_t prev;
          asm volatile("atom.release.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(tile_counters + t) : "memory");
        }
      } else if (!whole && threadIdx.x == 64) {
        tile_counters[t] = 0u;   // all contributors counted: reset for the next launch
      }
      it += n;
    }
    if (clm) {
      // contributors (and idle CTAs) publish in phase 1; phase 2 keeps every CTA's
      // shared memory alive until its cluster's owner has read it
      if (!phase1) {
        cluster_arrive();
        cluster_wait();
      }
      cluster_arrive();
      cluster_wait();
    }
    if (tr && threadIdx.x == 64) tr[5] = globaltimer();
  }
  if (sk.cluster > 1 && warp < 2) {
    // the producer / MMA warps take part in both cluster phases of the fixup
    cluster_arrive();
    cluster_wait();
    cluster_arrive();
    cluster_wait();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  if (kAR && ar.reduce) ar_reduce_tail(ar, ep.M, ep.N, err);
}

// =====================================================================================
// Grouped (mixture-of-experts) swap-AB GEMM over a device-built work list.  Expert
// weights are one K-major matrix [E * N, K]; the activations of the tokens routed to
// each expert are contiguous rows of x_perm (moe.cu builds both the permutation and the
// list of token blocks: expert, first row, rows).  Work item i = (block i / wtiles,
// weight tile i % wtiles) computes 128 weight rows of that expert against its block of
// <= BN tokens over the full K; persistent CTAs take items round-robin, with double TMEM
// accumulators so one item's epilogue overlaps the next item's MMAs.  Everything the
// CTAs need comes from the device, so the launch has a fixed grid and no host sync.
__device__ __forceinline__ MoeBlock load_block(const MoeBlock* blocks, int i) {
  const int4 v = reinterpret_cast<const int4*>(blocks)[i];
  return MoeBlock{v.x, v.y, v.z, v.w};
}

// Expert-parallel return epilogue: row r of the grouped output belongs to pair
// meta[r] % p_cap of rank meta[r] / p_cap and is stored straight into that rank's
// return buffer (half = epoch parity); the last CTA flags every rank.
struct MoeRet {
  const int* meta = nullptr;                 // this rank's meta buffer (both halves)
  __nv_bfloat16* const* yback = nullptr;     // [world] return buffers
  uint32_t* const* flags = nullptr;          // [world] flag arrays ([3][world])
  const uint32_t* epoch = nullptr;
  uint32_t* done = nullptr;
  int rank = 0, world = 1, p_cap = 0, H = 0;
};

template <int BN, int STAGES, bool kRet>
__global__ void __launch_bounds__(kGemmThreads, 1)
    moe_grouped_swap_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                            EpiParams ep, const MoeBlock* blocks, const int* num_blocks,
                            int n_per_expert, int k_tiles, uint32_t* __restrict__ err, MoeRet ret) {
  using L = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * L::kStageBytes);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull = empty_bar + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr uint32_t kTmemCols = 2 * BN < 32 ? 32 : 2 * BN;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_w);
    tma_prefetch_desc(&map_x);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  pdl_wait_for(blocks, num_blocks);  // the work list and x_perm come from earlier kernels
  const int* ret_meta = ret.meta;
  if (kRet) opaque_after_wait(ret_meta);
  const int wtiles = (n_per_expert + kBM - 1) / kBM;
  const int items = *num_blocks * wtiles;

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    const uint64_t pol_w = policy_evict_first();
    const uint64_t pol_x = policy_evict_last();
    int s = 0;
    uint32_t ph = 0;
    int64_t g = 0;
    bool failed = false;
    for (int i = blockIdx.x; i < items && !failed; i += gridDim.x) {
      const MoeBlock b = load_block(blocks, i / wtiles);
      const int wrow = b.expert * n_per_expert + (i % wtiles) * kBM;
      for (int k = 0; k < k_tiles; ++k, ++g) {
        if (g >= STAGES && !mbar_wait(&empty_bar[s], ph ^ 1u, err)) {
          failed = true;
          break;
        }
        uint8_t* sa = smem + s * L::kStageBytes;
        mbar_arrive_expect_tx(&full_bar[s], L::kStageBytes);
        tma_load_2d(sa, &map_w, &full_bar[s], k * kBK, wrow, pol_w);
        tma_load_2d(sa + L::kABytes, &map_x, &full_bar[s], k * kBK, b.row0, pol_x);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
    }
    // the CTA may not exit while its last loads are in flight
    const int64_t first = g > STAGES ? g - STAGES : 0;
    for (int64_t j = first; j < g; ++j) mbar_wait(&full_bar[j % STAGES], (uint32_t)((j / STAGES) & 1), err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc = make_idesc_bf16(kBM, BN);
    int s = 0;
    uint32_t ph = 0;
    int j = 0;
    bool failed = false;
    for (int i = blockIdx.x; i < items && !failed; i += gridDim.x, ++j) {
      const int acc = j & 1;
      if (!mbar_wait(&tempty[acc], (uint32_t)(((j >> 1) & 1) ^ 1), err)) break;
      tc_fence_after();
      const uint32_t d = tmem_base + (uint32_t)(acc * BN);
      for (int k = 0; k < k_tiles; ++k) {
        if (!mbar_wait(&full_bar[s], ph, err)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * L::kStageBytes);
        const uint64_t da = make_sw128_desc(sa);
        const uint64_t db = make_sw128_desc(sa + L::kABytes);
#pragma unroll
        for (int kk = 0; kk < kBK / kUmmaK; ++kk)
          umma_f16(d, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (k > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty_bar[s]);
        if (++s == STAGES) {
          s = 0;
          ph ^= 1u;
        }
      }
      umma_commit(&tfull[acc]);
    }
    umma_commit(drain);
    mbar_wait(drain, 0, err);
  } else if (warp >= 2) {
    // ---------------- epilogue: rows of TMEM = weight rows (features), columns = tokens
    const int lane_base = 32 * (warp & 3);
    const int row = lane_base + lane;
    const uint32_t t_lane = tmem_base + ((uint32_t)lane_base << 16);
    int j = 0;
    for (int i = blockIdx.x; i < items; i += gridDim.x, ++j) {
      const int acc = j & 1;
      const bool ok = mbar_wait(&tfull[acc], (uint32_t)((j >> 1) & 1), err);
      tc_fence_after();
      const MoeBlock b = load_block(blocks, i / wtiles);
      EpiParams e = ep;
      e.out = ep.out + (size_t)b.row0 * ep.ldo;
      e.M = b.nrows;
      const int r_glob = (i % wtiles) * kBM + row;
#pragma unroll 1
      for (int c0 = 0; c0 < BN; c0 += 16) {
        uint32_t r[16];
        tmem_ld_32x32b_x16(t_lane + (uint32_t)(acc * BN + c0), r);
        tmem_wait_ld();
        float v[16];
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = ok ? __uint_as_float(r[q]) : 0.f;
        if (!kRet) {
          epi_store<true>(e, r_glob, c0, v);
        } else if (r_glob < ep.N) {
          // feature r_glob of up to 16 rows, each to its source rank (lanes: consecutive features)
          const size_t half = (size_t)(*ret.epoch & 1u) * ret.p_cap;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            if (c0 + q >= b.nrows) break;
            const int tag = ret_meta[b.row0 + c0 + q];
            const int src = tag / ret.p_cap, p = tag - src * ret.p_cap;
            ret.yback[src][(half + p) * ret.H + r_glob] = __float2bfloat16(v[q]);
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (!ok) break;
    }
    if (kRet) {
      // every CTA counts itself done once its remote stores are ordered (barrier over
      // the epilogue warps, then one system fence: release is cumulative); the last one
      // flags every rank
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        uint32_t prev;
        asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;" : "=r"(prev) : "l"(ret.done) : "memory");
        if (prev == gridDim.x - 1) {
          *ret.done = 0u;
          asm volatile("fence.acq_rel.sys;" ::: "memory");
          const uint32_t epv = *ret.epoch;
          for (int o = 0; o < ret.world; ++o) st_release_sys(ret.flags[o] + 2 * ret.world + ret.rank, epv);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ---------------------------------------------------------------- host side
namespace {

struct MapKey {
  uint64_t ptr;
  int64_t rows, cols, ld;
  int box_rows;
  int dev;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && cols == o.cols && ld == o.ld && box_rows == o.box_rows && dev == o.dev;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    size_t h = std::hash<uint64_t>()(k.ptr);
    h ^= std::hash<int64_t>()(k.rows * 1315423911ll + k.cols * 2654435761ll + k.ld) + 0x9e3779b9 + (h << 6) + (h >> 2);
    return h ^ (size_t)(k.box_rows * 31 + k.dev);
  }
};

std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_map_cache;

}  // namespace

// K-major bf16 matrix [rows, cols] with row stride ld (elements); box = box_rows x 64.
CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  int dev = 0;
  cudaGetDevice(&dev);
  MapKey key{reinterpret_cast<uint64_t>(ptr), rows, cols, ld, box_rows, dev};
  {
    std::lock_guard<std::mutex> g(g_map_mu);
    auto it = g_map_cache.find(key);
    if (it != g_map_cache.end()) return it->second;
  }
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tensor_map()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VRM_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed (code " + std::to_string((int)r) + ", rows " +
                                     std::to_string(rows) + ", cols " + std::to_string(cols) + ")");
  std::lock_guard<std::mutex> g(g_map_mu);
  if (g_map_cache.size() > 16384) g_map_cache.clear();
  g_map_cache.emplace(key, map);
  return map;
}

// Prefill tiles: 3 stages (96 KB) so two CTAs share an SM and one's epilogue overlaps
// the other's main loop: 10-27% faster than one 6-stage CTA per SM on B200 at M = 512
// and 4096 of the Qwen2.5-14B projections (0.63-0.75 of cuBLAS instead of 0.56-0.65).
// VRM_GEMM_PREFILL_STAGES=6 restores the single-CTA layout.
static int prefill_stages() {
  static const int v = [] {
    const char* e = std::getenv("VRM_GEMM_PREFILL_STAGES");
    return (e && e[0] == '6') ? 6 : 3;
  }();
  return v;
}

template <int BN, int STAGES, bool kSwap>
static void launch_gemm(const CUtensorMap& ma, const CUtensorMap& mb, const EpiParams& ep, int K, int a_tiles,
                        int b_tiles, int full_tiles, int tail_splits, cudaStream_t stream) {
  using L = GemmSmem<BN, STAGES>;
  auto kern = gemm_bf16_tc_kernel<BN, STAGES, kSwap>;
  static int attr_dev_mask = 0;   // per-device "attribute set" bits (devices < 32)
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_dev_mask |= 1 << (dev & 31);
  }
  const int tiles = a_tiles * b_tiles;
  if (tail_splits <= 1) full_tiles = tiles;
  float* ws = nullptr;
  uint32_t* counters = nullptr;
  if (full_tiles < tiles) {
    const size_t need = (size_t)(tiles - full_tiles) * tail_splits * kBM * BN * sizeof(float);
    ws = static_cast<float*>(workspace_get(need, stream));
    VRM_REQUIRE((size_t)tiles <= 32768, "too many split-K tiles");
    counters = tile_counters_get(stream);
  }
  dim3 grid(full_tiles + (tiles - full_tiles) * std::max(1, tail_splits));
  launch_kernel(kern, grid, dim3(kGemmThreads), (size_t)L::kAlloc, stream, ma, mb, ep, ws, counters, K, a_tiles,
                full_tiles, tail_splits, error_word());
}

// Whole tiles for the complete rounds over the SMs, the remaining tiles split K-wise so
// the last round is filled: minimises rounds + (split cost) over the split count.
static void choose_tail_split(int tiles, int k_tiles, int min_k, int* full_tiles, int* tail_splits) {
  const int sms = device_sm_count();
  *full_tiles = tiles;
  *tail_splits = 1;
  const int rounds = tiles / sms, rem = tiles % sms;
  if (rem == 0) return;
  // cost in tile units.  A split tail tile also pays for writing and reducing its
  // partials; measured on B200 at about 12.8 / k_tiles tile per split (0.16 at K = 5120,
  // 0.06 at K = 13824), so only long-K tiles gain from splitting.
  double best = rounds + 1.0;
  const int full = rounds * sms;
  const double per_split = 12.8 / k_tiles;
  for (int sp = 2; sp <= 16 && k_tiles / sp >= min_k; ++sp) {
    const int pieces = rem * sp;
    const double cost = rounds + std::ceil((double)pieces / sms) / sp + per_split * sp;
    if (cost < best - 1e-9) {
      best = cost;
      *full_tiles = full;
      *tail_splits = sp;
    }
  }
}

// debug timeline buffer for the stream-K kernel (set by gemm_set_trace, null = off)
static unsigned long long* g_gemm_trace = nullptr;
void gemm_set_trace(void* buf) { g_gemm_trace = static_cast<unsigned long long*>(buf); }

template <int BN, int STAGES, bool kAR, bool kF8 = false>
static void launch_streamk(const CUtensorMap& mw, const CUtensorMap& mx, const EpiParams& ep, int N, int K,
                           int max_ctas, cudaStream_t stream, const ARParams& ar, int tiles_x = 1) {
  // smem: stages + 2*STAGES+4 barriers + slots.  K counts bf16 elements (for e4m3
  // operands: pairs of bytes, so that one K-tile is the same 128-byte swizzle row)
  constexpr int kSmem = STAGES * GemmSmem<BN, STAGES>::kStageBytes + (2 * STAGES + 5) * 8 + 16 + 512 + 1024;
  auto kern = gemm_streamk_swap_kernel<BN, STAGES, kAR, kF8>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr_dev_mask |= 1 << (dev & 31);
  }
  const int tiles = ((N + kBM - 1) / kBM) * tiles_x;
  const int k_tiles = (K + kBK - 1) / kBK;
  StreamK sk;
  sk.tiles_x = tiles_x;
  sk.iters = (int64_t)tiles * k_tiles;
  sk.ctas = (int)std::min<int64_t>(max_ctas, sk.iters);
  uint32_t* counters = tile_counters_get(stream);
  VRM_REQUIRE(tiles <= 32768, "stream-K: too many tiles");
  float* ws = static_cast<float*>(workspace_get((size_t)sk.ctas * kBM * BN * sizeof(float), stream));
  if (kAR) VRM_REQUIRE((long long)ep.M * N <= ar.half_floats, "fused all-reduce: output larger than the symmetric buffer");
  if (kAR && ar.reduce) {
    // every CTA polls data other CTAs of the launch produce: the whole grid must be
    // resident at once (two CTAs per SM fit by registers and shared memory, BN <= 128)
    VRM_REQUIRE(BN <= 128 && sk.ctas <= 2 * device_sm_count(), "fused reduce: grid larger than one resident wave");
    VRM_REQUIRE(ar.world >= 1 && ar.world <= 8 && N % 4 == 0 && ar.residual && ar.done,
                "fused reduce: world <= 8, N % 4 == 0, residual and completion counter required");
  }
  // a tile split evenly over k CTAs (k = 2..8) fixes up inside a thread-block cluster
  static const bool cluster_on = [] {
    const char* e = std::getenv("VRM_GEMM_CLUSTER");
    return !(e && e[0] == '0');
  }();
  const int k = sk.ctas % tiles == 0 ? sk.ctas / tiles : 0;
  sk.cluster = (cluster_on && k >= 2 && k <= 8 && k <= k_tiles) ? k : 0;
  if (sk.cluster > 1)
    launch_kernel_cluster(kern, dim3(sk.ctas), dim3(kGemmThreads), dim3(sk.cluster, 1, 1), (size_t)kSmem, stream,
                          mw, mx, ep, ws, counters, k_tiles, sk, error_word(), g_gemm_trace, ar);
  else
    launch_kernel(kern, dim3(sk.ctas), dim3(kGemmThreads), (size_t)kSmem, stream, mw, mx, ep, ws, counters,
                  k_tiles, sk, error_word(), g_gemm_trace, ar);
}

// Split count such that tiles * splits covers the SMs with >= min_k K-tiles per split.
static void choose_split(int tiles, int k_tiles, int min_k, int* splits, int* ktps) {
  const int sms = device_sm_count();
  int s = 1;
  if (tiles < sms) {
    s = (sms + tiles - 1) / tiles;
    s = std::min(s, std::max(1, k_tiles / min_k));
  }
  int per = (k_tiles + s - 1) / s;
  s = (k_tiles + per - 1) / per;
  *splits = s;
  *ktps = per;
}

// VRM_GEMM_PREFILL=streamk runs M > 128 on the stream-K swap kernel (default: the tiled
// kernel, whose concurrent CTAs share each weight tile in L2; stream-K walks a weight
// tile's token blocks one after another and re-reads it from HBM once it is evicted)
// 0: tiled kernel, 1: stream-K with 128-token tiles, 2: stream-K with 256-token tiles
// (MMA 128 x 256, four 48 KB stages, 512 TMEM columns: one CTA per SM)
// 0 automatic (tiled, or the 256-wide persistent kernel where it was measured faster),
// 1 stream-K, 2 stream-K with 256-token tiles, 3 persistent, 4 persistent with 256-wide
// weight tiles, 5 tiled only; VRM_GEMM_PREFILL or gemm_set_prefill_mode
static int g_prefill_mode = -1;
void gemm_set_prefill_mode(int mode) { g_prefill_mode = mode; }
static int prefill_mode() {
  if (g_prefill_mode < 0) {
    const char* e = std::getenv("VRM_GEMM_PREFILL");
    const std::string m(e ? e : "");
    g_prefill_mode = m == "streamk256" ? 2 : m == "streamk" ? 1 : m == "persistent" ? 3 : m == "persistent256" ? 4
                   : m == "tiled" ? 5 : 0;
  }
  return g_prefill_mode;
}
static bool prefill_streamk() { return prefill_mode() == 1 || prefill_mode() == 2; }

// Persistent prefill GEMM (gemm_persistent_kernel): whole tiles for the complete rounds
// over the SMs, the remaining tiles stream-K (WorkMap), one CTA per SM.
static int persist_splits_env() {
  static const int v = [] {
    const char* e = std::getenv("VRM_GEMM_PERSIST_SPLITS");
    return e ? std::atoi(e) : 0;
  }();
  return v;
}

static int persist_sk_env() {
  static const int v = [] {
    const char* e = std::getenv("VRM_GEMM_PERSIST_SK");
    return e && e[0] ? (e[0] == '1' ? 1 : 0) : -1;
  }();
  return v;
}

template <int BN, int STAGES>
static void launch_persistent(const CUtensorMap& ma, const CUtensorMap& mb, const EpiParams& ep, int K,
                              int a_tiles, int b_tiles, cudaStream_t stream) {
  using L = PersistSmem<BN, STAGES>;
  auto kern = gemm_persistent_kernel<BN, STAGES>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_dev_mask |= 1 << (dev & 31);
  }
  const int tiles = a_tiles * b_tiles;
  const int k_tiles = (K + kBK - 1) / kBK;
  const int sms = device_sm_count();
  // Two schedules for the tiles left after the whole-tile rounds.  Split: each split into
  // equal K pieces (choose_tail_split), pieces dealt round-robin.  Stream-K: their
  // k-iterations shared evenly by G' CTAs, each taking at least max(8, k_tiles / 4) (when
  // that leaves no more CTAs than remaining tiles, the remainder stays whole).
  // Split is the default: it measured faster at every Qwen2.5-14B projection and prompt
  // length tried (M 512-4096; stream-K 2 % slower at M = 4096, up to 1.9x at M = 512,
  // where every tile collects partials); VRM_GEMM_PERSIST_SK=1 selects stream-K.
  WorkMap wm{};
  wm.k_tiles = k_tiles;
  const bool use_sk = persist_sk_env() == 1;
  if (!use_sk) {
    int full = tiles, tail_splits = 1;
    choose_tail_split(tiles, k_tiles, 8, &full, &tail_splits);
    const int forced = persist_splits_env();   // tuning: split the remainder this many ways
    if (forced > 1 && tiles % sms != 0) {
      full = (tiles / sms) * sms;
      tail_splits = std::min(forced, std::max(1, k_tiles / 8));
    }
    if (tail_splits <= 1) full = tiles;
    wm.dp_tiles = full;
    wm.tail_splits = std::max(1, tail_splits);
    wm.num_units = full + (tiles - full) * wm.tail_splits;
    wm.grid = std::min(wm.num_units, sms);
    float* ws = nullptr;
    uint32_t* counters = nullptr;
    if (full < tiles) {
      ws = static_cast<float*>(workspace_get((size_t)(tiles - full) * wm.tail_splits * kBM * BN * sizeof(float),
                                             stream));
      VRM_REQUIRE((size_t)tiles <= 32768, "too many split-K tiles");
      counters = tile_counters_get(stream);
    }
    launch_kernel(kern, dim3(wm.grid), dim3(kGemmThreads), (size_t)L::kAlloc, stream, ma, mb, ep, ws, counters, K,
                  a_tiles, wm, error_word());
    return;
  }
  wm.dp_tiles = (tiles / sms) * sms;
  wm.sk_tiles = tiles - wm.dp_tiles;
  wm.sk_work = (long long)wm.sk_tiles * k_tiles;
  const long long min_share = std::max(8, (k_tiles + 3) / 4);
  wm.sk_grid = (int)std::min<long long>(sms, wm.sk_work / min_share);
  if (wm.sk_tiles == 0 || wm.sk_grid <= wm.sk_tiles) {
    wm.dp_tiles = tiles;
    wm.sk_tiles = 0;
    wm.sk_work = 0;
    wm.sk_grid = 0;
  }
  wm.grid = wm.sk_tiles > 0 ? (wm.dp_tiles > 0 ? sms : wm.sk_grid) : std::min(tiles, sms);
  float* ws = nullptr;
  uint32_t* counters = nullptr;
  if (wm.sk_tiles > 0) {
    // segments per tile <= k_tiles / (shortest CTA share) + 2
    wm.max_seg = (int)(k_tiles / (wm.sk_work / wm.sk_grid)) + 2;
    ws = static_cast<float*>(
        workspace_get((size_t)wm.sk_tiles * wm.max_seg * kBM * BN * sizeof(float), stream));
    VRM_REQUIRE((size_t)tiles <= 32768, "too many split-K tiles");
    counters = tile_counters_get(stream);
  }
  launch_kernel(kern, dim3(wm.grid), dim3(kGemmThreads), (size_t)L::kAlloc, stream, ma, mb, ep, ws, counters, K,
                a_tiles, wm, error_word());
}

// Persistent CTAs of the stream-K decode GEMM.  Latency model fitted on B200 (µs): a
// CTA streams its share of the weights at ~80 GB/s; tiles shared by nc CTAs add ~1 µs
// plus ~0.6 µs per batch of four partials per 16-column chunk for the owner's fixup.
// Short-K GEMMs (the tensor-parallel shards) then run fastest on one CTA per tile, long
// ones on every SM.  VRM_GEMM_CTAS overrides (tuning).
static int streamk_ctas(int tiles, int k_tiles, int BN, double weight_bytes) {
  static const int env = [] {
    const char* e = std::getenv("VRM_GEMM_CTAS");
    return e ? std::atoi(e) : 0;
  }();
  const int sms = device_sm_count();
  if (env > 0) return std::min(env, sms);
  static const bool cluster_on = [] {
    const char* e = std::getenv("VRM_GEMM_CLUSTER");
    return !(e && e[0] == '0');
  }();
  auto cost = [&](int ctas) {
    const int64_t iters = (int64_t)tiles * k_tiles;
    ctas = (int)std::min<int64_t>(ctas, iters);
    const double per_cta = weight_bytes / ctas;
    const int nc = (ctas + tiles - 1) / tiles;
    double t = per_cta / 80e3;
    const bool aligned = ctas % tiles == 0 && nc <= 8 && nc <= k_tiles;
    if (ctas > tiles || nc > 1) {
      // global fixup: the owner sums partials from L2, two per round; cluster fixup
      // (aligned splits): from its peers' shared memory, four per round.  Refitted on
      // B200: at K = 640 (10 k-tiles) two-CTA clusters lost to whole tiles (8.5 vs 7.5 us
      // at M = 32, N = 5120), at K = 5120 / 1728 they won (11.7 vs 13.3, 10.3 vs 11.3 us)
      t += (aligned && cluster_on) ? 0.9 + 0.3 * ((nc - 1 + 3) / 4) * (BN / 16)
                                   : 1.0 + 0.6 * ((nc - 1 + 3) / 4) * (BN / 16);
    }
    return t;
  };
  int best = sms;
  double best_t = cost(sms);
  for (int k = 1; k <= 8 && tiles * k <= sms; ++k) {
    const double t = cost(tiles * k);
    if (t < best_t - 1e-9) {
      best_t = t;
      best = tiles * k;
    }
  }
  return best;
}

static bool legacy_decode() {
  static const bool v = [] {
    const char* e = std::getenv("VRM_GEMM_LEGACY_DECODE");
    return e && e[0] == '1';
  }();
  return v;
}

static void force_split(int force, int k_tiles, int* splits, int* ktps) {
  int s = std::max(1, std::min(force, k_tiles));
  int per = (k_tiles + s - 1) / s;
  *splits = (k_tiles + per - 1) / per;
  *ktps = per;
}

void gemm_bf16(const GemmArgs& a, cudaStream_t stream) {
  VRM_REQUIRE(a.K % 8 == 0 && a.ldx % 8 == 0 && a.ldw % 8 == 0, "gemm: K and row strides must be multiples of 8");
  VRM_REQUIRE((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0,
              "gemm: operands must be 16-byte aligned");
  VRM_REQUIRE(a.epilogue != kEpiSiluMul || (a.N % 2 == 0 && a.residual == nullptr), "gemm: silu_mul epilogue");
  VRM_REQUIRE(!a.allreduce || (a.epilogue == kEpiNone && !a.bias && !a.residual),
              "gemm: the all-reduce push stores the raw partial (bias / residual go to ar_norm)");
  if (a.M <= 0 || a.N <= 0) return;
  EpiParams ep;
  ep.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  ep.ldo = (int)a.ldo;
  ep.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  ep.residual = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  ep.M = a.M;
  ep.N = a.N;
  ep.epilogue = a.epilogue;
  ep.scale_w = nullptr;
  ep.scale_x = nullptr;
  ep.ssq_out = a.ssq_out;
  ep.ssq_in = a.ssq_in;
  ep.ssq_ld = a.ssq_ld;
  ep.ssq_parts = a.ssq_parts;
  ep.norm_dim = a.norm_dim;
  ep.norm_eps = a.norm_eps;
  const int k_tiles = (a.K + kBK - 1) / kBK;
  if (a.ssq_out || a.ssq_in) {
    VRM_REQUIRE(a.M <= 128 && a.M <= a.ssq_ld && a.force_splits <= 0 && !legacy_decode() && !a.allreduce,
                "gemm: the folded RMSNorm runs on the stream-K decode path (M <= 128) only");
    VRM_REQUIRE(!a.ssq_out || (a.residual != nullptr && a.epilogue == kEpiNone &&
                               (a.N + kBM - 1) / kBM <= a.ssq_parts_cap),
                "gemm: norm sums come from a residual epilogue, one slot per weight tile");
    VRM_REQUIRE(!a.ssq_in || (a.ssq_parts > 0 && a.norm_dim > 0), "gemm: folded norm needs its sums");
  }

  if (a.M <= 128) {
    // decode: swap A/B so the weight rows fill the 128 TMEM lanes; stream-K schedule
    const int BN = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : 128;
    const CUtensorMap ma = make_kmajor_map(a.w, a.N, a.K, a.ldw, kBM);
    const CUtensorMap mb = make_kmajor_map(a.x, a.M, a.K, a.ldx, BN);
    VRM_REQUIRE(!a.allreduce || (a.force_splits <= 0 && !legacy_decode()),
                "fused all-reduce runs on the stream-K decode path only");
    if (a.force_splits <= 0 && !legacy_decode()) {
      const int ctas = streamk_ctas((a.N + kBM - 1) / kBM, k_tiles, BN, 2.0 * a.N * a.K);
      // <= 113 KB of smem per CTA: a CTA of the next GEMM fits beside it and (PDL)
      // prefetches its weights while this one drains
      const ARParams ar = a.allreduce ? *a.allreduce : ARParams{};
      if (a.allreduce) {
        switch (BN) {
          case 16: launch_streamk<16, 6, true>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          case 32: launch_streamk<32, 5, true>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          case 64: launch_streamk<64, 4, true>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          default: launch_streamk<128, 3, true>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
        }
      } else {
        switch (BN) {
          case 16: launch_streamk<16, 6, false>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          case 32: launch_streamk<32, 5, false>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          case 64: launch_streamk<64, 4, false>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
          default: launch_streamk<128, 3, false>(ma, mb, ep, a.N, a.K, ctas, stream, ar); break;
        }
      }
      return;
    }
    const int a_tiles = (a.N + kBM - 1) / kBM;
    int splits, ktps;
    choose_split(a_tiles, k_tiles, 4, &splits, &ktps);
    if (a.force_splits > 0) force_split(a.force_splits, k_tiles, &splits, &ktps);
    switch (BN) {   // every tile split `splits` ways (full_tiles = 0)
      case 16: launch_gemm<16, 8, true>(ma, mb, ep, a.K, a_tiles, 1, 0, splits, stream); break;
      case 32: launch_gemm<32, 8, true>(ma, mb, ep, a.K, a_tiles, 1, 0, splits, stream); break;
      case 64: launch_gemm<64, 6, true>(ma, mb, ep, a.K, a_tiles, 1, 0, splits, stream); break;
      default: launch_gemm<128, 5, true>(ma, mb, ep, a.K, a_tiles, 1, 0, splits, stream); break;
    }
  } else if (prefill_streamk() && a.M <= 4096 && a.force_splits <= 0) {
    // prefill: the same swap-AB stream-K kernel over ceil(M / 128) token blocks per
    // weight block (every SM gets the same number of k-iterations: no partial last
    // wave), six stages of 32 KB, one CTA per SM
    VRM_REQUIRE(!a.allreduce, "fused all-reduce needs M <= 128 (decode); use the collective for prefill");
    const CUtensorMap ma = make_kmajor_map(a.w, a.N, a.K, a.ldw, kBM);
    if (prefill_mode() == 2) {
      const CUtensorMap mb = make_kmajor_map(a.x, a.M, a.K, a.ldx, 256);
      launch_streamk<256, 4, false>(ma, mb, ep, a.N, a.K, device_sm_count(), stream, ARParams{}, (a.M + 255) / 256);
    } else {
      const CUtensorMap mb = make_kmajor_map(a.x, a.M, a.K, a.ldx, 128);
      launch_streamk<128, 6, false>(ma, mb, ep, a.N, a.K, device_sm_count(), stream, ARParams{}, (a.M + 127) / 128);
    }
  } else {
    VRM_REQUIRE(!a.allreduce, "fused all-reduce needs M <= 128 (decode); use the collective for prefill");
    constexpr int BN = 128;
    const int a_tiles = (a.M + kBM - 1) / kBM;
    const int b_tiles = (a.N + BN - 1) / BN;
    int full = a_tiles * b_tiles, tail_splits = 1;
    if (a.force_splits > 0) {
      int ktps;
      force_split(a.force_splits, k_tiles, &tail_splits, &ktps);
      full = 0;
    } else if (a_tiles * b_tiles * 2 <= device_sm_count()) {
      int ktps;
      choose_split(a_tiles * b_tiles, k_tiles, 8, &tail_splits, &ktps);
      full = 0;
    } else {
      choose_tail_split(a_tiles * b_tiles, k_tiles, 8, &full, &tail_splits);
    }
    const CUtensorMap ma = make_kmajor_map(a.x, a.M, a.K, a.ldx, kBM);
    // default (mode 0): the persistent kernel with 256-wide weight tiles (split-tail
    // schedule) for every prompt of 512+ tokens -- measured on B200 at M = 512 / 1024 /
    // 2048 / 4096 over the Qwen2.5-14B projections it beats the tiled kernel everywhere
    // (e.g. o 5120 x 5120: 37.6 vs 49.4, 72.4 vs 85.4, 106.9 vs 124.5, 186.7 vs 190.0 us)
    // except a long K over at most 4 token blocks (down 5120 x 13824 at M = 512: 80
    // tiles leave 68 SMs idle, 110.3 vs 85.7 us), which stays tiled
    const bool auto_persist = prefill_mode() == 0 && a.force_splits <= 0 && a.N % 256 == 0 && a.M >= 512 &&
                              !(a_tiles <= 4 && a.K >= 8192);
    if (auto_persist) {
      const CUtensorMap mb = make_kmajor_map(a.w, a.N, a.K, a.ldw, 256);
      launch_persistent<256, 4>(ma, mb, ep, a.K, a_tiles, a.N / 256, stream);
      return;
    }
    if ((prefill_mode() == 3 || prefill_mode() == 4) && a.force_splits <= 0) {
      if (prefill_mode() == 4 && a.N % 256 == 0) {
        const CUtensorMap mb = make_kmajor_map(a.w, a.N, a.K, a.ldw, 256);
        launch_persistent<256, 4>(ma, mb, ep, a.K, a_tiles, a.N / 256, stream);
      } else {
        const CUtensorMap mb = make_kmajor_map(a.w, a.N, a.K, a.ldw, BN);
        launch_persistent<128, 6>(ma, mb, ep, a.K, a_tiles, b_tiles, stream);
      }
      return;
    }
    const CUtensorMap mb = make_kmajor_map(a.w, a.N, a.K, a.ldw, BN);
    if (prefill_stages() == 3)   // two CTAs per SM: one's epilogue overlaps the other's main loop
      launch_gemm<BN, 3, false>(ma, mb, ep, a.K, a_tiles, b_tiles, full, tail_splits, stream);
    else
      launch_gemm<BN, 6, false>(ma, mb, ep, a.K, a_tiles, b_tiles, full, tail_splits, stream);
  }
}


// ---------------------------------------------------------------- FP8 (e4m3) W8A8
// The stream-K swap kernel with kind::f8f6f4 MMAs.  The e4m3 operands are described to
// TMA as bf16 pairs, so one K-tile is still a 128-byte swizzle row (128 elements) and
// every address, box and descriptor step is the bf16 one; the epilogue scales by
// scale_w[n] * scale_x[m].  Any M: token blocks of 128 beyond the first.
// ---------------------------------------------------------------- NVFP4 W4A16 decode (tcgen05)
// uint8 [rows, cols] row-major, box 64 bytes x 128 rows, no swizzle (the converters read
// whole 16-byte chunks of a row)
static CUtensorMap make_u8_rows_map(const void* ptr, int64_t rows, int64_t cols) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)(kW4KT / 2), (cuuint32_t)kBM};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tensor_map()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VRM_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (nvfp4 codes) failed (code " + std::to_string((int)r) + ")");
  return map;
}

template <int BN, int RS>
static void launch_nvfp4_tc(const CUtensorMap& mq, const CUtensorMap& mx, const uint8_t* sf, const float* gs,
                            const EpiParams& ep, int a_tiles, int k_tiles, int splits, cudaStream_t stream) {
  using L = W4Smem<BN, RS>;
  auto kern = nvfp4_tc_kernel<BN, RS>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kAlloc));
    attr_dev_mask |= 1 << (dev & 31);
  }
  float* ws = nullptr;
  uint32_t* counters = nullptr;
  if (splits > 1) {
    ws = static_cast<float*>(workspace_get((size_t)a_tiles * splits * kBM * BN * sizeof(float), stream));
    VRM_REQUIRE((size_t)a_tiles <= 32768, "too many split-K tiles");
    counters = tile_counters_get(stream);
  }
  launch_kernel(kern, dim3(a_tiles * splits), dim3(kGemmThreads), (size_t)L::kAlloc, stream, mq, mx, sf, gs, ep, ws,
                counters, k_tiles, splits, error_word());
}

void nvfp4_tc_gemm(const Nvfp4TcArgs& a, cudaStream_t stream) {
  VRM_REQUIRE(a.M >= 1 && a.M <= 128, "nvfp4 tcgen05 decode gemm: 1 <= M <= 128");
  VRM_REQUIRE(a.N % kBM == 0 && a.K % kW4KT == 0, "nvfp4 tcgen05 decode gemm: N % 128 and K % 128");
  VRM_REQUIRE(a.ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.q_rows) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.sf) & 15) == 0,
              "nvfp4 tcgen05 decode gemm: 16-byte aligned operands");
  VRM_REQUIRE(a.epilogue != kEpiSiluMul || (a.N % 2 == 0 && a.residual == nullptr), "nvfp4 gemm: silu_mul epilogue");
  EpiParams ep;
  ep.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  ep.ldo = (int)a.ldo;
  ep.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  ep.residual = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  ep.M = a.M;
  ep.N = a.N;
  ep.epilogue = a.epilogue;
  ep.scale_w = nullptr;
  ep.scale_x = nullptr;
  const int a_tiles = a.N / kBM, k_tiles = a.K / kW4KT;
  int splits, ktps;
  choose_split(a_tiles, k_tiles, 2, &splits, &ktps);
  const int BN = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : 128;
  const CUtensorMap mq = make_u8_rows_map(a.q_rows, a.N, a.K / 2);
  const CUtensorMap mx = make_kmajor_map(a.x, a.M, a.K, a.ldx, BN);
  switch (BN) {
    case 16: launch_nvfp4_tc<16, 8>(mq, mx, a.sf, a.gs, ep, a_tiles, k_tiles, splits, stream); break;
    case 32: launch_nvfp4_tc<32, 7>(mq, mx, a.sf, a.gs, ep, a_tiles, k_tiles, splits, stream); break;
    case 64: launch_nvfp4_tc<64, 5>(mq, mx, a.sf, a.gs, ep, a_tiles, k_tiles, splits, stream); break;
    default: launch_nvfp4_tc<128, 3>(mq, mx, a.sf, a.gs, ep, a_tiles, k_tiles, splits, stream); break;
  }
}

void gemm_fp8(const GemmArgs& a, const float* scale_x, const float* scale_w, cudaStream_t stream) {
  VRM_REQUIRE(a.K % 128 == 0 && a.ldx % 16 == 0 && a.ldw % 16 == 0, "gemm fp8: K % 128, row strides % 16 bytes");
  VRM_REQUIRE((reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0,
              "gemm fp8: operands must be 16-byte aligned");
  VRM_REQUIRE(scale_x && scale_w, "gemm fp8: scales required");
  VRM_REQUIRE(!a.allreduce || (a.M <= 128 && a.epilogue == kEpiNone && !a.bias && !a.residual),
              "gemm fp8: the all-reduce push stores the raw partial of a decode GEMM (M <= 128)");
  VRM_REQUIRE(a.epilogue != kEpiSiluMul || (a.N % 2 == 0 && a.residual == nullptr), "gemm fp8: silu_mul epilogue");
  if (a.M <= 0 || a.N <= 0) return;
  EpiParams ep;
  ep.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  ep.ldo = (int)a.ldo;
  ep.bias = reinterpret_cast<const __nv_bfloat16*>(a.bias);
  ep.residual = reinterpret_cast<const __nv_bfloat16*>(a.residual);
  ep.M = a.M;
  ep.N = a.N;
  ep.epilogue = a.epilogue;
  ep.scale_w = scale_w;
  ep.scale_x = scale_x;
  const int64_t Kp = a.K / 2;                               // bf16-pair units
  const int k_tiles = (int)((Kp + kBK - 1) / kBK);
  const CUtensorMap ma = make_kmajor_map(a.w, a.N, Kp, a.ldw / 2, kBM);
  const int n_tiles = (a.N + kBM - 1) / kBM;
  if (a.M <= 128) {
    const int BN = a.M <= 16 ? 16 : a.M <= 32 ? 32 : a.M <= 64 ? 64 : 128;
    const CUtensorMap mb = make_kmajor_map(a.x, a.M, Kp, a.ldx / 2, BN);
    const int ctas = streamk_ctas(n_tiles, k_tiles, BN, (double)a.N * a.K);
    if (a.allreduce) {
      const ARParams ar = *a.allreduce;
      switch (BN) {
        case 16: launch_streamk<16, 6, true, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ar); break;
        case 32: launch_streamk<32, 5, true, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ar); break;
        case 64: launch_streamk<64, 4, true, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ar); break;
        default: launch_streamk<128, 3, true, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ar); break;
      }
      return;
    }
    switch (BN) {
      case 16: launch_streamk<16, 6, false, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ARParams{}); break;
      case 32: launch_streamk<32, 5, false, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ARParams{}); break;
      case 64: launch_streamk<64, 4, false, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ARParams{}); break;
      default: launch_streamk<128, 3, false, true>(ma, mb, ep, a.N, (int)Kp, ctas, stream, ARParams{}); break;
    }
  } else {
    const CUtensorMap mb = make_kmajor_map(a.x, a.M, Kp, a.ldx / 2, 128);
    launch_streamk<128, 3, false, true>(ma, mb, ep, a.N, (int)Kp, device_sm_count(), stream, ARParams{},
                                        (a.M + 127) / 128);
  }
}

// ---------------------------------------------------------------- grouped MoE GEMM launcher
template <int BN, int STAGES, bool kRet>
static void launch_moe_grouped(const CUtensorMap& mw, const CUtensorMap& mx, const EpiParams& ep,
                               const MoeBlock* blocks, const int* num_blocks, int n_per_expert, int K, int grid,
                               cudaStream_t stream, const MoeRet& ret) {
  constexpr int kSmem = STAGES * GemmSmem<BN, STAGES>::kStageBytes + (2 * STAGES + 5) * 8 + 16 + 1024;
  auto kern = moe_grouped_swap_kernel<BN, STAGES, kRet>;
  static int attr_dev_mask = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(attr_dev_mask & (1 << (dev & 31)))) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem));
    attr_dev_mask |= 1 << (dev & 31);
  }
  launch_kernel(kern, dim3(grid), dim3(kGemmThreads), (size_t)kSmem, stream, mw, mx, ep, blocks, num_blocks,
                n_per_expert, (K + kBK - 1) / kBK, error_word(), ret);
}

template <bool kRet>
static void moe_grouped_dispatch(const MoeGemmArgs& a, cudaStream_t stream, const MoeRet& ret) {
  VRM_REQUIRE(a.K % 8 == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(a.x_perm) & 15) == 0,
              "moe gemm: K must be a multiple of 8 and operands 16-byte aligned");
  VRM_REQUIRE(a.BN == 16 || a.BN == 32 || a.BN == 64 || a.BN == 128, "moe gemm: BN must be 16, 32, 64 or 128");
  VRM_REQUIRE(a.epilogue != kEpiSiluMul || a.N % 2 == 0, "moe gemm: silu_mul needs an even N");
  if (a.max_blocks <= 0) return;
  EpiParams ep;
  ep.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  ep.ldo = (int)a.ldo;
  ep.bias = nullptr;
  ep.residual = nullptr;
  ep.M = 0;
  ep.N = a.N;
  ep.epilogue = a.epilogue;
  ep.scale_w = nullptr;
  ep.scale_x = nullptr;
  const CUtensorMap mw = make_kmajor_map(a.w, (int64_t)a.E * a.N, a.K, a.K, kBM);
  const CUtensorMap mx = make_kmajor_map(a.x_perm, a.rows_cap, a.K, a.ldx, a.BN);
  const int wtiles = (a.N + kBM - 1) / kBM;
  const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)a.max_blocks * wtiles, device_sm_count()));
  const auto* blocks = reinterpret_cast<const MoeBlock*>(a.blocks);
  switch (a.BN) {
    case 16: launch_moe_grouped<16, 8, kRet>(mw, mx, ep, blocks, a.num_blocks, a.N, a.K, grid, stream, ret); break;
    case 32: launch_moe_grouped<32, 8, kRet>(mw, mx, ep, blocks, a.num_blocks, a.N, a.K, grid, stream, ret); break;
    case 64: launch_moe_grouped<64, 6, kRet>(mw, mx, ep, blocks, a.num_blocks, a.N, a.K, grid, stream, ret); break;
    default: launch_moe_grouped<128, 5, kRet>(mw, mx, ep, blocks, a.num_blocks, a.N, a.K, grid, stream, ret); break;
  }
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_grouped_gemm(const MoeGemmArgs& a, cudaStream_t stream) { moe_grouped_dispatch<false>(a, stream, MoeRet{}); }

void moe_ep_grouped_return(const MoeEpBuffers& b, const MoeGemmArgs& g, cudaStream_t stream) {
  VRM_REQUIRE(g.epilogue == kEpiNone && g.N == b.H, "moe_ep_grouped_return: plain epilogue, N == H");
  MoeRet ret;
  ret.meta = b.meta_local;
  ret.yback = b.yback;
  ret.flags = b.flags;
  ret.epoch = b.epoch;
  ret.done = b.done + 1;
  ret.rank = b.rank;
  ret.world = b.world;
  ret.p_cap = b.p_cap;
  ret.H = b.H;
  moe_grouped_dispatch<true>(g, stream, ret);
}

}  // namespace vrm
