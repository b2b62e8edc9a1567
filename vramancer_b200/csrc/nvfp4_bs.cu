// NVFP4 x NVFP4 GEMM on the block-scaled tensor cores (tcgen05.mma kind::mxf4nvf4,
// scale_vec 16) and the row quantiser that feeds it (fused activation quantisation).
//
// Formats (both operands):
//   q    uint8 [rows, K/2]: e2m1 codes, element 2i in the low nibble of byte i
//   sf   e4m3 block scales, one per 16 elements of a row, in 512-byte atoms of
//        128 rows x 4 blocks: atom (row / 128, k / 64) at ((row/128) * K/64 + k/64) * 512,
//        byte (row % 32) * 16 + ((row / 32) % 4) * 4 + (k / 16) % 4 inside it
//   gs   fp32 global scale: one per tensor (weights) or one per row (activations)
//   value[r, k] = e2m1(q) * e4m3(sf) * gs
// The quantiser's rounding is the NVFP4 weight convention of nvfp4.cu (block scale
// e4m3_rn_sat(block_amax / 6 / gs), code e2m1_rn_sat(x / (scale * gs))), so weights
// quantised here hold the same codes and scales as the fragment-order copies.
//
// GEMM: D[m, n] = sum_k A[m, k] B[n, k] with A = activations (128-row tiles), B = weights
// (128-row tiles), K in tiles of 256 (128 bytes of codes per row).  Warp 0 issues the
// TMA loads of both code tiles (128-byte swizzle) and bulk copies of the four scale
// atoms of each operand per k-tile; warp 1 copies the atoms into tensor memory
// (tcgen05.cp 32x128b.warpx4: the 32 x 16-byte atom is broadcast to the four lane
// quarters, column = row / 32) and issues four MMAs (K = 64 each); warps 2-5 read the
// fp32 accumulator and scale it by gs_a[m] * gs_b.
//
// Reference parity: core/nvfp4_direct.py + core/fused_act_quant.py (W4A4 through
// torchao / cuBLAS block-scaled GEMMs; the reference's scale atoms use the same 128x4
// blocked layout, cuBLAS's "blocked" swizzle).
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kBsThreads = 192;
constexpr int kBsBM = 128;         // A rows per tile (MMA M)
constexpr int kBsBN = 128;         // B rows per tile (MMA N)
constexpr int kBsKB = 128;         // bytes of codes per row per k-tile (256 elements)
constexpr int kBsStages = 4;
constexpr int kAtom = 512;
constexpr int kTileA = kBsBM * kBsKB;            // 16 KB
constexpr int kTileB = kBsBN * kBsKB;            // 16 KB
constexpr int kStageB = kTileA + kTileB + 8 * kAtom;
constexpr int kBsSmem = kBsStages * kStageB + (2 * kBsStages + 1) * 8 + 16 + 1024;
constexpr uint32_t kBsTmemCols = 256;            // accumulator 128 + scale atoms 2 x 16

__device__ __forceinline__ uint16_t f32x2_to_e4m3x2_bs(float hi, float lo) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ float e4m3_to_f32_bs(uint8_t v) {
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"((uint16_t)v));
  return __half2float(__ushort_as_half((unsigned short)(h & 0xFFFFu)));
}
// 8 floats -> 8 e2m1 nibbles, element 2i in the low nibble of byte i
__device__ __forceinline__ uint32_t f32x8_to_e2m1x8_bs(const float (&v)[8]) {
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

__device__ __forceinline__ size_t sf_atom_offset(int row, int blk, int kb64) {
  return ((size_t)(row >> 7) * kb64 + (blk >> 2)) * kAtom + (row & 31) * 16 + ((row >> 5) & 3) * 4 + (blk & 3);
}

// One CTA per row: (per-row mode) amax -> gs; then every 16-block -> e4m3 scale + 8
// bytes of codes.  Rows in [valid, rows) are written as zeros.
__global__ void __launch_bounds__(256) nvfp4_rows_quant_kernel(const __nv_bfloat16* x, int64_t ldx, int valid,
                                                               int K, const float* gs_tensor, float* gs_rows,
                                                               uint8_t* q, uint8_t* sf) {
  pdl_launch();
  pdl_wait_for(x, gs_tensor);
  __shared__ float red[33];
  const int r = blockIdx.x;
  const int nb = K / 16, kb64 = K / 64;
  uint8_t* qrow = q + (size_t)r * (K / 2);
  if (r >= valid) {
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
      *reinterpret_cast<uint2*>(qrow + b * 8) = make_uint2(0u, 0u);
      sf[sf_atom_offset(r, b, kb64)] = 0;
    }
    if (gs_rows && threadIdx.x == 0) gs_rows[r] = 0.f;
    return;
  }
  const __nv_bfloat16* xr = x + (size_t)r * ldx;
  float gs;
  if (gs_tensor) {
    gs = *gs_tensor;
  } else {
    float m = 0.f;
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
      const uint4* p = reinterpret_cast<const uint4*>(xr + b * 16);
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint4 v = p[h];
        const uint32_t* pv = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int j = 0; j < 4; ++j) m = fmaxf(m, fmaxf(fabsf(bf16_lo(pv[j])), fabsf(bf16_hi(pv[j]))));
      }
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
    gs = amax > 0.f ? amax / 2688.f : 1.f;           // amax / (6 * 448)
    if (threadIdx.x == 0) gs_rows[r] = gs;
  }
  for (int b = threadIdx.x; b < nb; b += blockDim.x) {
    const uint4* p = reinterpret_cast<const uint4*>(xr + b * 16);
    float v[16];
    float bm = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = p[h];
      const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        v[8 * h + 2 * j] = bf16_lo(pu[j]);
        v[8 * h + 2 * j + 1] = bf16_hi(pu[j]);
        bm = fmaxf(bm, fmaxf(fabsf(v[8 * h + 2 * j]), fabsf(v[8 * h + 2 * j + 1])));
      }
    }
    const uint8_t s8 = (uint8_t)(f32x2_to_e4m3x2_bs(0.f, bm / 6.f / gs) & 0xFFu);
    const float denom = e4m3_to_f32_bs(s8) * gs;
    float lo[8], hi[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      lo[j] = denom > 0.f ? v[j] / denom : 0.f;
      hi[j] = denom > 0.f ? v[8 + j] / denom : 0.f;
    }
    *reinterpret_cast<uint2*>(qrow + b * 8) = make_uint2(f32x8_to_e2m1x8_bs(lo), f32x8_to_e2m1x8_bs(hi));
    sf[sf_atom_offset(r, b, kb64)] = s8;
  }
}

// ---------------------------------------------------------------- block-scaled MMA helpers
__device__ __forceinline__ void umma_nvf4(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t tsfa, uint32_t tsfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate), "r"(tsfa), "r"(tsfb)
      : "memory");
}

// 32 rows x 16 bytes of shared memory (one scale atom) -> 4 columns of every lane quarter
__device__ __forceinline__ void tmem_cp_atom(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// K-major, no swizzle: 8-row core matrices of 16-byte rows, 128 bytes apart
__device__ __forceinline__ uint64_t make_atom_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(128 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  return d;
}

// Instruction descriptor, kind::mxf4nvf4: A, B e2m1 (format 1), e4m3 scales, K-major, K 64
__host__ __device__ constexpr uint32_t make_idesc_nvf4(int M, int N) {
  return (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(smem_dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

struct BsParams {
  const uint8_t* sfa;
  const uint8_t* sfb;
  const float* gsa;      // [rows of A] per-row scale
  const float* gsb;      // [1]
  __nv_bfloat16* out;
  int64_t ldo;
  const __nv_bfloat16* bias;      // [N] or null
  const __nv_bfloat16* residual;  // [M, ldo] or null (may alias out)
  int silu_mul;          // 1: out[m, n/2] = silu(y[m, n]) * y[m, n+1] over interleaved pairs
  int M, N, k_tiles, kb64;
  uint32_t* err;
};

__global__ void __launch_bounds__(kBsThreads, 1) nvfp4_bs_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                                                                      const __grid_constant__ CUtensorMap map_b,
                                                                      BsParams P) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBsStages * kStageB);
  uint64_t* empty = full + kBsStages;
  uint64_t* tfull = empty + kBsStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.y * kBsBM, n0 = blockIdx.x * kBsBN;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
    for (int s = 0; s < kBsStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(tfull, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kBsTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const uint8_t* sfa = P.sfa;
  const uint8_t* sfb = P.sfb;
  const float* gsa = P.gsa;
  const float* gsb = P.gsb;
  pdl_wait_for(sfa, sfb, gsa, gsb);
  opaque_after_wait(P.bias);
  opaque_after_wait(P.residual);

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    const uint64_t pol_a = policy_evict_last(), pol_b = policy_evict_first();
    const uint8_t* sfa_row = sfa + (size_t)(m0 / kBsBM) * P.kb64 * kAtom;
    const uint8_t* sfb_row = sfb + (size_t)(n0 / kBsBN) * P.kb64 * kAtom;
    for (int t = 0; t < P.k_tiles; ++t) {
      const int s = t % kBsStages;
      if (t >= kBsStages && !mbar_wait(&empty[s], (uint32_t)(((t / kBsStages) & 1) ^ 1), P.err)) break;
      uint8_t* st = smem + s * kStageB;
      mbar_arrive_expect_tx(&full[s], kStageB);
      tma_load_2d(st, &map_a, &full[s], t * kBsKB, m0, pol_a);
      tma_load_2d(st + kTileA, &map_b, &full[s], t * kBsKB, n0, pol_b);
      bulk_load(st + kTileA + kTileB, sfa_row + (size_t)t * 4 * kAtom, 4 * kAtom, &full[s]);
      bulk_load(st + kTileA + kTileB + 4 * kAtom, sfb_row + (size_t)t * 4 * kAtom, 4 * kAtom, &full[s]);
    }
    // the CTA may not exit while loads are in flight
    const int first = P.k_tiles > kBsStages ? P.k_tiles - kBsStages : 0;
    for (int t = first; t < P.k_tiles; ++t) mbar_wait(&full[t % kBsStages], (uint32_t)((t / kBsStages) & 1), P.err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- scale-atom copies + MMA issue
    constexpr uint32_t idesc = make_idesc_nvf4(kBsBM, kBsBN);
    const uint32_t t_sfa = tmem_base + kBsBN, t_sfb = tmem_base + kBsBN + 16;
    for (int t = 0; t < P.k_tiles; ++t) {
      const int s = t % kBsStages;
      if (!mbar_wait(&full[s], (uint32_t)((t / kBsStages) & 1), P.err)) break;
      tc_fence_after();
      const uint32_t sa = smem_u32(smem + s * kStageB);
      const uint32_t sb = sa + kTileA;
      const uint32_t ssf = sb + kTileB;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        tmem_cp_atom(t_sfa + 4 * j, make_atom_desc(ssf + j * kAtom));
        tmem_cp_atom(t_sfb + 4 * j, make_atom_desc(ssf + (4 + j) * kAtom));
      }
      const uint64_t da = make_sw128_desc(sa), db = make_sw128_desc(sb);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        umma_nvf4(tmem_base, da + (uint64_t)(j * 2), db + (uint64_t)(j * 2), idesc, t_sfa + 4 * j, t_sfb + 4 * j,
                  (t > 0 || j > 0) ? 1u : 0u);
      umma_commit(&empty[s]);
    }
    umma_commit(tfull);
  } else if (warp >= 2) {
    // ---------------- epilogue: TMEM lane = row of A, column = row of B
    const int q = warp & 3;
    const int row = 32 * q + lane;
    const int m = m0 + row;
    const bool ok = mbar_wait(tfull, 0, P.err);
    tc_fence_after();
    const float g = (m < P.M) ? gsa[m] * gsb[0] : 0.f;
    const uint32_t t_lane = tmem_base + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
    for (int c0 = 0; c0 < kBsBN; c0 += 16) {
      uint32_t r[16];
      tmem_ld_32x32b_x16(t_lane + (uint32_t)c0, r);
      tmem_wait_ld();
      if (!ok || m >= P.M || n0 + c0 >= P.N) continue;
      const int n = n0 + c0;
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]) * g;
      if (P.bias) {
        const uint4 b0 = *reinterpret_cast<const uint4*>(P.bias + n);
        const uint4 b1 = *reinterpret_cast<const uint4*>(P.bias + n + 8);
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&b0);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&b1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] += bf16_lo(q0[j]);
          v[2 * j + 1] += bf16_hi(q0[j]);
          v[8 + 2 * j] += bf16_lo(q1[j]);
          v[8 + 2 * j + 1] += bf16_hi(q1[j]);
        }
      }
      if (P.silu_mul) {
        // interleaved (gate, up) pairs -> 8 outputs at column n / 2
        uint4 o;
        uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float g0 = v[4 * j], u0 = v[4 * j + 1], g1 = v[4 * j + 2], u1 = v[4 * j + 3];
          po[j] = pack_bf16x2(g0 / (1.f + __expf(-g0)) * u0, g1 / (1.f + __expf(-g1)) * u1);
        }
        *reinterpret_cast<uint4*>(P.out + (size_t)m * P.ldo + n / 2) = o;
        continue;
      }
      __nv_bfloat16* dst = P.out + (size_t)m * P.ldo + n;
      if (P.residual) {
        const __nv_bfloat16* rs = P.residual + (size_t)m * P.ldo + n;
        const uint4 r0 = *reinterpret_cast<const uint4*>(rs);
        const uint4 r1 = *reinterpret_cast<const uint4*>(rs + 8);
        const uint32_t* q0 = reinterpret_cast<const uint32_t*>(&r0);
        const uint32_t* q1 = reinterpret_cast<const uint32_t*>(&r1);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          v[2 * j] += bf16_lo(q0[j]);
          v[2 * j + 1] += bf16_hi(q0[j]);
          v[8 + 2 * j] += bf16_lo(q1[j]);
          v[8 + 2 * j + 1] += bf16_hi(q1[j]);
        }
      }
      uint4 o0, o1;
      uint32_t* p0 = reinterpret_cast<uint32_t*>(&o0);
      uint32_t* p1 = reinterpret_cast<uint32_t*>(&o1);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        p0[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
        p1[j] = pack_bf16x2(v[8 + 2 * j], v[8 + 2 * j + 1]);
      }
      *reinterpret_cast<uint4*>(dst) = o0;
      *reinterpret_cast<uint4*>(dst + 8) = o1;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kBsTmemCols);
  }
}

// uint8 [rows, cols] row-major (cols bytes per row), box = 128 bytes x box_rows, 128-byte swizzle
CUtensorMap make_u8_map(const void* ptr, int64_t rows, int64_t cols, int box_rows) {
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols};
  cuuint32_t box[2] = {(cuuint32_t)kBsKB, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_tensor_map()(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box,
                                   estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  VRM_REQUIRE(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (u8) failed (code " + std::to_string((int)r) + ")");
  return map;
}

}  // namespace

void nvfp4_rows_quantize(const void* x, int64_t ldx, int valid, int rows, int K, const float* gs_tensor,
                         float* gs_rows, uint8_t* q, uint8_t* sf, cudaStream_t st) {
  VRM_REQUIRE(K % 256 == 0 && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0,
              "nvfp4 rows: K must be a multiple of 256 and rows 16-byte aligned");
  VRM_REQUIRE(rows % 128 == 0 && valid <= rows, "nvfp4 rows: rows padded to 128");
  VRM_REQUIRE(gs_tensor != nullptr || gs_rows != nullptr, "nvfp4 rows: give a tensor scale or a row-scale output");
  if (rows == 0) return;
  launch_kernel(nvfp4_rows_quant_kernel, dim3(rows), dim3(256), 0, st, reinterpret_cast<const __nv_bfloat16*>(x),
                ldx, valid, K, gs_tensor, gs_rows, q, sf);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void nvfp4_bs_gemm(const uint8_t* qa, const uint8_t* sfa, const float* gsa, int M, int Mpad, const uint8_t* qb,
                   const uint8_t* sfb, const float* gsb, int N, int K, void* out, int64_t ldo, cudaStream_t st,
                   const void* bias, const void* residual, int silu_mul) {
  VRM_REQUIRE(!silu_mul || residual == nullptr, "nvfp4 block-scaled gemm: silu_mul takes no residual");
  VRM_REQUIRE(K % 256 == 0 && N % kBsBN == 0 && Mpad % kBsBM == 0 && M <= Mpad,
              "nvfp4 block-scaled gemm: K % 256, N % 128, padded M % 128");
  VRM_REQUIRE(ldo % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0, "nvfp4 block-scaled gemm: out alignment");
  if (M <= 0) return;
  const CUtensorMap ma = make_u8_map(qa, Mpad, K / 2, kBsBM);
  const CUtensorMap mb = make_u8_map(qb, N, K / 2, kBsBN);
  BsParams p;
  p.sfa = sfa;
  p.sfb = sfb;
  p.gsa = gsa;
  p.gsb = gsb;
  p.out = reinterpret_cast<__nv_bfloat16*>(out);
  p.ldo = ldo;
  p.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  p.residual = reinterpret_cast<const __nv_bfloat16*>(residual);
  p.silu_mul = silu_mul;
  p.M = M;
  p.N = N;
  p.k_tiles = K / 256;
  p.kb64 = K / 64;
  p.err = error_word();
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(nvfp4_bs_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kBsSmem));
    set[dev & 63] = true;
  }
  const dim3 grid(N / kBsBN, (M + kBsBM - 1) / kBsBM);
  launch_kernel(nvfp4_bs_gemm_kernel, grid, dim3(kBsThreads), (size_t)kBsSmem, st, ma, mb, p);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
