// Paged attention over the KV pool  cache[page, layer, {k,v}, kv_head, 16, row]
// with bf16 rows, fp8-e4m3 rows (per-(layer, k/v, kv_head) fp32 scales) or four-bit rows
// (head_dim/2 code bytes + one fp16 {scale, min} pair per 32 dims, dequantised into the
// bf16 MMA tile in shared memory).
//
// decode  (one new token per sequence):
//   grid (kv_heads, batch, splits), 4 warps.  One CTA serves the whole GQA group of a
//   KV head, so every K/V byte is read once for all its query heads.  The group
//   (<= 8 heads) is the MMA row block; the 16 tokens of a page are the columns.  Pages
//   of the split are dealt round-robin to the warps; each warp double-buffers its
//   pages with cp.async and keeps its own online-softmax state; warps merge in shared
//   memory.  With splits > 1 each CTA writes a normalised partial and the last CTA of
//   the (sequence, kv head) merges them (flash-decoding); that CTA resets the counter,
//   so the kernel replays inside CUDA graphs.
// prefill (causal, varlen, chunked-prefill aware):
//   grid (q_tiles of 64, q_heads, batch), 4 warps x 16 query rows.  Keys come from the
//   same paged pool (cached prefix pages included), 64 keys per stage, double-buffered.
//
// Decode attention is bound by HBM bandwidth (the GQA group gives at most 8 rows, far
// below the 64/128-row tcgen05 tile), so its MMAs use the warp-level m16n8k16 path and
// the kernel is measured by DRAM throughput.
//
// Reference parity: csrc/paged_attention_kernel.cu:61-438 (SIMT decode over fp32 /
// fp16 / q4 pages, not on the reference's forward path); the reference prefill runs
// HF SDPA (core/turbo_engine.py:72-93).
#include <cooperative_groups.h>

#include <algorithm>
#include <climits>
#include <cstdlib>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

constexpr int kPage = 16;

// Byte offset of 16-byte chunk `ch` of row `r` in a swizzled tile whose rows are ROWB
// bytes long.  XOR-ing the chunk with (r & 7) puts the eight rows of every ldmatrix
// 8x8 read in different banks.
template <int ROWB>
__device__ __forceinline__ uint32_t swz(int r, int ch) {
  return (uint32_t)(r * ROWB + ((ch ^ (r & 7)) << 4));
}

// Transpose of an 8x8 b16 matrix held in mma fragment layout (one register per lane).
__device__ __forceinline__ void movmatrix_trans(uint32_t in, uint32_t& out) {
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(out) : "r"(in));
}

// fp8 e4m3 x2 -> bf16 x2 (exact: every e4m3 value is a bf16 value)
__device__ __forceinline__ uint32_t fp8x2_to_bf16x2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(v, __NV_E4M3);
  const float2 f = __half22float2(*reinterpret_cast<__half2*>(&h));
  return pack_bf16x2(f.x, f.y);
}

// Convert rows x D fp8 bytes (row-major, contiguous) at raw into the swizzled bf16
// tile at dst, spread over nthr threads starting at index tid.
template <int D>
__device__ __forceinline__ void convert_fp8_tile(const uint8_t* raw, uint8_t* dst, int rows, int tid, int nthr) {
  constexpr int kChunks = D / 16;   // 16 fp8 per 16-byte chunk
  for (int i = tid; i < rows * kChunks; i += nthr) {
    const int r = i / kChunks, c = i % kChunks;
    const uint4 v = *reinterpret_cast<const uint4*>(raw + r * D + c * 16);
    const uint16_t* p = reinterpret_cast<const uint16_t*>(&v);
    uint4 o0, o1;
    uint32_t* q0 = reinterpret_cast<uint32_t*>(&o0);
    uint32_t* q1 = reinterpret_cast<uint32_t*>(&o1);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      q0[j] = fp8x2_to_bf16x2(p[j]);
      q1[j] = fp8x2_to_bf16x2(p[4 + j]);
    }
    *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, 2 * c)) = o0;
    *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, 2 * c + 1)) = o1;
  }
}

// rows x D four-bit rows (kBytes each, contiguous) at raw -> the swizzled bf16 tile at
// dst; one thread per (row, 32-dim group), spread over nthr threads from tid.
template <int D>
__device__ __forceinline__ void convert_q4_tile(const uint8_t* raw, uint8_t* dst, int rows, int tid, int nthr) {
  constexpr int kRowB = PageRow<D, kFmtQ4>::kBytes;
  constexpr int kGroups = D / 32;
  for (int i = tid; i < rows * kGroups; i += nthr) {
    const int r = i / kGroups, gi = i % kGroups;
    const uint8_t* row = raw + r * kRowB;
    // the group's 32 codes (rows are 8-byte aligned: D/2 + D/8 bytes, D = 64 or 128)
    const uint2 v0 = *reinterpret_cast<const uint2*>(row + gi * 16);
    const uint2 v1 = *reinterpret_cast<const uint2*>(row + gi * 16 + 8);
    const __half2 sm = *reinterpret_cast<const __half2*>(row + D / 2 + gi * 4);
    const float sc = __low2float(sm), mn = __high2float(sm);
    const uint32_t w[4] = {v0.x, v0.y, v1.x, v1.y};
#pragma unroll
    for (int c = 0; c < 4; ++c) {          // 8 values per output chunk
      uint4 o;
      uint32_t* q = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float a = fmaf((float)((w[c] >> (8 * j)) & 15u), sc, mn);
        const float b = fmaf((float)((w[c] >> (8 * j + 4)) & 15u), sc, mn);
        q[j] = pack_bf16x2(a, b);
      }
      *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, gi * 4 + c)) = o;
    }
  }
}

// ---- f16 operand path of the fp8 / four-bit decode kernels.  Their K fragments are
// built straight from the stored rows in registers (no shared-memory tile), their V
// tile is converted to f16 (exact for e4m3; one FMA per value for four-bit), and the
// MMAs run f16 x f16 -> f32.
__device__ __forceinline__ void mma_f16_m16n8k16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                                 uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t bf16x2_to_f16x2(uint32_t v) { return pack_f16x2(bf16_lo(v), bf16_hi(v)); }
__device__ __forceinline__ uint32_t fp8x2_to_f16x2(uint16_t v) {
  __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(v, __NV_E4M3);
  return (uint32_t)h.x | ((uint32_t)h.y << 16);
}
// one code byte (element 2i low nibble, 2i+1 high) -> f16x2 of code * s + m: 1024 + code is
// an exact f16 (the nibble in the mantissa), 1024 is subtracted exactly, then one FMA
__device__ __forceinline__ uint32_t q4_byte_to_f16x2(uint32_t byte, uint32_t s2, uint32_t m2) {
  const uint32_t x = 0x64006400u | (byte & 0xFu) | ((byte & 0xF0u) << 12);
  uint32_t y, r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(y) : "r"(x), "r"(0x64006400u));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(y), "r"(s2), "r"(m2));
  return r;
}
// 16-byte chunk of a stored fp8 K row: swizzled so the fragment gathers of the eight
// rows g of a warp hit different banks
template <int D>
__device__ __forceinline__ uint32_t f8_kchunk(int r, int ch) {
  return (uint32_t)(r * D + ((ch ^ (D == 128 ? (r & 7) : ((r >> 1) & 3))) << 4));
}

// fp8 rows -> swizzled f16 tile (V operand)
template <int D>
__device__ __forceinline__ void convert_fp8_tile_f16(const uint8_t* raw, uint8_t* dst, int rows, int tid, int nthr) {
  constexpr int kChunks = D / 16;
  for (int i = tid; i < rows * kChunks; i += nthr) {
    const int r = i / kChunks, c = i % kChunks;
    const uint4 v = *reinterpret_cast<const uint4*>(raw + r * D + c * 16);
    const uint16_t* p = reinterpret_cast<const uint16_t*>(&v);
    uint4 o0, o1;
    o0.x = fp8x2_to_f16x2(p[0]);
    o0.y = fp8x2_to_f16x2(p[1]);
    o0.z = fp8x2_to_f16x2(p[2]);
    o0.w = fp8x2_to_f16x2(p[3]);
    o1.x = fp8x2_to_f16x2(p[4]);
    o1.y = fp8x2_to_f16x2(p[5]);
    o1.z = fp8x2_to_f16x2(p[6]);
    o1.w = fp8x2_to_f16x2(p[7]);
    *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, 2 * c)) = o0;
    *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, 2 * c + 1)) = o1;
  }
}

// four-bit rows -> swizzled f16 tile (V operand): one thread per (row, 32-dim group)
template <int D>
__device__ __forceinline__ void convert_q4_tile_f16(const uint8_t* raw, uint8_t* dst, int rows, int tid, int nthr) {
  constexpr int kRowB = PageRow<D, kFmtQ4>::kBytes;
  constexpr int kGroups = D / 32;
  for (int i = tid; i < rows * kGroups; i += nthr) {
    const int r = i / kGroups, gi = i % kGroups;
    const uint8_t* row = raw + r * kRowB;
    const uint2 v0 = *reinterpret_cast<const uint2*>(row + gi * 16);
    const uint2 v1 = *reinterpret_cast<const uint2*>(row + gi * 16 + 8);
    const uint32_t sm = *reinterpret_cast<const uint32_t*>(row + D / 2 + gi * 4);   // {scale, min} f16
    const uint32_t s2 = __byte_perm(sm, 0, 0x1010), m2 = __byte_perm(sm, 0, 0x3232);
    const uint32_t w[4] = {v0.x, v0.y, v1.x, v1.y};
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 o;
      o.x = q4_byte_to_f16x2(w[c] & 0xFFu, s2, m2);
      o.y = q4_byte_to_f16x2((w[c] >> 8) & 0xFFu, s2, m2);
      o.z = q4_byte_to_f16x2((w[c] >> 16) & 0xFFu, s2, m2);
      o.w = q4_byte_to_f16x2(w[c] >> 24, s2, m2);
      *reinterpret_cast<uint4*>(dst + swz<D * 2>(r, gi * 4 + c)) = o;
    }
  }
}

// ============================================================== decode
template <int D, int FMT>
struct DecodeSmem {
  static constexpr int kTileB = kPage * D * 2;                       // one bf16 16 x D tile
  static constexpr int kRawB = kPage * PageRow<D, FMT>::kBytes;      // bytes per K (or V) page chunk
  static constexpr int kStageB = 2 * kRawB;                          // K + V
  static constexpr int kWarpB = 2 * kStageB + (FMT != kFmtBf16 ? 2 * kTileB : 0);
  static constexpr int kTotal = 4 * kWarpB;
};

struct DecodeParams {
  const __nv_bfloat16* q;
  int64_t ld_q;
  const uint8_t* cache;
  int layer, num_layers, KH, G;
  const int* block_tables;
  int bt_stride;
  const int* context_lens;
  const float* kv_scale;
  float sm_scale;
  __nv_bfloat16* out;
  int64_t ld_o;
  float* ws_o;
  float* ws_ml;
  uint32_t* counters;
  // Fused RoPE + KV write (positions != null): q holds the unrotated qkv rows (k of KV
  // head h at column (Hq + h) * D, v at (Hq + KH + h) * D); q and the new k are rotated
  // here (rotate-half over all D dims; cos_sin null = no rotation) and the token's k / v
  // are stored at slot_mapping[b] by the warp that reads that page.
  const int* positions;
  const float* cos_sin;      // [max_pos, D] = [cos | sin]
  const int* slot_mapping;
  uint8_t* cache_w;
  int Hq;
  long long num_pages;       // pool pages (checked in bounds-check builds)
  uint32_t* err;
  const uint8_t* pf;         // L2 prefetch region (the next GEMM's weights) or null
  unsigned long long pf_bytes;
};

// Bulk L2 prefetch of this CTA's equal slice of [pf, pf + bytes) (16-byte granules, in
// pieces of at most 64 KB).  Fire and forget: nothing waits on it, and the data only
// warms L2 for the kernel that follows.
__device__ __forceinline__ void l2_prefetch_slice(const uint8_t* pf, unsigned long long bytes) {
  const unsigned long long nct = (unsigned long long)gridDim.x * gridDim.y * gridDim.z;
  const unsigned long long id =
      blockIdx.x + (unsigned long long)gridDim.x * (blockIdx.y + (unsigned long long)gridDim.y * blockIdx.z);
  const unsigned long long chunk = (((bytes + nct - 1) / nct) + 15ull) & ~15ull;
  const unsigned long long beg = id * chunk;
  if (beg >= bytes) return;
  const unsigned long long end = beg + chunk < bytes ? beg + chunk : bytes;
  for (unsigned long long o = beg; o < end; o += 65536ull) {
    const uint32_t n = (uint32_t)((end - o) < 65536ull ? (end - o) : 65536ull);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(pf + o), "r"(n) : "memory");
  }
}

// Stores this step's k (rotated) and v of sequence b, KV head kvh, into its cache slot,
// with the rounding of the standalone RoPE + KV write kernel (k rounded to bf16 after
// rotation; fp8 pages take that bf16 value / scale, saturating; four-bit pages quantise
// the bf16 row per 32-dim group).
template <int D, int FMT>
__device__ __forceinline__ void decode_write_new_kv(const DecodeParams& P, int b, int kvh, int lane) {
  const int slot = P.slot_mapping[b];
  if (slot < 0 || !in_bounds(slot / kPage, P.num_pages, P.err)) return;
  constexpr bool kFp8 = FMT == kFmtFp8;
  constexpr int kRowB = PageRow<D, FMT>::kBytes;
  constexpr int H2 = D / 2;
  const int KH = P.KH;
  const __nv_bfloat16* row = P.q + (size_t)b * P.ld_q;
  const __nv_bfloat16* ks = row + (size_t)(P.Hq + kvh) * D;
  const __nv_bfloat16* vs = row + (size_t)(P.Hq + KH + kvh) * D;
  const int page = slot / kPage, off = slot % kPage;
  const size_t head_stride = (size_t)kPage * kRowB;
  uint8_t* kd = P.cache_w + (size_t)page * ((size_t)P.num_layers * 2 * KH * head_stride) +
                (((size_t)P.layer * 2 + 0) * KH + kvh) * head_stride + (size_t)off * kRowB;
  uint8_t* vd = kd + (size_t)KH * head_stride;
  const float* cs = P.cos_sin ? P.cos_sin + (size_t)P.positions[b] * D : nullptr;
  if constexpr (FMT == kFmtQ4) {
    // lane l quantises dims [D/32 l, D/32 (l + 1)) of k and of v
    constexpr int kV = D / 32;
    float xk[kV], xv[kV];
#pragma unroll
    for (int j = 0; j < kV; ++j) {
      const int d = lane * kV + j;
      float k = __bfloat162float(ks[d]);
      if (cs) {
        const int i = d < H2 ? d : d - H2;
        float o1, o2;
        rope_rotate(__bfloat162float(ks[i]), __bfloat162float(ks[i + H2]), cs[i], cs[H2 + i], o1, o2);
        k = __bfloat162float(__float2bfloat16(d < H2 ? o1 : o2));
      }
      xk[j] = k;
      xv[j] = __bfloat162float(vs[d]);
    }
    q4_store_row<D>(kd, xk, lane);
    q4_store_row<D>(vd, xv, lane);
    return;
  }
  float kinv = 1.f, vinv = 1.f;
  if (kFp8) {
    kinv = 1.f / P.kv_scale[(P.layer * 2 + 0) * KH + kvh];
    vinv = 1.f / P.kv_scale[(P.layer * 2 + 1) * KH + kvh];
  }
  auto put = [&](uint8_t* dst, int d, __nv_bfloat16 x, float inv) {
    if (kFp8) dst[d] = __nv_cvt_float_to_fp8(__bfloat162float(x) * inv, __NV_SATFINITE, __NV_E4M3);
    else reinterpret_cast<__nv_bfloat16*>(dst)[d] = x;
  };
  for (int i = lane; i < H2; i += 32) {
    __nv_bfloat16 a = ks[i], c2 = ks[i + H2];
    if (cs) {
      float o1, o2;
      rope_rotate(__bfloat162float(a), __bfloat162float(c2), cs[i], cs[H2 + i], o1, o2);
      a = __float2bfloat16(o1);
      c2 = __float2bfloat16(o2);
    }
    put(kd, i, a, kinv);
    put(kd, i + H2, c2, kinv);
  }
  for (int d = lane; d < D; d += 32) put(vd, d, vs[d], vinv);
}

// kCluster: the splits of one (sequence, KV head) are the CTAs of one thread-block
// cluster (2..8); each keeps its partial in shared memory and, after a cluster barrier,
// merges a slice of the outputs from its peers' shared memory (no global partials, no
// completion counter).  Otherwise splits merge through global scratch: the last CTA
// to finish (counter) combines them.
template <int D, int FMT, bool kCluster = false>
__global__ void __launch_bounds__(128) paged_decode_kernel(DecodeParams P) {
  pdl_launch();
  // weights are constant: their prefetch may start before the previous kernel ends
  if (P.pf != nullptr && threadIdx.x == 0) l2_prefetch_slice(P.pf, P.pf_bytes);
  using S = DecodeSmem<D, FMT>;
  constexpr bool kFp8 = FMT == kFmtFp8;
  constexpr int ROWB = D * 2;
  constexpr int kChunkPerRow = D * 2 / 16;   // bf16 pages: swizzled 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_m[4][8], s_l[4][8];
  __shared__ uint32_t s_last;

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z, nsplit = gridDim.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int G = P.G, KH = P.KH;

  const int ctx = P.context_lens[b];
  const int npages = (ctx + kPage - 1) / kPage;
  const int pps = (npages + nsplit - 1) / nsplit;
  const int p_begin = split * pps;
  const int p_end = min(npages, p_begin + pps);

  float k_scale = 1.f, v_scale = 1.f;
  if (kFp8) {
    k_scale = P.kv_scale[(P.layer * 2 + 0) * KH + kvh];
    v_scale = P.kv_scale[(P.layer * 2 + 1) * KH + kvh];
  }
  const float scale_log2 = P.sm_scale * 1.4426950408889634f * k_scale;

  uint8_t* wbase = smem + warp * S::kWarpB;
  const int* bt = P.block_tables + (size_t)b * P.bt_stride;
  const size_t head_stride = (size_t)S::kRawB;                              // one (k|v, head) chunk
  const size_t page_stride = (size_t)P.num_layers * 2 * KH * head_stride;   // one page, all layers

  auto issue = [&](int page_local, int stage) {
    int page = bt[page_local];
    if (!in_bounds(page, P.num_pages, P.err)) page = 0;   // bounds-check builds: read page 0 instead
    const uint8_t* kp = P.cache + (size_t)page * page_stride + (((size_t)P.layer * 2 + 0) * KH + kvh) * head_stride;
    const uint8_t* vp = kp + (size_t)KH * head_stride;
    uint8_t* dst = wbase + stage * S::kStageB;
    const uint32_t dk = smem_u32(dst), dv = smem_u32(dst + S::kRawB);
    constexpr int kTotalChunks = S::kRawB / 16;
#pragma unroll
    for (int i = lane; i < kTotalChunks; i += 32) {
      // bf16 pages land swizzled for ldmatrix; fp8 K rows with a chunk swizzle for the
      // register gathers; other fp8 / four-bit rows as stored
      const uint32_t off = FMT == kFmtBf16 ? swz<ROWB>(i / kChunkPerRow, i % kChunkPerRow) : (uint32_t)(i * 16);
      const uint32_t koff = FMT == kFmtFp8 ? f8_kchunk<D>(i / (D / 16), i % (D / 16)) : off;
      cp_async16(dk + koff, kp + (size_t)i * 16, true);
      cp_async16(dv + off, vp + (size_t)i * 16, true);
    }
  };

  // Block tables and context lengths come from the step's input copy, which completes
  // before the first kernel of the launch chain starts; KV pages before the one holding
  // this step's token were written by earlier steps.  So the warp's first page is
  // requested before waiting for the previous kernel (RoPE + KV write), unless it is
  // the page that kernel is writing.
  const int my_first = p_begin + warp;
  const int live_page = (ctx - 1) / kPage;
  const bool early = my_first < p_end && my_first < live_page;
  if (early) issue(my_first, 0);
  cp_async_commit();
  pdl_wait();
  if (P.positions != nullptr && ctx > 0 && live_page >= p_begin && live_page < p_end &&
      warp == ((live_page - p_begin) & 3)) {
    // fused KV write: the warp that reads the live page stores this step's token first;
    // the fence orders the stores before that warp's cp.async reads of the page
    decode_write_new_kv<D, FMT>(P, b, kvh, lane);
    __threadfence();
    __syncwarp();
  }
  if (!early && my_first < p_end) issue(my_first, 0);
  cp_async_commit();

  // Q as the MMA B operand (k = head dims, n = the group's heads; heads >= G are zero).
  // Scores are computed transposed, S^T = K Q^T: the 16 tokens of a page fill the MMA
  // rows and the (<= 8) heads the columns, so no MMA row is wasted on absent heads.
  uint32_t qb[D / 16][2];
  {
    const __nv_bfloat16* qrow = P.q + (size_t)b * P.ld_q + (size_t)(kvh * G + g) * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      if (g < G) {
        qb[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * c);
        qb[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * c);
      } else {
        qb[kk][0] = qb[kk][1] = 0u;
      }
    }
    if (P.positions != nullptr && P.cos_sin != nullptr && g < G) {
      // fused RoPE on q: dims d and d + D/2 sit in chunks kk and kk + D/32 of this thread
      const float* cs = P.cos_sin + (size_t)P.positions[b] * D;
#pragma unroll
      for (int kk = 0; kk < D / 32; ++kk) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int d = kk * 16 + h * 8 + 2 * c;
          const uint32_t lo = qb[kk][h], hi = qb[kk + D / 32][h];
          float a0, a1, b0, b1;
          rope_rotate(bf16_lo(lo), bf16_lo(hi), cs[d], cs[D / 2 + d], a0, b0);
          rope_rotate(bf16_hi(lo), bf16_hi(hi), cs[d + 1], cs[D / 2 + d + 1], a1, b1);
          qb[kk][h] = pack_bf16x2(a0, a1);
          qb[kk + D / 32][h] = pack_bf16x2(b0, b1);
        }
      }
    }
  }

  if constexpr (FMT != kFmtBf16) {
    // fp8 / four-bit pages run f16 MMAs: Q as f16 (saturating)
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      qb[kk][0] = bf16x2_to_f16x2(qb[kk][0]);
      qb[kk][1] = bf16x2_to_f16x2(qb[kk][1]);
    }
  }

  // O^T accumulators: tile mt covers dims [16 mt, 16 mt + 16); this thread holds
  // (dim 16 mt + g, heads 2c, 2c+1) in [0], [1] and (dim 16 mt + g + 8, same heads) in [2], [3]
  float o[D / 16][4];
#pragma unroll
  for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  // online-softmax state of heads 2c and 2c+1 (identical in the 8 lanes sharing c)
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

  int it = 0;
  for (int p = my_first; p < p_end; p += 4, ++it) {
    const int stage = it & 1;
    if (p + 4 < p_end) issue(p + 4, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncwarp();
    uint8_t* kt = wbase + stage * S::kStageB;
    uint8_t* vt = kt + S::kRawB;
    if constexpr (FMT != kFmtBf16) {
      // V -> swizzled f16 tile (K is read from its stored rows below)
      uint8_t* cv = wbase + 2 * S::kStageB + S::kTileB;
      if constexpr (FMT == kFmtFp8) convert_fp8_tile_f16<D>(vt, cv, kPage, lane, 32);
      else convert_q4_tile_f16<D>(vt, cv, kPage, lane, 32);
      __syncwarp();
      vt = cv;
    }
    const uint32_t kaddr = smem_u32(kt), vaddr = smem_u32(vt);

    // S^T = K Q^T: A = the page's K rows (tokens) x 16 dims, four 8x8 matrices
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if constexpr (FMT == kFmtBf16) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int ch = 2 * kk + (lane >> 4);
        uint32_t a0, a1, a2, a3;
        ldsm_x4(kaddr + swz<ROWB>(row, ch), a0, a1, a2, a3);
        mma_bf16_16816(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
    } else if constexpr (FMT == kFmtFp8) {
      // fragment (row g / g + 8, dims 16 kk + 2c (+ 8)): two e4m3 bytes each, exact in f16
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint8_t* r0 = kt + f8_kchunk<D>(g, kk) + 2 * c;
        const uint8_t* r1 = kt + f8_kchunk<D>(g + 8, kk) + 2 * c;
        const uint32_t a0 = fp8x2_to_f16x2(*reinterpret_cast<const uint16_t*>(r0));
        const uint32_t a1 = fp8x2_to_f16x2(*reinterpret_cast<const uint16_t*>(r1));
        const uint32_t a2 = fp8x2_to_f16x2(*reinterpret_cast<const uint16_t*>(r0 + 8));
        const uint32_t a3 = fp8x2_to_f16x2(*reinterpret_cast<const uint16_t*>(r1 + 8));
        mma_f16_m16n8k16(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
      }
    } else {
      // four-bit: the fragment's dims 2c, 2c + 1 are one code byte; scale / min per
      // 32-dim group of rows g and g + 8
      constexpr int kRowB = PageRow<D, kFmtQ4>::kBytes;
      const uint8_t* r0 = kt + g * kRowB;
      const uint8_t* r1 = kt + (g + 8) * kRowB;
#pragma unroll
      for (int gi = 0; gi < D / 32; ++gi) {
        const uint32_t sm0 = *reinterpret_cast<const uint32_t*>(r0 + D / 2 + gi * 4);
        const uint32_t sm1 = *reinterpret_cast<const uint32_t*>(r1 + D / 2 + gi * 4);
        const uint32_t s0 = __byte_perm(sm0, 0, 0x1010), m0 = __byte_perm(sm0, 0, 0x3232);
        const uint32_t s1 = __byte_perm(sm1, 0, 0x1010), m1 = __byte_perm(sm1, 0, 0x3232);
#pragma unroll
        for (int h2 = 0; h2 < 2; ++h2) {
          const int kk = 2 * gi + h2;
          const uint32_t a0 = q4_byte_to_f16x2(r0[8 * kk + c], s0, m0);
          const uint32_t a1 = q4_byte_to_f16x2(r1[8 * kk + c], s1, m1);
          const uint32_t a2 = q4_byte_to_f16x2(r0[8 * kk + c + 4], s0, m0);
          const uint32_t a3 = q4_byte_to_f16x2(r1[8 * kk + c + 4], s1, m1);
          mma_f16_m16n8k16(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
        }
      }
    }
    // sc[0] = (token g, head 2c), [1] = (g, 2c+1), [2] = (g+8, 2c), [3] = (g+8, 2c+1)
    const int tok0 = p * kPage;
    float x[4] = {sc[0] * scale_log2, sc[1] * scale_log2, sc[2] * scale_log2, sc[3] * scale_log2};
    if (tok0 + g >= ctx) x[0] = x[1] = -INFINITY;
    if (tok0 + g + 8 >= ctx) x[2] = x[3] = -INFINITY;
    float mx[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 4));
      mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 8));
      mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], 16));
    }
    float alpha[2], m_new[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      m_new[j] = fmaxf(m_run[j], mx[j]);
      alpha[j] = (m_new[j] == -INFINITY) ? 1.f : exp2f(m_run[j] - m_new[j]);
    }
    float pr[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pr[i] = (m_new[i & 1] == -INFINITY) ? 0.f : exp2f(x[i] - m_new[i & 1]);
    float rs[2] = {pr[0] + pr[2], pr[1] + pr[3]};
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      rs[j] += __shfl_xor_sync(0xffffffffu, rs[j], 4);
      rs[j] += __shfl_xor_sync(0xffffffffu, rs[j], 8);
      rs[j] += __shfl_xor_sync(0xffffffffu, rs[j], 16);
      l_run[j] = l_run[j] * alpha[j] + rs[j];
      m_run[j] = m_new[j];
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      o[mt][0] *= alpha[0];
      o[mt][1] *= alpha[1];
      o[mt][2] *= alpha[0];
      o[mt][3] *= alpha[1];
    }
    // P^T as the B operand (k = tokens, n = heads): transpose the two 8x8 16-bit blocks
    uint32_t pb0, pb1;
    if constexpr (FMT == kFmtBf16) {
      movmatrix_trans(pack_bf16x2(pr[0], pr[1]), pb0);
      movmatrix_trans(pack_bf16x2(pr[2], pr[3]), pb1);
    } else {
      movmatrix_trans(pack_f16x2(pr[0], pr[1]), pb0);
      movmatrix_trans(pack_f16x2(pr[2], pr[3]), pb1);
    }
    // O^T += V^T P^T: A = V^T (dims x tokens) from the V tile with transposing loads
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      const int row = (lane & 7) + (lane >> 4) * 8;
      const int ch = 2 * mt + ((lane >> 3) & 1);
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(vaddr + swz<ROWB>(row, ch), a0, a1, a2, a3);
      if constexpr (FMT == kFmtBf16) mma_bf16_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
      else mma_f16_m16n8k16(o[mt], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  __syncthreads();

  // ---- merge the 4 warps (row stride D + 4: the transposed stores hit distinct banks)
  constexpr int kOS = D + 4;
  float* s_o = reinterpret_cast<float*>(smem);   // [4][8][D + 4]
  if (g == 0) {
    s_m[warp][2 * c] = m_run[0];
    s_m[warp][2 * c + 1] = m_run[1];
    s_l[warp][2 * c] = l_run[0];
    s_l[warp][2 * c + 1] = l_run[1];
  }
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) {
    float* r0 = s_o + (warp * 8 + 2 * c) * kOS + mt * 16 + g;
    r0[0] = o[mt][0];
    r0[kOS] = o[mt][1];
    r0[8] = o[mt][2];
    r0[kOS + 8] = o[mt][3];
  }
  __syncthreads();

  const size_t grp = (size_t)b * KH + kvh;
  // cluster partials: past the warp-merge area (which is at most half the buffer)
  float* s_co = reinterpret_cast<float*>(smem + S::kTotal / 2);   // [G][D] normalised partial
  float* s_cm = s_co + 8 * D;                                    // [G] max
  float* s_cl = s_cm + 8;                                        // [G] sum
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < 4; ++w) M = fmaxf(M, s_m[w][h]);
    float L = 0.f, acc = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const float f = exp2f(s_m[w][h] - M);
        L += s_l[w][h] * f;
        acc += s_o[(w * 8 + h) * kOS + d] * f;
      }
    }
    if (nsplit == 1) {
      const float r = L > 0.f ? acc / L * v_scale : 0.f;
      P.out[(size_t)b * P.ld_o + (size_t)(kvh * G + h) * D + d] = __float2bfloat16(r);
    } else if (kCluster) {
      s_co[h * D + d] = L > 0.f ? acc / L : 0.f;
      if (d == 0) {
        s_cm[h] = M;
        s_cl[h] = L;
      }
    } else {
      P.ws_o[((grp * nsplit + split) * G + h) * D + d] = L > 0.f ? acc / L : 0.f;
      if (d == 0) {
        P.ws_ml[((grp * nsplit + split) * G + h) * 2 + 0] = M;
        P.ws_ml[((grp * nsplit + split) * G + h) * 2 + 1] = L;
      }
    }
  }
  if (nsplit == 1) return;

  if constexpr (kCluster) {
    // ---- every CTA of the cluster merges its slice of the G x D outputs from the
    // partials in its peers' shared memory
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    const int rank = (int)cluster.block_rank();
    const int n = G * D;
    const int per = (n + nsplit - 1) / nsplit;
    const int i0 = rank * per, i1 = min(n, i0 + per);
    for (int idx = i0 + threadIdx.x; idx < i1; idx += blockDim.x) {
      const int h = idx / D;
      float M = -INFINITY;
      for (int q = 0; q < nsplit; ++q) M = fmaxf(M, cluster.map_shared_rank(s_cm, q)[h]);
      float L = 0.f, acc = 0.f;
      if (M != -INFINITY) {
        for (int q = 0; q < nsplit; ++q) {
          const float w = cluster.map_shared_rank(s_cl, q)[h] * exp2f(cluster.map_shared_rank(s_cm, q)[h] - M);
          L += w;
          acc += w * cluster.map_shared_rank(s_co, q)[idx];
        }
      }
      const float r = L > 0.f ? acc / L * v_scale : 0.f;
      P.out[(size_t)b * P.ld_o + (size_t)(kvh * G) * D + idx] = __float2bfloat16(r);
    }
    cluster.sync();     // peers' shared memory stays valid until every CTA has read it
    return;
  }

  // ---- the last CTA of this (sequence, kv head) merges the splits
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&P.counters[grp], 1u);
    s_last = (prev == (uint32_t)(nsplit - 1)) ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // stage every split's (max, sum) in shared memory with parallel loads, turn them
  // into merge weights, then each output element sums independent loads
  float* s_w = reinterpret_cast<float*>(smem);          // [nsplit][G] maxima, then weights
  float* s_ls = s_w + nsplit * G;                       // [nsplit][G] sums
  float* s_L = s_ls + nsplit * G;                       // [G] totals
  const float* ml = P.ws_ml + grp * nsplit * G * 2;
  for (int i = threadIdx.x; i < nsplit * G; i += blockDim.x) {
    s_w[i] = __ldcg(ml + 2 * i);
    s_ls[i] = __ldcg(ml + 2 * i + 1);
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int h = threadIdx.x;
    float M = -INFINITY;
    for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, s_w[sp * G + h]);
    float L = 0.f;
    for (int sp = 0; sp < nsplit; ++sp) {
      const float w = (M == -INFINITY) ? 0.f : s_ls[sp * G + h] * exp2f(s_w[sp * G + h] - M);
      s_w[sp * G + h] = w;
      L += w;
    }
    s_L[h] = L;
  }
  __syncthreads();
  const float* po = P.ws_o + grp * nsplit * G * D;
  for (int idx = threadIdx.x; idx < G * D; idx += blockDim.x) {
    const int h = idx / D, d = idx % D;
    float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
    int sp = 0;
    for (; sp + 3 < nsplit; sp += 4) {
      const float o0 = __ldcg(po + ((size_t)(sp + 0) * G + h) * D + d);
      const float o1 = __ldcg(po + ((size_t)(sp + 1) * G + h) * D + d);
      const float o2 = __ldcg(po + ((size_t)(sp + 2) * G + h) * D + d);
      const float o3 = __ldcg(po + ((size_t)(sp + 3) * G + h) * D + d);
      a0 += s_w[(sp + 0) * G + h] * o0;
      a1 += s_w[(sp + 1) * G + h] * o1;
      a2 += s_w[(sp + 2) * G + h] * o2;
      a3 += s_w[(sp + 3) * G + h] * o3;
    }
    for (; sp < nsplit; ++sp) a0 += s_w[sp * G + h] * __ldcg(po + ((size_t)sp * G + h) * D + d);
    const float L = s_L[h];
    const float r = L > 0.f ? (a0 + a1 + a2 + a3) / L * v_scale : 0.f;
    P.out[(size_t)b * P.ld_o + (size_t)(kvh * G + h) * D + d] = __float2bfloat16(r);
  }
  if (threadIdx.x == 0) P.counters[grp] = 0u;
}

// ============================================================== decode, persistent + TMA (bf16 pages)
// Work items are (page chunk, sequence, KV head), chunk-major so that every CTA's share
// mixes sequences; CTAs walk them round-robin.  Warp 4 is the producer: one thread
// issues the 2D tensor loads (128-byte swizzle) of each page's K and V tiles into an
// 8-stage mbarrier ring, running ahead across item boundaries, and waits for the
// previous kernel only before the first page that kernel writes (the live page).
// Warps 0-3 take the item's pages round-robin with the same transposed MMA math as
// paged_decode_kernel, merge through shared memory at the end of each item, and the
// CTA finishing a sequence's last chunk merges the chunk partials.
template <int D>
struct DecodeTmaSmem {
  static constexpr int kBoxB = kPage * 128;                // one 16 x 64 bf16 box
  static constexpr int kTileB = kPage * D * 2;             // 16 x D tile (D / 64 boxes)
  static constexpr int kStageB = 2 * kTileB;               // K + V
  static constexpr int kStages = 8;
  static constexpr int kRingB = kStages * kStageB;
  static constexpr int kMergeB = 4 * 8 * (D + 4) * 4;
  static constexpr int kTotal = kRingB + kMergeB + 2 * kStages * 8 + 1024;
};

// byte offset of 16-byte chunk ch of row r in a tile made of 128-byte-swizzled boxes
__device__ __forceinline__ uint32_t swz_box(int r, int ch) {
  return (uint32_t)((ch >> 3) * (kPage * 128) + r * 128 + (((ch & 7) ^ (r & 7)) << 4));
}

struct DecodeTmaParams {
  const __nv_bfloat16* q;
  int64_t ld_q;
  int layer, num_layers, KH, G, B;
  const int* block_tables;
  int bt_stride;
  const int* context_lens;
  float sm_scale;
  __nv_bfloat16* out;
  int64_t ld_o;
  float* ws_o;
  float* ws_ml;
  uint32_t* counters;
  int chunk_pages, max_chunks;
  uint32_t* err;
};

struct DecodeItem {
  int b, kvh, c, p0, p1, nchunks;
};

__device__ __forceinline__ bool decode_item(const DecodeTmaParams& P, int w, DecodeItem& it) {
  const int per = P.B * P.KH;
  it.c = w / per;
  const int rem = w - it.c * per;
  it.b = rem / P.KH;
  it.kvh = rem - it.b * P.KH;
  const int ctx = P.context_lens[it.b];
  const int npages = (ctx + kPage - 1) / kPage;
  it.nchunks = min(P.max_chunks, (npages + P.chunk_pages - 1) / P.chunk_pages);
  if (it.c >= it.nchunks) return false;
  it.p0 = it.c * P.chunk_pages;
  it.p1 = it.c == it.nchunks - 1 ? npages : it.p0 + P.chunk_pages;   // the last chunk takes the rest
  return true;
}

template <int D>
__global__ void __launch_bounds__(160, 1) paged_decode_tma_kernel(const __grid_constant__ CUtensorMap kvmap,
                                                                   DecodeTmaParams P) {
  using S = DecodeTmaSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* ring = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  float* s_o = reinterpret_cast<float*>(ring + S::kRingB);     // [4][8][D + 4]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S::kRingB + S::kMergeB);
  uint64_t* empty = full + S::kStages;
  __shared__ float s_m[4][8], s_l[4][8];
  __shared__ uint32_t s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = P.G, KH = P.KH;
  const int total = P.B * KH * P.max_chunks;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&kvmap);
    for (int s = 0; s < S::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == 4) {
    // ---------------- producer: the warp fetches up to 32 block-table entries at once
    // (one per lane), lane 0 issues the loads
    const uint64_t pol = policy_evict_first();
    bool waited = false;
    long long g = 0;
    for (int w = blockIdx.x; w < total; w += gridDim.x) {
      DecodeItem it;
      if (!decode_item(P, w, it)) continue;
      const int* bt = P.block_tables + (size_t)it.b * P.bt_stride;
      const int live = (P.context_lens[it.b] - 1) / kPage;
      for (int pb = it.p0; pb < it.p1; pb += 32) {
        const int n = min(32, it.p1 - pb);
        const int my_page = lane < n ? bt[pb + lane] : 0;
        for (int j = 0; j < n; ++j, ++g) {
          const long long page = __shfl_sync(0xffffffffu, my_page, j);
          int fail = 0;
          if (lane == 0) {
            const int s = (int)(g % S::kStages);
            if (g >= S::kStages && !mbar_wait(&empty[s], (uint32_t)(((g / S::kStages) & 1) ^ 1), P.err)) {
              fail = 1;
            } else {
              if (pb + j == live && !waited) {
                pdl_wait();          // the previous kernel writes this page (this step's token)
                waited = true;
              }
              const int row_k = (int)(((page * P.num_layers + P.layer) * 2 * KH + it.kvh) * kPage);
              const int row_v = row_k + KH * kPage;
              uint8_t* dst = ring + s * S::kStageB;
              mbar_arrive_expect_tx(&full[s], S::kStageB);
#pragma unroll
              for (int q = 0; q < D / 64; ++q) {
                tma_load_2d(dst + q * S::kBoxB, &kvmap, &full[s], q * 64, row_k, pol);
                tma_load_2d(dst + S::kTileB + q * S::kBoxB, &kvmap, &full[s], q * 64, row_v, pol);
              }
            }
          }
          if (__shfl_sync(0xffffffffu, fail, 0)) return;
        }
      }
    }
    return;
  }

  // ---------------- consumers: warps 0-3
  pdl_wait();
  const int g8 = lane >> 2, c = lane & 3;
  const float scale_log2 = P.sm_scale * 1.4426950408889634f;
  long long g_base = 0;
  bool ok = true;
  for (int w = blockIdx.x; w < total; w += gridDim.x) {
    DecodeItem it;
    if (!decode_item(P, w, it)) continue;
    const int b = it.b, kvh = it.kvh;
    const int ctx = P.context_lens[b];
    const int npg = it.p1 - it.p0;
    uint32_t qb[D / 16][2];
    {
      const __nv_bfloat16* qrow = P.q + (size_t)b * P.ld_q + (size_t)(kvh * G + g8) * D;
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        if (g8 < G) {
          qb[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * c);
          qb[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * c);
        } else {
          qb[kk][0] = qb[kk][1] = 0u;
        }
      }
    }
    float o[D / 16][4];
#pragma unroll
    for (int i = 0; i < D / 16; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};

    for (int j = warp; j < npg; j += 4) {
      const long long gp = g_base + j;
      const int s = (int)(gp % S::kStages);
      if (ok && !mbar_wait(&full[s], (uint32_t)((gp / S::kStages) & 1), P.err)) ok = false;
      if (ok) {
        const uint32_t kaddr = smem_u32(ring + s * S::kStageB), vaddr = kaddr + S::kTileB;
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const int row = (lane & 7) + ((lane >> 3) & 1) * 8;
          const int ch = 2 * kk + (lane >> 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4(kaddr + swz_box(row, ch), a0, a1, a2, a3);
          mma_bf16_16816(sc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
        }
        const int tok0 = (it.p0 + j) * kPage;
        float x[4] = {sc[0] * scale_log2, sc[1] * scale_log2, sc[2] * scale_log2, sc[3] * scale_log2};
        if (tok0 + g8 >= ctx) x[0] = x[1] = -INFINITY;
        if (tok0 + g8 + 8 >= ctx) x[2] = x[3] = -INFINITY;
        float mx[2] = {fmaxf(x[0], x[2]), fmaxf(x[1], x[3])};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], 4));
          mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], 8));
          mx[q] = fmaxf(mx[q], __shfl_xor_sync(0xffffffffu, mx[q], 16));
        }
        float alpha[2], m_new[2];
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          m_new[q] = fmaxf(m_run[q], mx[q]);
          alpha[q] = (m_new[q] == -INFINITY) ? 1.f : exp2f(m_run[q] - m_new[q]);
        }
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pr[i] = (m_new[i & 1] == -INFINITY) ? 0.f : exp2f(x[i] - m_new[i & 1]);
        float rs[2] = {pr[0] + pr[2], pr[1] + pr[3]};
#pragma unroll
        for (int q = 0; q < 2; ++q) {
          rs[q] += __shfl_xor_sync(0xffffffffu, rs[q], 4);
          rs[q] += __shfl_xor_sync(0xffffffffu, rs[q], 8);
          rs[q] += __shfl_xor_sync(0xffffffffu, rs[q], 16);
          l_run[q] = l_run[q] * alpha[q] + rs[q];
          m_run[q] = m_new[q];
        }
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          o[mt][0] *= alpha[0];
          o[mt][1] *= alpha[1];
          o[mt][2] *= alpha[0];
          o[mt][3] *= alpha[1];
        }
        uint32_t pb0, pb1;
        movmatrix_trans(pack_bf16x2(pr[0], pr[1]), pb0);
        movmatrix_trans(pack_bf16x2(pr[2], pr[3]), pb1);
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int row = (lane & 7) + (lane >> 4) * 8;
          const int ch = 2 * mt + ((lane >> 3) & 1);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_t(vaddr + swz_box(row, ch), a0, a1, a2, a3);
          mma_bf16_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);     // stage free for the producer
    }
    g_base += npg;

    // ---- merge the 4 warps of this item
    constexpr int kOS = D + 4;
    asm volatile("bar.sync 1, 128;" ::: "memory");
    if (g8 == 0) {
      s_m[warp][2 * c] = m_run[0];
      s_m[warp][2 * c + 1] = m_run[1];
      s_l[warp][2 * c] = l_run[0];
      s_l[warp][2 * c + 1] = l_run[1];
    }
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt) {
      float* r0 = s_o + (warp * 8 + 2 * c) * kOS + mt * 16 + g8;
      r0[0] = o[mt][0];
      r0[kOS] = o[mt][1];
      r0[8] = o[mt][2];
      r0[kOS + 8] = o[mt][3];
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    const int nsplit = it.nchunks, split = it.c;
    const size_t grp = (size_t)b * KH + kvh;
    for (int idx = threadIdx.x; idx < G * D; idx += 128) {
      const int h = idx / D, d = idx % D;
      float M = -INFINITY;
#pragma unroll
      for (int q = 0; q < 4; ++q) M = fmaxf(M, s_m[q][h]);
      float L = 0.f, acc = 0.f;
      if (M != -INFINITY) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float f = exp2f(s_m[q][h] - M);
          L += s_l[q][h] * f;
          acc += s_o[(q * 8 + h) * kOS + d] * f;
        }
      }
      if (nsplit == 1) {
        P.out[(size_t)b * P.ld_o + (size_t)(kvh * G + h) * D + d] = __float2bfloat16(L > 0.f ? acc / L : 0.f);
      } else {
        P.ws_o[((grp * P.max_chunks + split) * G + h) * D + d] = L > 0.f ? acc / L : 0.f;
        if (d == 0) {
          P.ws_ml[((grp * P.max_chunks + split) * G + h) * 2 + 0] = M;
          P.ws_ml[((grp * P.max_chunks + split) * G + h) * 2 + 1] = L;
        }
      }
    }
    if (nsplit > 1) {
      // the CTA finishing this sequence's last chunk merges the chunk partials
      __threadfence();
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 0) {
        const uint32_t prev = atomicAdd(&P.counters[grp], 1u);
        s_last = (prev == (uint32_t)(nsplit - 1)) ? 1u : 0u;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (s_last) {
        __threadfence();
        float* s_w = s_o;                          // [nsplit][G] maxima, then weights
        float* s_ls = s_w + nsplit * G;            // [nsplit][G] sums
        float* s_L = s_ls + nsplit * G;            // [G] totals
        const float* ml = P.ws_ml + grp * P.max_chunks * G * 2;
        for (int i = threadIdx.x; i < nsplit * G; i += 128) {
          s_w[i] = __ldcg(ml + 2 * i);
          s_ls[i] = __ldcg(ml + 2 * i + 1);
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x < G) {
          const int h = threadIdx.x;
          float M = -INFINITY;
          for (int sp = 0; sp < nsplit; ++sp) M = fmaxf(M, s_w[sp * G + h]);
          float L = 0.f;
          for (int sp = 0; sp < nsplit; ++sp) {
            const float wv = (M == -INFINITY) ? 0.f : s_ls[sp * G + h] * exp2f(s_w[sp * G + h] - M);
            s_w[sp * G + h] = wv;
            L += wv;
          }
          s_L[h] = L;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");
        const float* po = P.ws_o + grp * P.max_chunks * G * D;
        for (int idx = threadIdx.x; idx < G * D; idx += 128) {
          const int h = idx / D, d = idx % D;
          float a0 = 0.f, a1 = 0.f;
          int sp = 0;
          for (; sp + 1 < nsplit; sp += 2) {
            a0 += s_w[sp * G + h] * __ldcg(po + ((size_t)sp * G + h) * D + d);
            a1 += s_w[(sp + 1) * G + h] * __ldcg(po + ((size_t)(sp + 1) * G + h) * D + d);
          }
          if (sp < nsplit) a0 += s_w[sp * G + h] * __ldcg(po + ((size_t)sp * G + h) * D + d);
          const float L = s_L[h];
          P.out[(size_t)b * P.ld_o + (size_t)(kvh * G + h) * D + d] = __float2bfloat16(L > 0.f ? (a0 + a1) / L : 0.f);
        }
        if (threadIdx.x == 0) P.counters[grp] = 0u;
      }
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");   // merge area free for the next item
  }
}

// ============================================================== prefill
template <int D, int FMT>
struct PrefillSmem {
  static constexpr int kRows = 64;
  static constexpr int kQB = kRows * D * 2;
  static constexpr int kTileB = kRows * D * 2;
  static constexpr int kRawB = kRows * PageRow<D, FMT>::kBytes;
  static constexpr int kStageB = 2 * kRawB;
  static constexpr int kTotal = kQB + 2 * kStageB + (FMT != kFmtBf16 ? 2 * kTileB : 0);
};

struct PrefillParams {
  const __nv_bfloat16* q;
  int64_t ld_q;
  const uint8_t* cache;
  int layer, num_layers, KH, G;
  const int* block_tables;
  int bt_stride;
  const int* cu_q;
  const int* context_lens;
  const float* kv_scale;
  float sm_scale;
  __nv_bfloat16* out;
  int64_t ld_o;
  long long num_pages;       // pool pages (checked in bounds-check builds)
  uint32_t* err;
};

template <int D, int FMT>
__global__ void __launch_bounds__(128) paged_prefill_kernel(PrefillParams P) {
  pdl_launch();
  pdl_wait();
  using S = PrefillSmem<D, FMT>;
  constexpr bool kFp8 = FMT == kFmtFp8;
  constexpr int ROWB = D * 2;
  constexpr int kChunkPerRow = D * 2 / 16;   // bf16 pages: swizzled 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];

  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q_start = P.cu_q[b];
  const int q_len = P.cu_q[b + 1] - q_start;
  const int q0 = qt * 64;
  if (q0 >= q_len) return;
  const int ctx = P.context_lens[b];
  const int prefix = ctx - q_len;   // tokens already in the cache before this chunk
  const int KH = P.KH;
  const int kvh = h / P.G;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;

  float k_scale = 1.f, v_scale = 1.f;
  if (kFp8) {
    k_scale = P.kv_scale[(P.layer * 2 + 0) * KH + kvh];
    v_scale = P.kv_scale[(P.layer * 2 + 1) * KH + kvh];
  }
  const float scale_log2 = P.sm_scale * 1.4426950408889634f * k_scale;

  uint8_t* sq = smem;
  uint8_t* stages = smem + S::kQB;
  const uint32_t sq_addr = smem_u32(sq);

  // Q tile -> smem (rows past q_len zero-filled)
  for (int i = threadIdx.x; i < 64 * (D / 8); i += 128) {
    const int r = i / (D / 8), ch = i % (D / 8);
    const bool valid = q0 + r < q_len;
    const __nv_bfloat16* src = P.q + (size_t)(q_start + (valid ? q0 + r : 0)) * P.ld_q + (size_t)h * D + ch * 8;
    cp_async16(sq_addr + swz<ROWB>(r, ch), src, valid);
  }
  cp_async_commit();

  const int kv_end = min(ctx, prefix + q0 + 64);
  const int nchunks = (kv_end + 63) / 64;
  const int* bt = P.block_tables + (size_t)b * P.bt_stride;
  constexpr int kPageB = kPage * PageRow<D, FMT>::kBytes;
  const size_t head_stride = (size_t)kPageB;
  const size_t page_stride = (size_t)P.num_layers * 2 * KH * head_stride;

  auto issue = [&](int chunk, int stage) {
    uint8_t* dst = stages + stage * S::kStageB;
    const uint32_t dk = smem_u32(dst), dv = smem_u32(dst + S::kRawB);
    constexpr int kPageChunks = kPageB / 16;
    for (int i = threadIdx.x; i < 4 * kPageChunks; i += 128) {
      const int pg = i / kPageChunks, w = i % kPageChunks;
      const int page_local = chunk * 4 + pg;
      const bool valid = page_local * kPage < ctx;
      int page = valid ? bt[page_local] : 0;
      if (!in_bounds(page, P.num_pages, P.err)) page = 0;   // bounds-check builds
      const uint8_t* kp = P.cache + (size_t)page * page_stride + (((size_t)P.layer * 2 + 0) * KH + kvh) * head_stride;
      const uint8_t* vp = kp + (size_t)KH * head_stride;
      const uint32_t off = FMT == kFmtBf16 ? swz<ROWB>(pg * kPage + w / kChunkPerRow, w % kChunkPerRow)
                                           : (uint32_t)(pg * kPageB + w * 16);
      cp_async16(dk + off, kp + (size_t)w * 16, valid);
      cp_async16(dv + off, vp + (size_t)w * 16, valid);
    }
  };

  issue(0, 0);
  cp_async_commit();
  cp_async_wait<1>();
  __syncthreads();

  // Q fragments for this warp's 16 rows
  uint32_t qf[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int row = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
    const int ch = 2 * kk + (lane >> 4);
    ldsm_x4(sq_addr + swz<ROWB>(row, ch), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
  }

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  const int qrow0 = q0 + warp * 16 + g;   // query index within the sequence's new tokens
  const int qpos[2] = {prefix + qrow0, prefix + qrow0 + 8};

  for (int ck = 0; ck < nchunks; ++ck) {
    const int stage = ck & 1;
    if (ck + 1 < nchunks) issue(ck + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    uint8_t* kt = stages + stage * S::kStageB;
    uint8_t* vt = kt + S::kRawB;
    if constexpr (FMT != kFmtBf16) {
      uint8_t* ckb = stages + 2 * S::kStageB;
      uint8_t* cvb = ckb + S::kTileB;
      if constexpr (FMT == kFmtFp8) {
        convert_fp8_tile<D>(kt, ckb, 64, threadIdx.x, 128);
        convert_fp8_tile<D>(vt, cvb, 64, threadIdx.x, 128);
      } else {
        convert_q4_tile<D>(kt, ckb, 64, threadIdx.x, 128);
        convert_q4_tile<D>(vt, cvb, 64, threadIdx.x, 128);
      }
      __syncthreads();
      kt = ckb;
      vt = cvb;
    }
    const uint32_t kaddr = smem_u32(kt), vaddr = smem_u32(vt);

    float s[8][4];
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int nt = 0; nt < 8; nt += 2) {
        const int j = lane >> 3;
        const int row = nt * 8 + (lane & 7) + (j >> 1) * 8;
        const int ch = 2 * kk + (j & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kaddr + swz<ROWB>(row, ch), b0, b1, b2, b3);
        mma_bf16_16816(s[nt], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b0, b1);
        mma_bf16_16816(s[nt + 1], qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3], b2, b3);
      }
    }
    const int key0 = ck * 64;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + nt * 8 + 2 * c + (e & 1);
        const int r = e >> 1;
        float v = s[nt][e] * scale_log2;
        if (key > qpos[r] || key >= ctx) v = -INFINITY;
        s[nt][e] = v;
        mx[r] = fmaxf(mx[r], v);
      }
    }
    float alpha[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mn = fmaxf(m_run[r], mx[r]);
      alpha[r] = (mn == -INFINITY) ? 1.f : exp2f(m_run[r] - mn);
      m_run[r] = mn;
    }
    float rs[2] = {0.f, 0.f};
#pragma unroll
    for (int nt = 0; nt < 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = e >> 1;
        const float pv = (m_run[r] == -INFINITY) ? 0.f : exp2f(s[nt][e] - m_run[r]);
        s[nt][e] = pv;
        rs[r] += pv;
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 1);
      rs[r] += __shfl_xor_sync(0xffffffffu, rs[r], 2);
      l_run[r] = l_run[r] * alpha[r] + rs[r];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= alpha[0];
      o[i][1] *= alpha[0];
      o[i][2] *= alpha[1];
      o[i][3] *= alpha[1];
    }
#pragma unroll
    for (int kt2 = 0; kt2 < 4; ++kt2) {
      const uint32_t a0 = pack_bf16x2(s[2 * kt2][0], s[2 * kt2][1]);
      const uint32_t a1 = pack_bf16x2(s[2 * kt2][2], s[2 * kt2][3]);
      const uint32_t a2 = pack_bf16x2(s[2 * kt2 + 1][0], s[2 * kt2 + 1][1]);
      const uint32_t a3 = pack_bf16x2(s[2 * kt2 + 1][2], s[2 * kt2 + 1][3]);
#pragma unroll
      for (int nd = 0; nd < D / 8; nd += 2) {
        const int j = lane >> 3;
        const int row = kt2 * 16 + (lane & 7) + (j & 1) * 8;
        const int ch = nd + (j >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vaddr + swz<ROWB>(row, ch), b0, b1, b2, b3);
        mma_bf16_16816(o[nd], a0, a1, a2, a3, b0, b1);
        mma_bf16_16816(o[nd + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qrow0 + r * 8;
    if (qi >= q_len) continue;
    const float inv = l_run[r] > 0.f ? v_scale / l_run[r] : 0.f;
    __nv_bfloat16* orow = P.out + (size_t)(q_start + qi) * P.ld_o + (size_t)h * D;
#pragma unroll
    for (int nd = 0; nd < D / 8; ++nd)
      *reinterpret_cast<uint32_t*>(orow + nd * 8 + 2 * c) = pack_bf16x2(o[nd][2 * r] * inv, o[nd][2 * r + 1] * inv);
  }
}

// ============================================================== prefill on tcgen05
// Causal paged prefill with the 5th-generation tensor cores, bf16 pages.  One CTA per
// (128-query tile, query head, sequence); keys in blocks of 128 (8 pages).
//   warp 0      TMA: the Q tile once, then each block's K and V page chunks (16 rows x 64
//               dims boxes, 128-byte swizzle) into a 2-stage ring
//   warp 1      MMA issuer: S_j = Q K_j^T into one of two TMEM score buffers (128 cols),
//               then O_j = P_j V_j into one of two TMEM output buffers (D cols), V read
//               as an MN-major operand straight from its TMA layout
//   warps 2-9   two warps per TMEM lane quarter, one query row per thread, each warp of
//               a pair owning half the key columns and half the output dims: scores ->
//               online softmax (row max / sum exchanged within the pair) -> P_j (bf16,
//               K-major, 128-byte swizzle) in shared memory; then its half of O_j from
//               TMEM into a register accumulator rescaled by the running max
// S_{j+1} runs on the tensor cores while the softmax of block j runs, and O_j while the
// softmax of block j+1 runs.  Query tiles are taken last-first (the diagonal-heavy
// tiles start first).  The mma.sync kernel above stays for fp8 / four-bit pages.
template <int D>
struct PrefillTcSmem {
  static constexpr int kQ = 128 * D * 2;             // Q tile [128, D] (D/64 swizzle columns)
  static constexpr int kP = 128 * 128 * 2;           // P tile [128 q, 128 keys]
  static constexpr int kKV = 128 * D * 2;            // one K (or V) block [128 keys, D]
  static constexpr int kStages = 2;
  static constexpr int kPOff = kQ;
  static constexpr int kKVOff = kPOff + 2 * kP;
  static constexpr int kBarOff = kKVOff + kStages * 2 * kKV;
  // q_full, kv_full[2], kv_empty[2], s_full[2], s_empty[2], p_full[2], o_full[2], o_empty[2],
  // tmem slot (16 B), softmax pair exchange [2 halves][128 rows] fp32 (max, then sum)
  static constexpr int kTotal = kBarOff + 16 * 8 + 16 + 2 * 128 * 4;
  static constexpr int kAlloc = kTotal + 1024;
  static constexpr uint32_t kTmemCols = 512;         // S x 2 (256) + O x 2 (2 D <= 256)
};

struct PrefillTcParams {
  const int* block_tables;
  int bt_stride;
  const int* cu_q;
  const int* context_lens;
  int layer, num_layers, KH, G, Hq;
  float sm_scale;
  __nv_bfloat16* out;
  int64_t ld_o;
  int max_tiles;
  long long num_pages;
  uint32_t* err;
};

// MN-major operand, 128-byte swizzle: 64-element (128 B) MN blocks lbo bytes apart,
// 8-row K groups sbo bytes apart
__device__ __forceinline__ uint64_t make_mn_sw128_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

template <int D>
__global__ void __launch_bounds__(320, 1) paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                   const __grid_constant__ CUtensorMap kvmap,
                                                                   PrefillTcParams P) {
  using S = PrefillTcSmem<D>;
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = bars + 3;
  uint64_t* s_full = bars + 5;
  uint64_t* s_empty = bars + 7;
  uint64_t* p_full = bars + 9;
  uint64_t* o_full = bars + 11;
  uint64_t* o_empty = bars + 13;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  const int b = blockIdx.z, h = blockIdx.y;
  const int q_start = P.cu_q[b];
  const int q_len = P.cu_q[b + 1] - q_start;
  const int ntiles = (q_len + 127) / 128;
  const int qt = ntiles - 1 - (int)blockIdx.x;   // the longest (diagonal-heavy) tiles first
  if (qt < 0) return;
  const int q0 = qt * 128;
  const int ctx = P.context_lens[b];
  const int prefix = ctx - q_len;
  const int kvh = h / P.G;
  const int kv_end = min(ctx, prefix + q0 + 128);
  const int nblk = (kv_end + 127) / 128;
  const int npages = (ctx + kPage - 1) / kPage;
  const int* bt = P.block_tables + (size_t)b * P.bt_stride;

  pdl_launch();
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kvmap);
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 256);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, S::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_s = tmem, t_o = tmem + 256;   // S[2] at columns 0 / 128, O[2] at 256 / 256 + D

  if (warp == 0 && lane == 0) {
    // ---------------- producer
    const uint64_t pol = policy_evict_normal();
    pdl_wait();   // q and this chunk's K / V come from the previous kernel
    mbar_arrive_expect_tx(q_full, S::kQ);
#pragma unroll
    for (int hh = 0; hh < D / 64; ++hh)
      tma_load_2d(smem + hh * (128 * 128), &qmap, q_full, h * D + hh * 64, q_start + q0, pol);
    for (int j = 0; j < nblk; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, P.err)) break;
      uint8_t* kb = smem + S::kKVOff + st * 2 * S::kKV;
      uint8_t* vb = kb + S::kKV;
      mbar_arrive_expect_tx(&kv_full[st], 2 * S::kKV);
#pragma unroll 1
      for (int pg = 0; pg < 8; ++pg) {
        const int pl = j * 8 + pg;
        int page = bt[pl < npages ? pl : npages - 1];   // past the context: any valid page (masked)
        if (!in_bounds(page, P.num_pages, P.err)) page = 0;
        const int row = (((page * P.num_layers + P.layer) * 2 + 0) * P.KH + kvh) * kPage;
        const int vrow = row + P.KH * kPage;
#pragma unroll
        for (int hh = 0; hh < D / 64; ++hh) {
          tma_load_2d(kb + hh * (128 * 128) + pg * (kPage * 128), &kvmap, &kv_full[st], hh * 64, row, pol);
          tma_load_2d(vb + hh * (128 * 128) + pg * (kPage * 128), &kvmap, &kv_full[st], hh * 64, vrow, pol);
        }
      }
    }
    // drain: none of our copies may be in flight at exit
    mbar_wait(q_full, 0, P.err);
    const int first = nblk > 2 ? nblk - 2 : 0;
    for (int j = first; j < nblk; ++j) mbar_wait(&kv_full[j & 1], (j >> 1) & 1, P.err);
  } else if (warp == 1 && lane == 0) {
    // ---------------- MMA issuer
    constexpr uint32_t idesc_s = make_idesc_bf16(128, 128);
    constexpr uint32_t idesc_o = make_idesc_bf16(128, D) | (1u << 16);   // B (V) MN-major
    const uint32_t q_addr = smem_u32(smem);
    bool failed = !mbar_wait(q_full, 0, P.err);
    auto issue_s = [&](int j) {
      const int st = j & 1;
      if (!mbar_wait(&kv_full[st], (j >> 1) & 1, P.err) || !mbar_wait(&s_empty[st], ((j >> 1) & 1) ^ 1, P.err)) {
        failed = true;
        return;
      }
      tc_fence_after();
      const uint32_t kb = smem_u32(smem + S::kKVOff + st * 2 * S::kKV);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int hh = kk >> 2;
        const uint64_t da = make_sw128_desc(q_addr + hh * (128 * 128)) + (uint64_t)((kk & 3) * 2);
        const uint64_t db = make_sw128_desc(kb + hh * (128 * 128)) + (uint64_t)((kk & 3) * 2);
        umma_f16(t_s + st * 128, da, db, idesc_s, kk > 0 ? 1u : 0u);
      }
      umma_commit(&s_full[st]);
    };
    if (!failed && nblk > 0) issue_s(0);
    for (int j = 0; j < nblk && !failed; ++j) {
      if (j + 1 < nblk) issue_s(j + 1);
      if (failed) break;
      const int st = j & 1;
      if (!mbar_wait(&p_full[st], (j >> 1) & 1, P.err) || !mbar_wait(&o_empty[st], ((j >> 1) & 1) ^ 1, P.err)) {
        failed = true;
        break;
      }
      tc_fence_after();
      const uint32_t pa = smem_u32(smem + S::kPOff + st * S::kP);
      const uint32_t vb = smem_u32(smem + S::kKVOff + st * 2 * S::kKV + S::kKV);
#pragma unroll
      for (int kk = 0; kk < 128 / 16; ++kk) {
        const uint64_t da = make_sw128_desc(pa + (kk >> 2) * (128 * 128)) + (uint64_t)((kk & 3) * 2);
        const uint64_t db = make_mn_sw128_desc(vb + kk * (16 * 128), 128 * 128, 1024);
        umma_f16(t_o + st * D, da, db, idesc_o, kk > 0 ? 1u : 0u);
      }
      umma_commit(&o_full[st]);
      umma_commit(&kv_empty[st]);   // K_j (read by S_j, issued earlier) and V_j are consumed
    }
  } else if (warp >= 2) {
    // ---------------- softmax + output accumulation: two warps per TMEM lane quarter,
    // warp half hf owns key columns [64 hf, 64 hf + 64) of S and output dims
    // [hf D/2, (hf + 1) D/2); the pair exchanges row maxima and sums in shared memory
    constexpr int DH = D / 2;
    const int quarter = warp & 3, hf = (warp - 2) >> 2;
    const int lb = 32 * quarter;
    const int r = lb + lane;
    const uint32_t lane_off = (uint32_t)lb << 16;
    const int qpos = prefix + q0 + r;
    const float sl2 = P.sm_scale * 1.4426950408889634f;
    float* red = reinterpret_cast<float*>(bars + 16) + 4;   // [2 halves][128 rows]: max, then sum
    auto pair_sync = [&]() { asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory"); };
    float m_run = -INFINITY, l_run = 0.f, alpha_prev = 1.f;
    float o[DH];
#pragma unroll
    for (int d = 0; d < DH; ++d) o[d] = 0.f;
    bool ok = true;
    // accumulate this warp's half of O_j (TMEM) into the registers: o = o * alpha + O_j
    auto take_o = [&](int j, float alpha) {
      const int st = j & 1;
      if (!mbar_wait(&o_full[st], (j >> 1) & 1, P.err)) ok = false;
      tc_fence_after();
#pragma unroll
      for (int c0 = 0; c0 < DH; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(t_o + st * D + hf * DH + lane_off + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; ++t) o[c0 + t] = o[c0 + t] * alpha + (ok ? __uint_as_float(v[t]) : 0.f);
      }
      tc_fence_before();
      mbar_arrive(&o_empty[st]);
    };
    for (int j = 0; j < nblk; ++j) {
      const int st = j & 1;
      if (!mbar_wait(&s_full[st], (j >> 1) & 1, P.err)) ok = false;
      tc_fence_after();
      const uint32_t srow = t_s + st * 128 + hf * 64 + lane_off;
      const int key0 = j * 128 + hf * 64;
      const bool need_mask = key0 + 63 > qpos || key0 + 64 > ctx;
      // pass 1: this half's maximum of the scaled, masked scores
      float mx = -INFINITY;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(srow + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int key = key0 + c0 + t;
          float x = __uint_as_float(v[t]) * sl2;
          if (need_mask && (key > qpos || key >= ctx)) x = -INFINITY;
          mx = fmaxf(mx, x);
        }
      }
      red[hf * 128 + r] = mx;
      pair_sync();
      const float m_new = fmaxf(m_run, fmaxf(mx, red[(hf ^ 1) * 128 + r]));
      pair_sync();                        // both maxima read before the slots take the sums
      const float alpha = (m_new == -INFINITY) ? 1.f : exp2f(m_run - m_new);
      // pass 2: P = exp2(s - m_new) -> this half of the bf16 K-major swizzled P rows
      uint8_t* half = smem + S::kPOff + st * S::kP + hf * (128 * 128) + (r >> 3) * 1024 + (r & 7) * 128;
      float sum = 0.f;
#pragma unroll
      for (int c0 = 0; c0 < 64; c0 += 16) {
        uint32_t v[16];
        tmem_ld_32x32b_x16(srow + c0, v);
        tmem_wait_ld();
        float pv[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) {
          const int key = key0 + c0 + t;
          float x = __uint_as_float(v[t]) * sl2;
          if (need_mask && (key > qpos || key >= ctx)) x = -INFINITY;
          pv[t] = (m_new == -INFINITY || !ok) ? 0.f : exp2f(x - m_new);
          sum += pv[t];
        }
        const int ch = c0 >> 3;
        uint4 w0, w1;
        w0.x = pack_bf16x2(pv[0], pv[1]);
        w0.y = pack_bf16x2(pv[2], pv[3]);
        w0.z = pack_bf16x2(pv[4], pv[5]);
        w0.w = pack_bf16x2(pv[6], pv[7]);
        w1.x = pack_bf16x2(pv[8], pv[9]);
        w1.y = pack_bf16x2(pv[10], pv[11]);
        w1.z = pack_bf16x2(pv[12], pv[13]);
        w1.w = pack_bf16x2(pv[14], pv[15]);
        *reinterpret_cast<uint4*>(half + ((ch ^ (r & 7)) << 4)) = w0;
        *reinterpret_cast<uint4*>(half + (((ch + 1) ^ (r & 7)) << 4)) = w1;
      }
      tc_fence_before();
      mbar_arrive(&s_empty[st]);          // the scores are read: the slot takes S_{j+2}
      fence_proxy_async_smem();           // P written by this thread -> visible to the MMA
      mbar_arrive(&p_full[st]);
      red[hf * 128 + r] = sum;
      pair_sync();
      l_run = l_run * alpha + sum + red[(hf ^ 1) * 128 + r];
      m_run = m_new;
      // O_{j-1} (finished while this block's softmax ran) into the accumulator
      if (j > 0) take_o(j - 1, alpha_prev);
      alpha_prev = alpha;
    }
    if (nblk > 0) take_o(nblk - 1, alpha_prev);
    // O_j is relative to the running max after block j; taking it with that block's
    // alpha keeps the accumulator (and l_run) relative to the final running max
    if (q0 + r < q_len && ok) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* orow = P.out + (size_t)(q_start + q0 + r) * P.ld_o + (size_t)h * D + hf * DH;
#pragma unroll
      for (int d = 0; d < DH; d += 8) {
        uint4 w;
        w.x = pack_bf16x2(o[d] * inv, o[d + 1] * inv);
        w.y = pack_bf16x2(o[d + 2] * inv, o[d + 3] * inv);
        w.z = pack_bf16x2(o[d + 4] * inv, o[d + 5] * inv);
        w.w = pack_bf16x2(o[d + 6] * inv, o[d + 7] * inv);
        *reinterpret_cast<uint4*>(orow + d) = w;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, S::kTmemCols);
  }
}

// ============================================================== host
static int cache_format(bool fp8, bool q4) { return q4 ? kFmtQ4 : fp8 ? kFmtFp8 : kFmtBf16; }

int decode_attention_choose_splits(int B, int KH, int max_pages) {
  // Chunks per sequence for the persistent kernel (2 resident CTAs per SM): about one
  // (sequence, head, chunk) item per resident CTA (an item's merge is serial work, so
  // fewer, longer items win), chunks of at least 4 pages.  The
  // per-(sequence, head, split) kernel of fp8 pages uses the same count as its splits.
  const int slots = device_sm_count() * 2;
  const int groups = std::max(1, B * KH);
  int s = slots / groups;                      // about one item per resident CTA
  s = std::min(s, std::max(1, max_pages / 4));
  // up to 2048 tokens, eight splits (at most 16 pages each) merge inside a thread-block
  // cluster, which beats more splits merged through global memory (B200, one KV head:
  // 6.4 us with 8 cluster splits vs 9.7 us with 8-16 global-merge splits)
  const char* e = std::getenv("VRM_DECODE_CLUSTER");
  if (s > 8 && max_pages <= 128 && !(e && e[0] == '0')) s = 8;
  return std::max(1, std::min(s, 64));
}

size_t decode_attention_scratch_bytes(int B, int Hq, int D, int splits) {
  if (splits <= 1) return 0;
  return ((size_t)B * Hq * splits * D + (size_t)B * Hq * splits * 2) * sizeof(float);
}

template <int D, int FMT, bool C = false>
static void launch_decode(dim3 grid, const DecodeParams& p, cudaStream_t st) {
  constexpr int smem = DecodeSmem<D, FMT>::kTotal;
  auto kern = paged_decode_kernel<D, FMT, C>;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev & 63] = true;
  }
  if (C) launch_kernel_cluster(kern, grid, dim3(128), dim3(1, 1, grid.z), (size_t)smem, st, p);
  else launch_kernel(kern, grid, dim3(128), (size_t)smem, st, p);
}

// split merge through a thread-block cluster (VRM_DECODE_CLUSTER=0 keeps the counter merge)
static bool decode_cluster_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VRM_DECODE_CLUSTER");
    return !(e && e[0] == '0');
  }();
  return on;
}

CUtensorMap make_kmajor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows);

// The persistent TMA kernel is opt-in (VRM_DECODE_TMA=1 or set_decode_tma): on B200 it
// measured 12.4 / 16.2 / 56.7 us against 8.6 / 14.6 / 48.8 us for paged_decode_kernel at
// batch 1 / 32 / 128 (ctx 560, 40 q / 8 kv heads), which already streams 5-6 TB/s.
static int g_decode_tma = -1;
void set_decode_tma(bool on) { g_decode_tma = on ? 1 : 0; }
static bool decode_tma_enabled() {
  if (g_decode_tma < 0) {
    const char* e = std::getenv("VRM_DECODE_TMA");
    g_decode_tma = (e && e[0] == '1') ? 1 : 0;
  }
  return g_decode_tma == 1;
}

template <int D>
static void launch_decode_tma(const CUtensorMap& map, const DecodeTmaParams& p, int grid, cudaStream_t st) {
  constexpr int smem = DecodeTmaSmem<D>::kTotal;
  auto kern = paged_decode_tma_kernel<D>;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev & 63] = true;
  }
  launch_kernel(kern, dim3(grid), dim3(160), (size_t)smem, st, map, p);
}

// L2 prefetch of the next GEMM's weights from the decode attention kernel (VRM_L2_PREFETCH=1;
// off by default: measured on B200, Qwen2.5-14B decode with the o_proj weights prefetched,
// batch 32 ran 2 % slower (4207 / 4155 vs 4122 / 4068 tok/s in alternating runs) and batch
// 1 1.7 % slower -- the prefetch competes with attention's own KV reads and the stream-K
// o_proj GEMM gains less from L2 than that costs)
static bool l2_prefetch_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VRM_L2_PREFETCH");
    return e && e[0] == '1';
  }();
  return on;
}

void paged_attention_decode(const DecodeAttnArgs& a, cudaStream_t st) {
  VRM_REQUIRE(a.D == 64 || a.D == 128, "decode attention: head_dim must be 64 or 128");
  VRM_REQUIRE(a.KH > 0 && a.Hq % a.KH == 0 && a.Hq / a.KH <= 8, "decode attention: GQA group must be <= 8 heads");
  VRM_REQUIRE(!a.cache_fp8 || a.kv_scale != nullptr, "decode attention: fp8 cache needs kv_scale");
  VRM_REQUIRE(!(a.cache_fp8 && a.cache_q4), "decode attention: one page format");
  if (a.B <= 0) return;
  const int G = a.Hq / a.KH;
  int splits = a.num_splits > 0 ? a.num_splits : decode_attention_choose_splits(a.B, a.KH, a.max_pages);
  splits = std::min(splits, 128);
  DecodeParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.ld_q = a.ld_q;
  p.cache = reinterpret_cast<const uint8_t*>(a.cache);
  p.layer = a.layer;
  p.num_layers = a.num_layers;
  p.KH = a.KH;
  p.G = G;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.context_lens = a.context_lens;
  p.kv_scale = a.kv_scale;
  p.sm_scale = a.sm_scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.ld_o = a.ld_o;
  p.ws_o = p.ws_ml = nullptr;
  p.counters = nullptr;
  p.positions = a.positions;
  p.cos_sin = a.cos_sin;
  p.slot_mapping = a.slot_mapping;
  p.cache_w = reinterpret_cast<uint8_t*>(const_cast<void*>(a.cache));
  p.Hq = a.Hq;
  p.num_pages = a.cache_pages;
  p.err = a.err ? a.err : error_word();
  p.pf = l2_prefetch_enabled() && a.l2_prefetch_bytes >= 16 ? reinterpret_cast<const uint8_t*>(a.l2_prefetch) : nullptr;
  p.pf_bytes = p.pf != nullptr ? (a.l2_prefetch_bytes & ~15ull) : 0ull;
  if (a.positions != nullptr) {
    VRM_REQUIRE(a.slot_mapping != nullptr, "decode attention: fused KV write needs slot_mapping");
    VRM_REQUIRE(a.cos_sin == nullptr || a.rot_dim == a.D, "decode attention: fused RoPE needs rot_dim == head_dim");
  }
  const int64_t pool_rows = a.cache_pages * a.num_layers * 2 * a.KH * kPage;
  const bool tma = !a.cache_fp8 && !a.cache_q4 && a.positions == nullptr && a.cache_pages > 0 && pool_rows < (int64_t)INT32_MAX &&
                   decode_tma_enabled() && (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0;
  const bool cluster = !tma && splits > 1 && splits <= 8 && a.ws == nullptr && decode_cluster_enabled();
  if (splits > 1 && !cluster) {
    const size_t need = decode_attention_scratch_bytes(a.B, a.Hq, a.D, splits);
    float* ws = a.ws;
    if (ws == nullptr) {
      ws = static_cast<float*>(workspace_get(need, st));
    } else {
      VRM_REQUIRE(a.ws_bytes >= need, "decode attention: caller scratch too small");
    }
    p.ws_o = ws;
    p.ws_ml = ws + (size_t)a.B * a.Hq * splits * a.D;
    VRM_REQUIRE((size_t)a.B * a.KH <= 32768, "decode attention: too many (sequence, kv head) groups");
    // counters: the upper half of the per-device array (GEMM split-K uses the lower half)
    p.counters = a.counters ? a.counters : tile_counters_get(st) + 32768;
  }
  // persistent TMA kernel: bf16 pages, row coordinates of the pool within int32
  if (tma) {
    if (splits > 1) VRM_REQUIRE(p.ws_o != nullptr && p.counters != nullptr, "decode attention: scratch");
    DecodeTmaParams t;
    t.q = p.q;
    t.ld_q = p.ld_q;
    t.layer = a.layer;
    t.num_layers = a.num_layers;
    t.KH = a.KH;
    t.G = G;
    t.B = a.B;
    t.block_tables = a.block_tables;
    t.bt_stride = a.bt_stride;
    t.context_lens = a.context_lens;
    t.sm_scale = a.sm_scale;
    t.out = p.out;
    t.ld_o = p.ld_o;
    t.ws_o = p.ws_o;
    t.ws_ml = p.ws_ml;
    t.counters = p.counters;
    t.max_chunks = splits;
    t.chunk_pages = std::max(1, (std::max(1, a.max_pages) + splits - 1) / splits);
    t.err = p.err;
    const CUtensorMap map = make_kmajor_map(a.cache, pool_rows, a.D, a.D, kPage);
    const int items = a.B * a.KH * splits;
    const int grid = std::max(1, std::min(items, 2 * device_sm_count()));
    if (a.D == 128) launch_decode_tma<128>(map, t, grid, st);
    else launch_decode_tma<64>(map, t, grid, st);
    VRM_CUDA_CHECK(cudaGetLastError());
    return;
  }
  dim3 grid(a.KH, a.B, splits);
  // 2..8 splits of a caller without its own scratch merge inside a cluster (the caller
  // that brings scratch keeps the counter merge over it)
  const int fmt = cache_format(a.cache_fp8, a.cache_q4);
  auto go = [&](auto d_tag, auto c_tag) {
    constexpr int D = decltype(d_tag)::value;
    constexpr bool C = decltype(c_tag)::value;
    if (fmt == kFmtFp8) launch_decode<D, kFmtFp8, C>(grid, p, st);
    else if (fmt == kFmtQ4) launch_decode<D, kFmtQ4, C>(grid, p, st);
    else launch_decode<D, kFmtBf16, C>(grid, p, st);
  };
  using D128 = std::integral_constant<int, 128>;
  using D64 = std::integral_constant<int, 64>;
  if (cluster) {
    if (a.D == 128) go(D128{}, std::true_type{});
    else go(D64{}, std::true_type{});
  } else {
    if (a.D == 128) go(D128{}, std::false_type{});
    else go(D64{}, std::false_type{});
  }
}

// tcgen05 prefill for bf16 pages: opt-in (VRM_PREFILL_TC=1 or set_prefill_tc(true)).
// Measured on B200 (40 / 8 heads, D = 128): 160-199 TFLOP/s against 206-234 for the
// warp-MMA kernel; its four softmax warps (one per TMEM lane quarter) are the bottleneck.
static int g_prefill_tc = -1;
void set_prefill_tc(bool on) { g_prefill_tc = on ? 1 : 0; }
static bool prefill_tc_enabled() {
  if (g_prefill_tc < 0) {
    const char* e = std::getenv("VRM_PREFILL_TC");
    g_prefill_tc = (e && e[0] == '1') ? 1 : 0;
  }
  return g_prefill_tc == 1;
}

template <int D>
static void launch_prefill_tc(const CUtensorMap& qm, const CUtensorMap& kv, const PrefillTcParams& p, dim3 grid,
                              cudaStream_t st) {
  constexpr int smem = PrefillTcSmem<D>::kAlloc;
  auto kern = paged_prefill_tc_kernel<D>;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev & 63] = true;
  }
  launch_kernel(kern, grid, dim3(320), (size_t)smem, st, qm, kv, p);
}

template <int D, int FMT>
static void launch_prefill(dim3 grid, const PrefillParams& p, cudaStream_t st) {
  constexpr int smem = PrefillSmem<D, FMT>::kTotal;
  auto kern = paged_prefill_kernel<D, FMT>;
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    set[dev & 63] = true;
  }
  launch_kernel(kern, grid, dim3(128), (size_t)smem, st, p);
}

void paged_attention_prefill(const PrefillAttnArgs& a, cudaStream_t st) {
  VRM_REQUIRE(a.D == 64 || a.D == 128, "prefill attention: head_dim must be 64 or 128");
  VRM_REQUIRE(a.KH > 0 && a.Hq % a.KH == 0, "prefill attention: heads");
  VRM_REQUIRE(!a.cache_fp8 || a.kv_scale != nullptr, "prefill attention: fp8 cache needs kv_scale");
  VRM_REQUIRE(!(a.cache_fp8 && a.cache_q4), "prefill attention: one page format");
  VRM_REQUIRE(a.ld_q % 8 == 0, "prefill attention: q row stride must be a multiple of 8");
  if (a.B <= 0 || a.max_q_len <= 0) return;
  PrefillParams p;
  p.q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  p.ld_q = a.ld_q;
  p.cache = reinterpret_cast<const uint8_t*>(a.cache);
  p.layer = a.layer;
  p.num_layers = a.num_layers;
  p.KH = a.KH;
  p.G = a.Hq / a.KH;
  p.block_tables = a.block_tables;
  p.bt_stride = a.bt_stride;
  p.cu_q = a.cu_q;
  p.context_lens = a.context_lens;
  p.kv_scale = a.kv_scale;
  p.sm_scale = a.sm_scale;
  p.out = reinterpret_cast<__nv_bfloat16*>(a.out);
  p.ld_o = a.ld_o;
  p.num_pages = a.cache_pages;
  p.err = error_word();
  const int64_t pool_rows = a.cache_pages * a.num_layers * 2 * a.KH * kPage;
  const int fmt = cache_format(a.cache_fp8, a.cache_q4);
  if (fmt == kFmtBf16 && prefill_tc_enabled() && a.cache_pages > 0 && a.num_tokens > 0 &&
      pool_rows < (int64_t)INT32_MAX && a.num_tokens < (int64_t)INT32_MAX &&
      (reinterpret_cast<uintptr_t>(a.cache) & 15) == 0 && (reinterpret_cast<uintptr_t>(a.q) & 15) == 0) {
    PrefillTcParams t;
    t.block_tables = a.block_tables;
    t.bt_stride = a.bt_stride;
    t.cu_q = a.cu_q;
    t.context_lens = a.context_lens;
    t.layer = a.layer;
    t.num_layers = a.num_layers;
    t.KH = a.KH;
    t.G = a.Hq / a.KH;
    t.Hq = a.Hq;
    t.sm_scale = a.sm_scale;
    t.out = p.out;
    t.ld_o = a.ld_o;
    t.max_tiles = (a.max_q_len + 127) / 128;
    t.num_pages = a.cache_pages;
    t.err = p.err;
    const CUtensorMap kv = make_kmajor_map(a.cache, pool_rows, a.D, a.D, kPage);
    const CUtensorMap qm = make_kmajor_map(a.q, a.num_tokens, (int64_t)a.Hq * a.D, a.ld_q, 128);
    const dim3 grid(t.max_tiles, a.Hq, a.B);
    if (a.D == 128) launch_prefill_tc<128>(qm, kv, t, grid, st);
    else launch_prefill_tc<64>(qm, kv, t, grid, st);
    return;
  }
  dim3 grid((a.max_q_len + 63) / 64, a.Hq, a.B);
  if (a.D == 128) {
    if (fmt == kFmtFp8) launch_prefill<128, kFmtFp8>(grid, p, st);
    else if (fmt == kFmtQ4) launch_prefill<128, kFmtQ4>(grid, p, st);
    else launch_prefill<128, kFmtBf16>(grid, p, st);
  } else {
    if (fmt == kFmtFp8) launch_prefill<64, kFmtFp8>(grid, p, st);
    else if (fmt == kFmtQ4) launch_prefill<64, kFmtQ4>(grid, p, st);
    else launch_prefill<64, kFmtBf16>(grid, p, st);
  }
}

}  // namespace vrm
