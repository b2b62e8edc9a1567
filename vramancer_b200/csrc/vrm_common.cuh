// Shared device helpers for the sm_100a kernels of vramancer_b200.
//
// Everything here is thin inline PTX around Blackwell primitives:
//   * mbarrier (init / arrive / expect_tx / bounded try_wait)
//   * TMA tiled loads (cp.async.bulk.tensor), each CTA loading its own tiles (no cluster
//     multicast of loads anywhere in this code)
//   * tcgen05 (TMEM alloc/dealloc, UMMA issue, commit, TMEM->register loads)
//   * warp-level mma.sync / ldmatrix / cp.async for the small-M kernels
// plus a device-wide error word that every bounded wait reports into.
//
// Bounded waits: every spin on an mbarrier or a flag gives up after
// VRM_SPIN_LIMIT_CYCLES (about one second at boost clock), records a code in the
// error word and lets the caller unwind (free TMEM, return).  No wait in this code
// base can hang a GPU forever.
#pragma once

#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#ifndef VRM_SPIN_LIMIT_CYCLES
#define VRM_SPIN_LIMIT_CYCLES (2000000000ull)
#endif

namespace vrm {

// Error codes written into the per-device error word (host reads it back).
enum ErrCode : uint32_t {
  kErrNone = 0,
  kErrMbarTimeout = 1,     // an mbarrier wait ran out of its budget
  kErrFlagTimeout = 2,     // a cross-CTA / cross-GPU flag wait ran out
  kErrBadShape = 4,        // launch-time shape check failed on device
  kErrBounds = 8,          // bounds-check build: a page / slot index outside its pool
};

__device__ __forceinline__ void report_error(uint32_t* err, uint32_t code) {
  if (err) atomicOr(err, code);
}

// Bounds-check builds (VRM_BOUNDS_CHECK=1 python setup.py build_ext --inplace): page
// and slot indices read from block tables / slot maps / page lists are checked against
// the pool they index (n > 0); an index out of range sets kErrBounds in the error word
// and the caller skips or redirects the access instead of touching memory outside the
// pool.  Default builds compile the check away.
#if defined(VRM_BOUNDS_CHECK) && VRM_BOUNDS_CHECK
__device__ __forceinline__ bool in_bounds(long long i, long long n, uint32_t* err) {
  if (n <= 0 || (i >= 0 && i < n)) return true;
  report_error(err, kErrBounds);
  return false;
}
#else
__device__ __forceinline__ bool in_bounds(long long, long long, uint32_t*) { return true; }
#endif

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false (and
// records kErrMbarTimeout) when the budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((unsigned long long)(clock64() - t0) > VRM_SPIN_LIMIT_CYCLES) {
      report_error(err, kErrMbarTimeout);
      return false;
    }
  }
}

// ---------------------------------------------------------------- TMA
// 2D tiled load global->shared, completion signalled on an mbarrier (tx bytes).
// Coordinates: c0 = innermost (element index, c0*elemsize % 16 == 0), c1 = row.
// No multicast: the source is always this GPU's own memory.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(cache_hint)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// L2 eviction policies for TMA cache hints (createpolicy is documented PTX).
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one full warp; writes the base address to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t desc_a, uint64_t desc_b, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(desc_a), "l"(desc_b), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA with
// 128-byte swizzle: rows of 128 B (64 bf16 of K), 8-row groups 1024 B apart.
//   bits [0,14)  start address >> 4
//   bits [16,30) leading byte offset >> 4   (unused for swizzled K-major; 1)
//   bits [32,46) stride byte offset >> 4    (1024 B between 8-row groups)
//   bits [46,48) descriptor version (1 on sm_100)
//   bits [61,64) layout type (2 = 128B swizzle)
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor, kind::f16 with bf16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_bf16(int M, int N) {
  return (1u << 4)                       // D format f32
         | (1u << 7)                     // A format bf16
         | (1u << 10)                    // B format bf16
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// Instruction descriptor, kind::f8f6f4 with e4m3 A/B (format 0), fp32 D, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_e4m3(int M, int N) {
  return (1u << 4)                       // D format f32
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// ---------------------------------------------------------------- warp-level MMA path
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int sz = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------- programmatic dependent launch
// pdl_wait: block until the preceding kernel in the stream has completed and its
// writes are visible (no-op when the kernel was not launched with the programmatic
// serialization attribute).  Every global read of a predecessor's output and every
// global write must come after it.  pdl_launch: allow the next kernel's CTAs to be
// scheduled now (they still pdl_wait before touching our outputs).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// A load through a `const T* __restrict__` kernel parameter may be compiled as an
// invariant, non-coherent load, and the compiler may then schedule it above
// griddepcontrol.wait, i.e. before the kernel that writes the data has finished (on
// B200 this showed up as a MoE work list read three kernels after it was written).
// pdl_wait_for(p...) waits and then passes each pointer through an opaque asm that is
// ordered after the wait, so every load through them is an ordinary load below it.
// Use it for every pointer to data that an earlier kernel writes.
template <typename P>
__device__ __forceinline__ void opaque_after_wait(P& p) {
  unsigned long long v = reinterpret_cast<unsigned long long>(p);
  asm volatile("" : "+l"(v)::"memory");
  p = reinterpret_cast<P>(v);
}
template <typename... P>
__device__ __forceinline__ void pdl_wait_for(P&... p) {
  pdl_wait();
  (opaque_after_wait(p), ...);
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- misc
// Rotate-half RoPE of one (x1, x2) pair: (x1 c - x2 s, x2 c + x1 s), with the products
// and sums rounded separately (no FMA contraction), so every kernel that rotates q or k
// (the standalone RoPE + KV write and the fused decode attention) gives the same bits.
__device__ __forceinline__ void rope_rotate(float x1, float x2, float c, float s, float& o1, float& o2) {
  o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  o2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
}

__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 t = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&t);
}

// ---- page formats: 0 bf16, 1 fp8 e4m3 (per-head scale), 2 four-bit (kFmtQ4).  A stored
// 4-bit row of D values is D/2 code bytes (element 2i in the low nibble of byte i), then
// D/32 groups of {scale, min} fp16: value = code * scale + min.
constexpr int kFmtBf16 = 0, kFmtFp8 = 1, kFmtQ4 = 2;
template <int D, int FMT>
struct PageRow {
  static constexpr int kBytes = FMT == kFmtBf16 ? 2 * D : FMT == kFmtFp8 ? D : D / 2 + D / 8;
};

// One warp quantises one row of D values (lane l holds dims D/32 * l ..): per 32-dim
// group scale = (max - min) / 15 and min, both rounded to fp16 first so that the codes
// are computed against what readers will use; codes = round((x - min) / scale) in 0..15.
template <int D>
__device__ __forceinline__ void q4_store_row(uint8_t* dst, const float (&x)[D / 32], int lane) {
  constexpr int kV = D / 32;
  constexpr int kLpg = 32 / kV;            // lanes of a 32-dim group
  float mn = x[0], mx = x[0];
#pragma unroll
  for (int j = 1; j < kV; ++j) {
    mn = fminf(mn, x[j]);
    mx = fmaxf(mx, x[j]);
  }
#pragma unroll
  for (int o = 1; o < kLpg; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  __half hs = __float2half_rn((mx - mn) / 15.f);
  if (!(__half2float(hs) > 0.f)) hs = __float2half_rn(6.103515625e-05f);   // constant group
  const __half hm = __float2half_rn(mn);
  const float s = __half2float(hs), m = __half2float(hm);
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < kV; ++j) {
    const float cf = fminf(fmaxf(rintf((x[j] - m) / s), 0.f), 15.f);
    packed |= (uint32_t)cf << (4 * j);
  }
  if (kV == 4) *reinterpret_cast<uint16_t*>(dst + lane * 2) = (uint16_t)packed;
  else dst[lane] = (uint8_t)packed;
  if (lane % kLpg == 0) *reinterpret_cast<__half2*>(dst + D / 2 + (lane / kLpg) * 4) = __halves2half2(hs, hm);
}


__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Acquire/release accesses used by cross-CTA and cross-GPU flag protocols.
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Data-polled ("empty pattern") exchange of bf16 values between GPUs: a free receive
// slot holds 0x8000 (bf16 -0.0) in every element; a producer stores finished values
// with -0.0 turned into +0.0 (numerically the same), so a reader knows an element has
// arrived as soon as it differs from 0x8000, without a flag or a fence.
constexpr uint32_t kBf16Empty = 0x8000u;
constexpr uint32_t kBf16EmptyX2 = 0x80008000u;
__device__ __forceinline__ uint16_t bf16_bits_nonempty(float v) {
  const uint16_t b = __bfloat16_as_ushort(__float2bfloat16(v));
  return b == (uint16_t)kBf16Empty ? (uint16_t)0 : b;
}
__device__ __forceinline__ void st_relaxed_sys_u16(void* p, uint16_t v) {
  asm volatile("st.relaxed.sys.global.b16 [%0], %1;" ::"l"(p), "h"(v) : "memory");
}
__device__ __forceinline__ uint4 ld_relaxed_sys_v4(const void* p) {
  uint4 v;
  asm volatile("ld.relaxed.sys.global.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ uint2 ld_relaxed_sys_v2(const void* p) {
  uint2 v;
  asm volatile("ld.relaxed.sys.global.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool bf16x4_has_empty(uint2 x) {
  auto e = [](uint32_t w) { return (w & 0xffffu) == kBf16Empty || (w >> 16) == kBf16Empty; };
  return e(x.x) || e(x.y);
}
// true when any of the 8 bf16 lanes of x still holds the empty pattern
__device__ __forceinline__ bool bf16x8_has_empty(uint4 x) {
  auto e = [](uint32_t w) { return (w & 0xffffu) == kBf16Empty || (w >> 16) == kBf16Empty; };
  return e(x.x) || e(x.y) || e(x.z) || e(x.w);
}

}  // namespace vrm
