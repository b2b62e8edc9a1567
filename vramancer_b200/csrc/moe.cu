// Mixture-of-experts routing on the device: router softmax + top-k, the plan (counts,
// grouped rows, token blocks), gather of the routed activations, and the weighted
// combine back to token order (fused with the residual add and the next RMSNorm).  The
// expert GEMMs in between are the grouped tcgen05 kernel of gemm_tc.cu.  Nothing here
// reads back to the host, so a whole MoE layer can be captured in a CUDA graph.
//
// Grouped row order within an expert follows atomic arrival, which may vary between
// runs; every grouped row is computed independently and the combine sums each token's
// top-k rows in k order, so the layer output does not depend on it.
//
// Ordering under programmatic dependent launch: the plan is consumed up to four
// kernels later (gather, both grouped GEMMs, combine), by grids that the chain of
// early triggers may have launched before the plan kernel finished.  That is safe as
// long as no load of plan data is scheduled above griddepcontrol.wait, which is what
// pdl_wait_for() guarantees for the pointers it is given.
//
// Reference parity: the reference has no MoE kernels (it defers MoE to vLLM /
// llama.cpp); its expert placement hook is core/expert_pinning.py:115-642.
#include <algorithm>

#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxExperts = 2048;
constexpr int kPlanPer = kMaxExperts / kPlanThreads;    // experts per thread in the scans
constexpr int kFuseRouteTokens = 128;                   // route + plan in one CTA up to this many tokens

struct PlanSmem {
  int cnt[kMaxExperts];
  int off[kMaxExperts];
  int warp_a[32], warp_b[32];
  int tot_a, tot_b;
};

// Exclusive prefix sums of a and b over the CTA in thread order; totals in sm.tot_*.
__device__ __forceinline__ void block_scan2(int a, int b, int& pa, int& pb, PlanSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int ia = a, ib = b;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int xa = __shfl_up_sync(0xffffffffu, ia, o), xb = __shfl_up_sync(0xffffffffu, ib, o);
    if (lane >= o) {
      ia += xa;
      ib += xb;
    }
  }
  if (lane == 31) {
    sm.warp_a[warp] = ia;
    sm.warp_b[warp] = ib;
  }
  __syncthreads();
  if (warp == 0) {
    const int wa = lane < nw ? sm.warp_a[lane] : 0, wb = lane < nw ? sm.warp_b[lane] : 0;
    int sa = wa, sb = wb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int xa = __shfl_up_sync(0xffffffffu, sa, o), xb = __shfl_up_sync(0xffffffffu, sb, o);
      if (lane >= o) {
        sa += xa;
        sb += xb;
      }
    }
    if (lane < nw) {
      sm.warp_a[lane] = sa - wa;
      sm.warp_b[lane] = sb - wb;
    }
    if (lane == nw - 1) {
      sm.tot_a = sa;
      sm.tot_b = sb;
    }
  }
  __syncthreads();
  pa = sm.warp_a[warp] + ia - a;
  pb = sm.warp_b[warp] + ib - b;
}

// The plan of P ids, run by one CTA of kPlanThreads threads.
template <typename Id>
__device__ void build_plan(const Id* ids, const MoePlanArgs& a, PlanSmem& sm, uint32_t* err) {
  const int E = a.E;
  for (int e = threadIdx.x; e < E; e += blockDim.x) sm.cnt[e] = 0;
  __syncthreads();
  // rank of each pair within its expert (arrival order), kept in row_of until the end
  for (int p = threadIdx.x; p < a.P; p += blockDim.x) {
    int e = (int)ids[p];
    if (e < 0 || e >= E) {
      report_error(err, kErrBadShape);
      e = 0;
    }
    a.row_of[p] = atomicAdd(&sm.cnt[e], 1);
  }
  __syncthreads();
  // row offsets and block offsets: thread t owns experts [t * kPlanPer, (t + 1) * kPlanPer)
  int c[kPlanPer], nb[kPlanPer], sc = 0, sb = 0;
#pragma unroll
  for (int j = 0; j < kPlanPer; ++j) {
    const int e = threadIdx.x * kPlanPer + j;
    c[j] = e < E ? sm.cnt[e] : 0;
    nb[j] = (c[j] + a.BN - 1) / a.BN;
    sc += c[j];
    sb += nb[j];
  }
  int pc, pb;
  block_scan2(sc, sb, pc, pb, sm);
#pragma unroll
  for (int j = 0; j < kPlanPer; ++j) {
    const int e = threadIdx.x * kPlanPer + j;
    if (e < E) {
      sm.off[e] = pc;
      a.counts[e] = c[j];
      a.offsets[e] = pc;
      for (int r = 0; r < nb[j]; ++r) {
        const int bi = pb + r;
        if (bi < a.max_blocks) a.blocks[bi] = MoeBlock{e, pc + r * a.BN, min(a.BN, c[j] - r * a.BN), 0};
      }
    }
    pc += c[j];
    pb += nb[j];
  }
  if (threadIdx.x == 0) {
    a.offsets[E] = sm.tot_a;
    int total = sm.tot_b;
    if (total > a.max_blocks) {
      report_error(err, kErrBadShape);
      total = a.max_blocks;
    }
    *a.num_blocks = total;
  }
  __syncthreads();
  for (int p = threadIdx.x; p < a.P; p += blockDim.x) {
    int e = (int)ids[p];
    if (e < 0 || e >= E) e = 0;
    const int row = sm.off[e] + a.row_of[p];
    a.row_of[p] = row;
    a.tok_of_row[row] = p / a.topk;
  }
}

template <typename Id>
__global__ void __launch_bounds__(kPlanThreads) moe_plan_kernel(MoePlanArgs a, const Id* ids, uint32_t* err) {
  __shared__ PlanSmem sm;
  pdl_launch();
  pdl_wait_for(ids);
  build_plan(ids, a, sm, err);
}

// Router top-k: a group of LPT lanes per token, VPL logits per lane (expert e sits in
// lane e % LPT, slot e / LPT).  Softmax in fp32, then k rounds of a group argmax (ties
// to the lower expert id), then the optional renormalisation.  Every lane of the warp
// runs this (the shuffles need them all); lanes of an absent token write nothing.
template <int LPT, int VPL>
__device__ __forceinline__ void route_token(const MoeRouteArgs& a, int t, bool valid) {
  const int g = threadIdx.x & (LPT - 1);
  const unsigned mask = 0xffffffffu;
  const int E = a.plan.E, k = a.plan.topk;
  const __nv_bfloat16* row = reinterpret_cast<const __nv_bfloat16*>(a.logits) + (size_t)t * a.ldl;
  float v[VPL];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = g + LPT * i;
    v[i] = !valid ? 0.f : (e < E ? __bfloat162float(row[e]) : -INFINITY);
    m = fmaxf(m, v[i]);
  }
#pragma unroll
  for (int o = LPT / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(mask, m, o, LPT));
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    v[i] = (g + LPT * i < E) ? expf(v[i] - m) : 0.f;
    s += v[i];
  }
#pragma unroll
  for (int o = LPT / 2; o > 0; o >>= 1) s += __shfl_xor_sync(mask, s, o, LPT);
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] = (g + LPT * i < E) ? v[i] / s : -1.f;
  float wsum = 0.f;
  for (int r = 0; r < k; ++r) {
    float bv = -1.f;
    int be = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (v[i] > bv) {
        bv = v[i];
        be = g + LPT * i;
      }
#pragma unroll
    for (int o = LPT / 2; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(mask, bv, o, LPT);
      const int oe = __shfl_xor_sync(mask, be, o, LPT);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (g + LPT * i == be) v[i] = -1.f;
    wsum += bv;
    if (valid && g == (r % LPT)) {
      a.ids32[(size_t)t * k + r] = be;
      if (a.ids64) a.ids64[(size_t)t * k + r] = be;
      a.weights[(size_t)t * k + r] = bv;
    }
  }
  if (valid && a.norm_topk) {
    // round r was written by lane r % LPT: each lane rescales its own rounds
    const float inv = 1.f / wsum;
    for (int r = g; r < k; r += LPT) a.weights[(size_t)t * k + r] *= inv;
  }
}

template <int LPT, int VPL>
__device__ __forceinline__ void route_tokens(const MoeRouteArgs& a, int tok0, int tok_stride) {
  constexpr int kTpw = 32 / LPT;   // tokens per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int base = tok0 + warp * kTpw; base < a.T; base += tok_stride) {   // warp-uniform
    const int t = base + lane / LPT;
    route_token<LPT, VPL>(a, t < a.T ? t : 0, t < a.T);
  }
}

template <int LPT, int VPL>
__global__ void __launch_bounds__(256) moe_topk_kernel(MoeRouteArgs a) {
  pdl_launch();
  pdl_wait_for(a.logits);
  constexpr int kTpw = 32 / LPT;
  const int per_cta = (blockDim.x >> 5) * kTpw;
  route_tokens<LPT, VPL>(a, blockIdx.x * per_cta, gridDim.x * per_cta);
}

template <int LPT, int VPL>
__global__ void __launch_bounds__(kPlanThreads) moe_route_plan_kernel(MoeRouteArgs a, uint32_t* err) {
  __shared__ PlanSmem sm;
  pdl_launch();
  pdl_wait_for(a.logits);
  constexpr int kTpw = 32 / LPT;
  route_tokens<LPT, VPL>(a, 0, (blockDim.x >> 5) * kTpw);
  __syncthreads();                  // every token's ids written (global memory, this CTA)
  build_plan(static_cast<const int*>(a.ids32), a.plan, sm, err);
}

// one CTA per grouped row, 16-byte copies
__global__ void moe_gather_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const int* __restrict__ tok,
                                  int K, __nv_bfloat16* __restrict__ xp, int64_t ldp) {
  pdl_launch();
  pdl_wait_for(x, tok);
  const int r = blockIdx.x;
  const uint4* src = reinterpret_cast<const uint4*>(x + (size_t)tok[r] * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (size_t)r * ldp);
  for (int v = threadIdx.x; v < K / 8; v += blockDim.x) dst[v] = src[v];
}

constexpr int kCombThreads = 256;
constexpr int kCombMaxV = 4;         // vectors of 8 per thread: H <= 8192

__device__ __forceinline__ float comb_block_sum(float v, float* red) {
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

__device__ __forceinline__ void add8(float (&acc)[8], uint4 u, float s) {
  const uint32_t* pu = reinterpret_cast<const uint32_t*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    acc[2 * j] += s * bf16_lo(pu[j]);
    acc[2 * j + 1] += s * bf16_hi(pu[j]);
  }
}

// one CTA per token: fp32 sum of its top-k expert rows in k order (+ add), then either
// the plain output or residual += sum with the optional RMSNorm of the new residual
__global__ void __launch_bounds__(kCombThreads) moe_combine_kernel(MoeCombineArgs a, uint32_t* err) {
  pdl_launch();
  const __nv_bfloat16* yp = reinterpret_cast<const __nv_bfloat16*>(a.y_perm);
  const __nv_bfloat16* add = reinterpret_cast<const __nv_bfloat16*>(a.add);
  const __nv_bfloat16* nw = reinterpret_cast<const __nv_bfloat16*>(a.norm_w);
  __nv_bfloat16* res = reinterpret_cast<__nv_bfloat16*>(a.residual);
  const int* row_of = a.row_of;
  const float* w = a.weights;
  pdl_wait_for(yp, add, nw, res, row_of, w);
  __shared__ float red[33];
  const int t = blockIdx.x;
  if (a.wait_flags) {
    // expert parallelism: every owner's rows for this rank have landed in the epoch's half
    const uint32_t ep = *reinterpret_cast<const volatile uint32_t*>(a.epoch);
    if (threadIdx.x == 0) {
      for (int r = 0; r < a.wait_world; ++r) {
        const unsigned long long t0 = clock64();
        while ((int)(ld_acquire_sys(a.wait_flags + r) - ep) < 0) {
          if ((unsigned long long)(clock64() - t0) > VRM_SPIN_LIMIT_CYCLES) {
            report_error(err, kErrFlagTimeout);
            break;
          }
        }
      }
    }
    __syncthreads();
    yp += (size_t)(ep & 1u) * a.half_rows * a.ld_perm;
  }
  const int nvec = a.H / 8;
  float acc[kCombMaxV][8];
#pragma unroll
  for (int i = 0; i < kCombMaxV; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;
  for (int k = 0; k < a.topk; ++k) {
    const float wk = w[t * a.topk + k];
    const int row = row_of ? row_of[t * a.topk + k] : t * a.topk + k;
    const uint4* src = reinterpret_cast<const uint4*>(yp + (size_t)row * a.ld_perm);
#pragma unroll
    for (int i = 0; i < kCombMaxV; ++i) {
      const int v = threadIdx.x + i * kCombThreads;
      // rows stored by peer GPUs are read from L2, past any line this SM may hold
      if (v < nvec) add8(acc[i], a.wait_flags ? __ldcg(src + v) : src[v], wk);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kCombMaxV; ++i) {
    const int v = threadIdx.x + i * kCombThreads;
    if (v >= nvec) continue;
    if (add) add8(acc[i], *reinterpret_cast<const uint4*>(add + (size_t)t * a.H + v * 8), 1.f);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
    if (res) {
      __nv_bfloat16* rp = res + (size_t)t * a.H + v * 8;
      add8(acc[i], *reinterpret_cast<const uint4*>(rp), 1.f);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        po[j] = pack_bf16x2(acc[i][2 * j], acc[i][2 * j + 1]);
        // the residual stream is bf16: the norm sees the rounded values
        acc[i][2 * j] = bf16_lo(po[j]);
        acc[i][2 * j + 1] = bf16_hi(po[j]);
        ss += acc[i][2 * j] * acc[i][2 * j] + acc[i][2 * j + 1] * acc[i][2 * j + 1];
      }
      *reinterpret_cast<uint4*>(rp) = o;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) po[j] = pack_bf16x2(acc[i][2 * j], acc[i][2 * j + 1]);
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.ldo + v * 8) = o;
    }
  }
  if (!res || !nw) return;   // uniform over the CTA
  const float inv = rsqrtf(comb_block_sum(ss, red) / (float)a.H + a.eps);
  __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * a.ldo;
#pragma unroll
  for (int i = 0; i < kCombMaxV; ++i) {
    const int v = threadIdx.x + i * kCombThreads;
    if (v >= nvec) continue;
    const uint4 g = *reinterpret_cast<const uint4*>(nw + v * 8);
    const uint32_t* pg = reinterpret_cast<const uint32_t*>(&g);
    uint4 o;
    uint32_t* po = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      po[j] = pack_bf16x2(acc[i][2 * j] * inv * bf16_lo(pg[j]), acc[i][2 * j + 1] * inv * bf16_hi(pg[j]));
    *reinterpret_cast<uint4*>(orow + v * 8) = o;
  }
}

template <int LPT, int VPL>
void launch_route(const MoeRouteArgs& a, cudaStream_t st) {
  if (a.T <= kFuseRouteTokens) {
    launch_kernel(moe_route_plan_kernel<LPT, VPL>, dim3(1), dim3(kPlanThreads), 0, st, a, error_word());
    return;
  }
  constexpr int kPerCta = (256 / 32) * (32 / LPT);
  const int grid = (a.T + kPerCta - 1) / kPerCta;
  launch_kernel(moe_topk_kernel<LPT, VPL>, dim3(grid), dim3(256), 0, st, a);
  launch_kernel(moe_plan_kernel<int>, dim3(1), dim3(kPlanThreads), 0, st, a.plan,
                static_cast<const int*>(a.ids32), error_word());
}

}  // namespace

void moe_plan(const MoePlanArgs& a, cudaStream_t st) {
  VRM_REQUIRE(a.E > 0 && a.E <= kMaxExperts && a.P >= 0 && a.topk > 0 && a.BN > 0, "moe_plan: bad sizes");
  VRM_REQUIRE((a.ids64 != nullptr) != (a.ids32 != nullptr), "moe_plan: give ids64 or ids32");
  if (a.P == 0) return;
  if (a.ids64)
    launch_kernel(moe_plan_kernel<int64_t>, dim3(1), dim3(kPlanThreads), 0, st, a, a.ids64, error_word());
  else
    launch_kernel(moe_plan_kernel<int>, dim3(1), dim3(kPlanThreads), 0, st, a, a.ids32, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_route(const MoeRouteArgs& a, cudaStream_t st) {
  const int E = a.plan.E, k = a.plan.topk;
  VRM_REQUIRE(E > 0 && E <= 1024 && k > 0 && k <= E && a.ldl >= E, "moe_route: E must be in [1, 1024], k <= E");
  VRM_REQUIRE(a.ids32 && a.weights && a.plan.ids32 == a.ids32 && !a.plan.ids64, "moe_route: output buffers");
  VRM_REQUIRE(a.plan.P == a.T * k && a.plan.BN > 0, "moe_route: plan.P must be T * topk");
  if (a.T == 0) return;
  if (E <= 32) launch_route<2, 16>(a, st);
  else if (E <= 64) launch_route<4, 16>(a, st);
  else if (E <= 128) launch_route<8, 16>(a, st);
  else if (E <= 256) launch_route<16, 16>(a, st);
  else if (E <= 512) launch_route<32, 16>(a, st);
  else launch_route<32, 32>(a, st);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_gather(const void* x, int64_t ldx, const int* tok_of_row, int P, int K, void* x_perm, int64_t ld_perm,
                cudaStream_t st) {
  VRM_REQUIRE(K % 8 == 0 && ldx % 8 == 0 && ld_perm % 8 == 0, "moe_gather: rows must be 16-byte multiples");
  if (P <= 0) return;
  launch_kernel(moe_gather_kernel, dim3(P), dim3(std::min(256, std::max(32, K / 8))), 0, st,
                reinterpret_cast<const __nv_bfloat16*>(x), ldx, tok_of_row, K,
                reinterpret_cast<__nv_bfloat16*>(x_perm), ld_perm);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_combine(const MoeCombineArgs& a, cudaStream_t st) {
  if (a.T <= 0) return;
  VRM_REQUIRE(a.H % 8 == 0 && a.H <= 8 * kCombThreads * kCombMaxV && a.ld_perm % 8 == 0 && a.ldo % 8 == 0,
              "moe_combine: H must be a multiple of 8 and <= 8192");
  VRM_REQUIRE(a.out || (a.residual && !a.norm_w), "moe_combine: output missing");
  VRM_REQUIRE(!a.norm_w || a.residual, "moe_combine: the fused norm needs the residual");
  if (a.T <= 0) return;
  launch_kernel(moe_combine_kernel, dim3(a.T), dim3(kCombThreads), 0, st, a, error_word());
  VRM_CUDA_CHECK(cudaGetLastError());
}

void moe_ep_combine(const MoeEpBuffers& b, const MoeCombineArgs& c, cudaStream_t st) {
  MoeCombineArgs a = c;
  a.y_perm = b.yback_local;
  a.ld_perm = b.H;
  a.row_of = nullptr;
  a.wait_flags = b.flags_local + 2 * b.world;
  a.wait_world = b.world;
  a.epoch = b.epoch;
  a.half_rows = b.p_cap;
  moe_combine(a, st);
}

}  // namespace vrm
