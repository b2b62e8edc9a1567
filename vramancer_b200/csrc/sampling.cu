// Token selection over bf16 logits [B, V], one CTA (1024 threads) per row.
//
//   greedy:   argmax (lowest index on ties)
//   sampling: temperature, top-k and top-p (nucleus) with exact thresholds found by
//             two-digit radix select over the 16-bit order keys of the bf16 logits
//             (count histograms for top-k, probability-mass histograms for top-p),
//             then an exact draw from the renormalised kept set with the Gumbel-max
//             trick: argmax_i (z_i + G_i), G_i = -log(-log(U_i)), U_i from a
//             counter-based hash of (seed, row, step, i).  No sort, no host sync,
//             fixed launch shape: replayable inside a captured decode graph.
//
// Reference parity: core/triton_sampling.py:55-206 (Triton softmax + torch.topk +
// torch.multinomial), core/turbo_engine.py:605-638 (argmax fused into the graph).
#include "vrm_common.cuh"
#include "vrm_host.h"
#include "vrm_kernels.h"

namespace vrm {

constexpr int kSampThreads = 1024;

// Monotone 16-bit key of a bf16 value: larger value -> larger key.
__device__ __forceinline__ uint32_t bf16_key(uint16_t bits) {
  return (bits & 0x8000u) ? (uint32_t)(~bits & 0xFFFFu) : (uint32_t)(bits | 0x8000u);
}

// splitmix64 finaliser (Steele, Lea, Flood 2014) -> uniform in (0, 1)
__device__ __forceinline__ float hash_uniform(uint64_t seed, uint64_t row, uint64_t step, uint64_t i) {
  uint64_t z = seed ^ (row * 0x9E3779B97F4A7C15ull) ^ (step * 0xD1B54A32D192ED03ull) ^ (i * 0xBF58476D1CE4E5B9ull);
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= (z >> 31);
  return ((float)(z >> 40) + 0.5f) * (1.0f / 16777216.0f);
}

struct ArgBest {
  float v;
  int i;
};
__device__ __forceinline__ ArgBest better(ArgBest a, ArgBest b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}

__device__ ArgBest block_argmax(ArgBest a, ArgBest* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgBest b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = a;
  __syncthreads();
  if (w == 0) {
    a = (l < (int)(blockDim.x >> 5)) ? sh[l] : ArgBest{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgBest b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
      a = better(a, b);
    }
    if (l == 0) sh[0] = a;
  }
  __syncthreads();
  return sh[0];
}

__device__ float block_sum(float v, float* sh) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) sh[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? sh[l] : 0.f;
    v = warp_sum(v);
    if (l == 0) sh[0] = v;
  }
  __syncthreads();
  return sh[0];
}


// Row argmax with 16-byte loads, four in flight per thread (the scan is latency-bound
// when one CTA reads a whole 150k-entry row).
__device__ __forceinline__ void upd8(ArgBest& b, uint4 v, int base) {
  const uint32_t* p = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    b = better(b, ArgBest{bf16_lo(p[j]), base + 2 * j});
    b = better(b, ArgBest{bf16_hi(p[j]), base + 2 * j + 1});
  }
}

__device__ ArgBest row_argmax(const __nv_bfloat16* __restrict__ x, int V, ArgBest* sh) {
  ArgBest best{-INFINITY, 0x7fffffff};
  const int bd = blockDim.x;
  if ((V & 7) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int nv = V >> 3;
    int i = threadIdx.x;
    for (; i + 3 * bd < nv; i += 4 * bd) {
      const uint4 a0 = __ldg(xv + i), a1 = __ldg(xv + i + bd), a2 = __ldg(xv + i + 2 * bd), a3 = __ldg(xv + i + 3 * bd);
      upd8(best, a0, i * 8);
      upd8(best, a1, (i + bd) * 8);
      upd8(best, a2, (i + 2 * bd) * 8);
      upd8(best, a3, (i + 3 * bd) * 8);
    }
    for (; i < nv; i += bd) upd8(best, __ldg(xv + i), i * 8);
  } else {
    for (int i = threadIdx.x; i < V; i += bd) best = better(best, ArgBest{__bfloat162float(x[i]), i});
  }
  return block_argmax(best, sh);
}

__global__ void __launch_bounds__(kSampThreads)
    argmax_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V, int* __restrict__ out) {
  pdl_launch();
  pdl_wait_for(logits);
  __shared__ ArgBest sh[32];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const ArgBest best = row_argmax(x, V, sh);
  if (threadIdx.x == 0) out[row] = best.i;
}

// Calls f(i, bits, valid) for every element of a row with 16-byte loads, four in flight
// per thread: one CTA scans a whole ~150k-entry row several times, and with one 2-byte
// load outstanding per thread each pass is bound by L2 latency (about 50 us per pass
// was measured on B200 that way).  Trip counts are warp-uniform, so f may use
// warp-synchronous intrinsics; calls past the end have valid == false.
template <typename F>
__device__ __forceinline__ void scan_row(const __nv_bfloat16* __restrict__ x, int V, F&& f) {
  const int bd = blockDim.x, tid = threadIdx.x;
  int done = 0;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const uint4* xv = reinterpret_cast<const uint4*>(x);
    const int nv = V >> 3;
    for (int base = 0; base < nv; base += 4 * bd) {
      uint4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * bd + tid;
        a[u] = idx < nv ? __ldg(xv + idx) : make_uint4(0u, 0u, 0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int idx = base + u * bd + tid;
        const uint32_t* p = reinterpret_cast<const uint32_t*>(&a[u]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const uint16_t bits = (uint16_t)((j & 1) ? (p[j >> 1] >> 16) : (p[j >> 1] & 0xFFFFu));
          f(idx * 8 + j, bits, idx < nv);
        }
      }
    }
    done = nv << 3;
  }
  for (int b0 = done; b0 < V; b0 += bd) {
    const int i = b0 + tid;
    const bool ok = i < V;
    f(i, ok ? __bfloat16_as_ushort(x[i]) : (uint16_t)0u, ok);
  }
}

__device__ __forceinline__ float bf16_bits_to_float(uint16_t bits) { return __uint_as_float((uint32_t)bits << 16); }

// Among elements with key >= floor_key whose high digit matches `pref`, finds the
// 8-bit digit at `shift` where the weight accumulated from the top reaches `target`.
// Weights are counts (mass = false) or exp((x - M) / T) (mass = true).
//
// Logits crowd into a handful of high-digit bins (sign and exponent), so one shared
// histogram updated by every thread serialises on a few addresses (1.2 ms per row was
// measured on B200 with that layout).  Each warp owns a private histogram instead;
// in count mode the lanes of a warp that hit the same bin are merged with
// match.any and only their leader updates it (no atomics: one writer per bin per
// warp instruction), in mass mode the lanes add with shared atomics into their own
// warp's bins.  The 32 warp histograms are summed before the scan.
//
// `scan(f)` calls f(i, bits, valid) for every element (GlobalRow, CandRow).
template <class Scan>
__device__ void radix_digit(const Scan& scan, int shift, uint32_t pref_mask, uint32_t pref,
                            uint32_t floor_key, bool mass, float M, float invT, float target,
                            float (*whist)[256], float* hist, uint32_t* out_digit, float* out_above) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < nw * 256; i += blockDim.x) whist[i >> 8][i & 255] = 0.f;
  __syncthreads();
  float* my = whist[w];
  scan([&](int, uint16_t bits, bool ok) {
    uint32_t bin = 256u;                                // 256 = not counted
    float wt = 0.f;
    if (ok) {
      const uint32_t k = bf16_key(bits);
      if (k >= floor_key && (k & pref_mask) == pref) {
        bin = (k >> shift) & 0xFFu;
        if (mass) wt = __expf((bf16_bits_to_float(bits) - M) * invT);
      }
    }
    if (mass) {
      if (bin < 256u) atomicAdd(&my[bin], wt);
    } else {
      const unsigned peers = __match_any_sync(0xffffffffu, bin);
      if (bin < 256u && l == __ffs(peers) - 1) my[bin] += (float)__popc(peers);
    }
  });
  __syncthreads();
  for (int b = threadIdx.x; b < 256; b += blockDim.x) {
    float t = 0.f;
    for (int j = 0; j < nw; ++j) t += whist[j][b];
    hist[b] = t;
  }
  __syncthreads();
  if (threadIdx.x < 32) {
    // scan the 256 bins from the top: lane l owns bins 255-8l .. 255-8l-7
    float loc[8];
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      loc[j] = hist[255 - 8 * l - j];
      s += loc[j];
    }
    float incl = s;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float t = __shfl_up_sync(0xffffffffu, incl, o);
      if (l >= o) incl += t;
    }
    float run = incl - s;   // weight strictly above this lane's bins
    int found = -1;
    float above = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (found < 0 && run + loc[j] >= target) {
        found = 255 - 8 * l - j;
        above = run;
      }
      run += loc[j];
    }
    const unsigned m = __ballot_sync(0xffffffffu, found >= 0);
    if (m == 0u) {
      if (l == 0) {
        *out_digit = 0u;   // target not reached: keep everything in this prefix
        *out_above = 0.f;
      }
    } else {
      const int first = __ffs(m) - 1;
      const int d = __shfl_sync(0xffffffffu, found, first);
      const float ab = __shfl_sync(0xffffffffu, above, first);
      if (l == 0) {
        *out_digit = (uint32_t)d;
        *out_above = ab;
      }
    }
  }
  __syncthreads();
}

// A bf16 logits row in global memory.
struct GlobalRow {
  const __nv_bfloat16* x;
  int V;
  template <class F>
  __device__ __forceinline__ void operator()(F&& f) const { scan_row(x, V, f); }
};

// n candidate logits held in shared memory as bf16 bit patterns; kCandEmpty marks an
// unused slot.  Trip counts are warp-uniform (blockDim is a multiple of 32).
constexpr uint16_t kCandEmpty = 0xFFFFu;   // a NaN pattern no candidate carries
struct CandRow {
  const uint16_t* bits;
  int n;
  template <class F>
  __device__ __forceinline__ void operator()(F&& f) const {
    for (int b0 = 0; b0 < n; b0 += blockDim.x) {
      const int i = b0 + threadIdx.x;
      const uint16_t v = i < n ? bits[i] : kCandEmpty;
      f(i, v, v != kCandEmpty);
    }
  }
};

struct SampleSmem {
  ArgBest sh[32];
  float shf[32];
  float hist[256];
  uint32_t digit;
  float above;
};

// x / T + G(u), G = -log(-log u): no contraction, so every kernel that scores an
// element gets the same bits
__device__ __forceinline__ float gumbel_score(float x, float invT, float u) {
  return __fadd_rn(__fmul_rn(x, invT), -logf(-logf(u)));
}

// Temperature / top-k / top-p selection over the elements `scan` visits (V of them
// valid, maximum M), Gumbel-max draw keyed by gidx(i) (the element's vocabulary index).
// Every thread of the block must call it; returns the chosen element's position i.
template <class Scan, class GIdx>
__device__ int sample_select(const Scan& scan, int V, float M, float T, int k, float p, uint64_t seed, int row,
                             uint64_t step, const GIdx& gidx, SampleSmem& S, float (*whist)[256]) {
  const float invT = 1.f / T;
  // ---- top-k threshold: count radix select over the two bytes of the 16-bit key
  uint32_t floor_key = 0u;
  if (k > 0 && k < V) {
    radix_digit(scan, 8, 0u, 0u, 0u, false, M, invT, (float)k, whist, S.hist, &S.digit, &S.above);
    const uint32_t hi = S.digit;
    const float need = (float)k - S.above;
    radix_digit(scan, 0, 0xFF00u, hi << 8, 0u, false, M, invT, need, whist, S.hist, &S.digit, &S.above);
    floor_key = (hi << 8) | S.digit;
  }
  // ---- top-p threshold: mass radix select inside the top-k set
  if (p < 1.f) {
    float z = 0.f;
    scan([&](int, uint16_t bits, bool ok) {
      if (ok && bf16_key(bits) >= floor_key) z += __expf((bf16_bits_to_float(bits) - M) * invT);
    });
    z = block_sum(z, S.shf);
    const float target = fmaxf(p, 0.f) * z;
    radix_digit(scan, 8, 0u, 0u, floor_key, true, M, invT, target, whist, S.hist, &S.digit, &S.above);
    const uint32_t hi = S.digit;
    const float need = target - S.above;
    radix_digit(scan, 0, 0xFF00u, hi << 8, floor_key, true, M, invT, need, whist, S.hist, &S.digit, &S.above);
    const uint32_t pk = (hi << 8) | S.digit;
    floor_key = floor_key > pk ? floor_key : pk;
  }
  // ---- Gumbel-max draw over the kept set.  The score x / T + G does not subtract the
  // row maximum, so a rank that holds part of the vocabulary scores its elements
  // exactly as a rank holding all of it.
  ArgBest gb{-INFINITY, 0x7fffffff};
  scan([&](int i, uint16_t bits, bool ok) {
    if (!ok || bf16_key(bits) < floor_key) return;
    const float u = hash_uniform(seed, (uint64_t)row, step, (uint64_t)gidx(i));
    gb = better(gb, ArgBest{gumbel_score(bf16_bits_to_float(bits), invT, u), i});
  });
  gb = block_argmax(gb, S.sh);
  return gb.i;
}

struct IdentityIdx {
  __device__ __forceinline__ int operator()(int i) const { return i; }
};

__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temperature,
                  const int* __restrict__ top_k, const float* __restrict__ top_p, uint64_t seed,
                  const int* __restrict__ steps, int* __restrict__ out) {
  pdl_launch();
  pdl_wait_for(logits, temperature, top_k, top_p, steps);
  __shared__ SampleSmem S;
  __shared__ float whist[kSampThreads / 32][256];
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const float T = temperature ? temperature[row] : 0.f;

  const ArgBest best = row_argmax(x, V, S.sh);
  if (!(T > 0.f)) {
    if (threadIdx.x == 0) out[row] = best.i;
    return;
  }
  const int k = top_k ? top_k[row] : 0;
  const float p = top_p ? top_p[row] : 1.f;
  const uint64_t step = steps ? (uint64_t)steps[row] : 0ull;
  const int i = sample_select(GlobalRow{x, V}, V, best.v, T, k, p, seed, row, step, IdentityIdx{}, S, whist);
  if (threadIdx.x == 0) out[row] = i < V ? i : best.i;
}

// ---------------------------------------------------------------- vocabulary-parallel
// Under tensor parallelism each rank holds logits of vocabulary columns
// [v_off, v_off + Vs).  Instead of gathering every rank's logits, each rank reduces its
// shard to at most KC candidates per row (vp_local_kernel), the ranks all-gather the
// candidates (KC x 8 bytes per row and rank), and every rank picks the same token from
// the gathered candidates (vp_combine_kernel):
//   T <= 0            : the shard's argmax (value, index); the pick is the largest value,
//                       lowest index on ties -- the full-row argmax.
//   T > 0, no top-k,  : the shard's Gumbel-max winner x / T + G(seed, row, step, index);
//   top-p >= 1          the pick is the largest score -- the full-row draw.
//   T > 0, top-k <= KMAX: every element of the shard whose key is >= the shard's k-th
//                       largest key (the global k-th largest can only be larger, so
//                       every element of the global top-k set is a candidate); the
//                       combine runs top-k, top-p and the Gumbel draw over the
//                       candidates, keyed by vocabulary index.  Exact unless more than
//                       KC - k elements of one shard tie at its k-th value (the extra
//                       ties are dropped).
// Rows with top-p < 1 and no top-k (or top-k > KMAX) need the whole distribution; the
// caller gathers full logits for those steps.  Candidates: value (fp32: a bf16 logit,
// or the Gumbel score) and vocabulary index; empty slots carry index -1.
constexpr int kVpThreads = 256;

__device__ __forceinline__ int vp_mode(float T, int k, float p, int V_total, int kmax) {
  if (!(T > 0.f)) return 0;                       // greedy
  if ((k <= 0 || k >= V_total) && p >= 1.f) return 1;   // plain temperature: Gumbel-max
  if (k > 0 && k <= kmax) return 2;               // top-k (+ top-p): candidates
  return 3;                                       // needs the full distribution
}

__global__ void __launch_bounds__(kSampThreads)
    vp_local_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int Vs, int v_off, int V_total,
                    const float* __restrict__ temperature, const int* __restrict__ top_k,
                    const float* __restrict__ top_p, uint64_t seed, const int* __restrict__ steps, int KC, int kmax,
                    float* __restrict__ cand_val, int* __restrict__ cand_idx) {
  pdl_launch();
  pdl_wait_for(logits, temperature, top_k, top_p, steps);
  __shared__ SampleSmem S;
  __shared__ float whist[kSampThreads / 32][256];
  __shared__ int s_n;
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const int V = max(0, min(Vs, V_total - v_off));   // the last shard may hold padding columns
  float* cv = cand_val + (size_t)row * KC;
  int* ci = cand_idx + (size_t)row * KC;
  for (int j = threadIdx.x; j < KC; j += blockDim.x) {
    cv[j] = -INFINITY;
    ci[j] = -1;
  }
  const float T = temperature[row];
  const int k = top_k[row];
  const float p = top_p[row];
  const int mode = vp_mode(T, k, p, V_total, kmax);
  const ArgBest best = mode != 1 ? row_argmax(x, V, S.sh) : ArgBest{0.f, 0};
  __syncthreads();   // the candidate slots are initialised before any thread fills them
  if (mode == 0) {
    if (threadIdx.x == 0 && V > 0) {
      cv[0] = best.v;
      ci[0] = v_off + best.i;
    }
    return;
  }
  const float invT = 1.f / T;
  if (mode == 1) {
    const uint64_t step = (uint64_t)steps[row];
    ArgBest gb{-INFINITY, 0x7fffffff};
    scan_row(x, V, [&](int i, uint16_t bits, bool ok) {
      if (!ok) return;
      const float u = hash_uniform(seed, (uint64_t)row, step, (uint64_t)(v_off + i));
      gb = better(gb, ArgBest{gumbel_score(bf16_bits_to_float(bits), invT, u), i});
    });
    gb = block_argmax(gb, S.sh);
    if (threadIdx.x == 0 && V > 0) {
      cv[0] = gb.v;
      ci[0] = v_off + gb.i;
    }
    return;
  }
  // modes 2 / 3: the shard's elements with key >= its k-th largest key (k = KC for
  // rows that need the full distribution: the best KC of the shard)
  const int kk = mode == 2 ? k : KC;
  uint32_t floor_key = 0u;
  const GlobalRow scan{x, V};
  if (kk < V) {
    radix_digit(scan, 8, 0u, 0u, 0u, false, best.v, invT, (float)kk, whist, S.hist, &S.digit, &S.above);
    const uint32_t hi = S.digit;
    const float need = (float)kk - S.above;
    radix_digit(scan, 0, 0xFF00u, hi << 8, 0u, false, best.v, invT, need, whist, S.hist, &S.digit, &S.above);
    floor_key = (hi << 8) | S.digit;
  }
  if (threadIdx.x == 0) s_n = 0;
  __syncthreads();
  // elements strictly above the threshold first (at most kk - 1 of them), then ties
  for (int pass = 0; pass < 2; ++pass) {
    scan([&](int i, uint16_t bits, bool ok) {
      if (!ok) return;
      const uint32_t key = bf16_key(bits);
      if (pass == 0 ? key <= floor_key : key != floor_key) return;
      const int slot = atomicAdd(&s_n, 1);
      if (slot < KC) {
        cv[slot] = bf16_bits_to_float(bits);
        ci[slot] = v_off + i;
      }
    });
    __syncthreads();
  }
}

__global__ void __launch_bounds__(kVpThreads)
    vp_combine_kernel(const float* __restrict__ cand_val, const int* __restrict__ cand_idx, int64_t rank_stride, int tp,
                      int B, int KC,
                      int V_total, const float* __restrict__ temperature, const int* __restrict__ top_k,
                      const float* __restrict__ top_p, uint64_t seed, const int* __restrict__ steps, int kmax,
                      int* __restrict__ out) {
  pdl_launch();
  pdl_wait_for(cand_val, cand_idx, temperature, top_k, top_p, steps);
  extern __shared__ __align__(16) uint8_t vp_smem[];
  __shared__ SampleSmem S;
  __shared__ float whist[kVpThreads / 32][256];
  const int row = blockIdx.x;
  const float T = temperature[row];
  const int k = top_k[row];
  const float p = top_p[row];
  const int mode = vp_mode(T, k, p, V_total, kmax);
  if (mode <= 1) {
    // every rank's slot 0: the largest value (greedy) or score (Gumbel), lowest index on ties
    ArgBest b{-INFINITY, 0x7fffffff};
    for (int r = threadIdx.x; r < tp; r += blockDim.x) {
      const size_t o = (size_t)r * rank_stride + (size_t)row * KC;
      if (cand_idx[o] >= 0) b = better(b, ArgBest{cand_val[o], cand_idx[o]});
    }
    b = block_argmax(b, S.sh);
    if (threadIdx.x == 0) out[row] = b.i != 0x7fffffff ? b.i : 0;
    return;
  }
  const int n = tp * KC;
  uint16_t* bits = reinterpret_cast<uint16_t*>(vp_smem);              // [n]
  int* gidx = reinterpret_cast<int*>(vp_smem + ((n * 2 + 15) & ~15));   // [n]
  ArgBest best{-INFINITY, 0x7fffffff};
  int valid = 0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const int r = j / KC, c = j % KC;
    const size_t o = (size_t)r * rank_stride + (size_t)row * KC + c;
    const int gi = cand_idx[o];
    const float v = cand_val[o];
    bits[j] = gi >= 0 ? __bfloat16_as_ushort(__float2bfloat16(v)) : kCandEmpty;
    gidx[j] = gi;
    if (gi >= 0) {
      ++valid;
      best = better(best, ArgBest{v, gi});
    }
  }
  best = block_argmax(best, S.sh);
  const int V = (int)block_sum((float)valid, S.shf);
  const uint64_t step = (uint64_t)steps[row];
  struct MapIdx {
    const int* g;
    __device__ __forceinline__ int operator()(int i) const { return g[i]; }
  };
  const int i = sample_select(CandRow{bits, n}, V, best.v, T, k, p, seed, row, step, MapIdx{gidx}, S, whist);
  if (threadIdx.x == 0) out[row] = (i >= 0 && i < n && gidx[i] >= 0) ? gidx[i] : best.i;
}

void argmax_rows(const void* logits, int64_t ld, int B, int V, int* out, cudaStream_t st) {
  if (B <= 0) return;
  launch_kernel(argmax_kernel, dim3(B), dim3(kSampThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(logits), ld,
                V, out);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void sample_rows(const void* logits, int64_t ld, int B, int V, const float* temperature, const int* top_k,
                 const float* top_p, uint64_t seed, const int* steps, int* out, cudaStream_t st) {
  if (B <= 0) return;
  launch_kernel(sample_kernel, dim3(B), dim3(kSampThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(logits), ld,
                V, temperature, top_k, top_p, seed, steps, out);
  VRM_CUDA_CHECK(cudaGetLastError());
}

size_t vp_combine_smem(int tp, int KC) {
  const int n = tp * KC;
  return (size_t)((n * 2 + 15) & ~15) + (size_t)n * 4;
}

void sample_vp_local(const void* logits, int64_t ld, int B, int Vs, int v_off, int V_total, const float* temperature,
                     const int* top_k, const float* top_p, uint64_t seed, const int* steps, int KC, int kmax,
                     float* cand_val, int* cand_idx, cudaStream_t st) {
  if (B <= 0) return;
  VRM_REQUIRE(KC >= 1 && kmax >= 1 && kmax <= KC, "vocab-parallel sampling: 1 <= kmax <= KC");
  launch_kernel(vp_local_kernel, dim3(B), dim3(kSampThreads), 0, st, reinterpret_cast<const __nv_bfloat16*>(logits),
                ld, Vs, v_off, V_total, temperature, top_k, top_p, seed, steps, KC, kmax, cand_val, cand_idx);
  VRM_CUDA_CHECK(cudaGetLastError());
}

void sample_vp_combine(const float* cand_val, const int* cand_idx, int64_t rank_stride, int tp, int B, int KC,
                       int V_total, const float* temperature, const int* top_k, const float* top_p, uint64_t seed,
                       const int* steps, int kmax, int* out, cudaStream_t st) {
  if (B <= 0) return;
  const size_t smem = vp_combine_smem(tp, KC);
  VRM_REQUIRE(smem <= 160 * 1024, "vocab-parallel sampling: tp * KC candidates exceed shared memory");
  static bool set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (!set[dev & 63]) {
    VRM_CUDA_CHECK(cudaFuncSetAttribute(vp_combine_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024));
    set[dev & 63] = true;
  }
  launch_kernel(vp_combine_kernel, dim3(B), dim3(kVpThreads), smem, st, cand_val, cand_idx, rank_stride, tp, B, KC,
                V_total,
                temperature, top_k, top_p, seed, steps, kmax, out);
  VRM_CUDA_CHECK(cudaGetLastError());
}

}  // namespace vrm
