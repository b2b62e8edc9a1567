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
__device__ void radix_digit(const __nv_bfloat16* __restrict__ x, int V, int shift, uint32_t pref_mask, uint32_t pref,
                            uint32_t floor_key, bool mass, float M, float invT, float target,
                            float (*whist)[256], float* hist, uint32_t* out_digit, float* out_above) {
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int i = threadIdx.x; i < nw * 256; i += blockDim.x) whist[i >> 8][i & 255] = 0.f;
  __syncthreads();
  float* my = whist[w];
  scan_row(x, V, [&](int, uint16_t bits, bool ok) {
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

__global__ void __launch_bounds__(kSampThreads)
    sample_kernel(const __nv_bfloat16* __restrict__ logits, int64_t ld, int V, const float* __restrict__ temperature,
                  const int* __restrict__ top_k, const float* __restrict__ top_p, uint64_t seed,
                  const int* __restrict__ steps, int* __restrict__ out) {
  pdl_launch();
  pdl_wait_for(logits, temperature, top_k, top_p, steps);
  __shared__ ArgBest sh[32];
  __shared__ float shf[32];
  __shared__ float hist[256];
  __shared__ float whist[kSampThreads / 32][256];
  __shared__ uint32_t s_digit;
  __shared__ float s_above;
  const int row = blockIdx.x;
  const __nv_bfloat16* x = logits + (size_t)row * ld;
  const float T = temperature ? temperature[row] : 0.f;

  const ArgBest best = row_argmax(x, V, sh);
  if (!(T > 0.f)) {
    if (threadIdx.x == 0) out[row] = best.i;
    return;
  }
  const float M = best.v;
  const float invT = 1.f / T;
  const int k = top_k ? top_k[row] : 0;
  const float p = top_p ? top_p[row] : 1.f;

  // ---- top-k threshold: count radix select over the two bytes of the 16-bit key
  uint32_t floor_key = 0u;
  if (k > 0 && k < V) {
    radix_digit(x, V, 8, 0u, 0u, 0u, false, M, invT, (float)k, whist, hist, &s_digit, &s_above);
    const uint32_t hi = s_digit;
    const float need = (float)k - s_above;
    radix_digit(x, V, 0, 0xFF00u, hi << 8, 0u, false, M, invT, need, whist, hist, &s_digit, &s_above);
    floor_key = (hi << 8) | s_digit;
  }
  // ---- top-p threshold: mass radix select inside the top-k set
  if (p < 1.f) {
    float z = 0.f;
    scan_row(x, V, [&](int, uint16_t bits, bool ok) {
      if (ok && bf16_key(bits) >= floor_key) z += __expf((bf16_bits_to_float(bits) - M) * invT);
    });
    z = block_sum(z, shf);
    const float target = fmaxf(p, 0.f) * z;
    radix_digit(x, V, 8, 0u, 0u, floor_key, true, M, invT, target, whist, hist, &s_digit, &s_above);
    const uint32_t hi = s_digit;
    const float need = target - s_above;
    radix_digit(x, V, 0, 0xFF00u, hi << 8, floor_key, true, M, invT, need, whist, hist, &s_digit, &s_above);
    const uint32_t pk = (hi << 8) | s_digit;
    floor_key = floor_key > pk ? floor_key : pk;
  }
  // ---- Gumbel-max draw over the kept set
  const uint64_t step = steps ? (uint64_t)steps[row] : 0ull;
  ArgBest gb{-INFINITY, 0x7fffffff};
  scan_row(x, V, [&](int i, uint16_t bits, bool ok) {
    if (!ok || bf16_key(bits) < floor_key) return;
    const float u = hash_uniform(seed, (uint64_t)row, step, (uint64_t)i);
    const float gum = -logf(-logf(u));
    gb = better(gb, ArgBest{(bf16_bits_to_float(bits) - M) * invT + gum, i});
  });
  gb = block_argmax(gb, sh);
  if (threadIdx.x == 0) out[row] = gb.i < V ? gb.i : best.i;
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

}  // namespace vrm
