// Raw-pointer launch interface of every vramancer_b200 CUDA kernel.
//
// The .cu files implement these with plain CUDA (no framework headers), which keeps
// them fast to compile and callable from any host code; torch_ops.cpp wraps them for
// Python with shape/dtype checks.  All pointers are device pointers of the current
// device; every launch goes to `stream`.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstddef>
#include <cstdint>
#include <vector>

namespace vrm {

// ---------------------------------------------------------------- GEMM (gemm_tc.cu)
// Y[M, N] = X[M, K] @ W[N, K]^T (+ bias[N]) in bf16 with fp32 accumulation on tcgen05.
enum GemmEpilogue : int {
  kEpiNone = 0,
  // W rows are interleaved gate/up pairs (row 2j = gate j, row 2j+1 = up j); the output
  // has N/2 columns: Y[m, j] = silu(gate) * up.
  kEpiSiluMul = 1,
};

struct GemmArgs {
  const void* x = nullptr;
  int64_t ldx = 0;
  const void* w = nullptr;
  int64_t ldw = 0;
  const void* bias = nullptr;
  void* out = nullptr;
  int64_t ldo = 0;
  int M = 0, N = 0, K = 0;
  int force_splits = 0;
  int epilogue = kEpiNone;
  const void* residual = nullptr;   // optional: Y += residual[M, N] (same ld as out)
  // optional fused all-reduce over the TP group (decode shapes): instead of storing Y,
  // push the fp32 partial into every rank's receive buffer (see ARPush)
  const struct ARPush* allreduce = nullptr;
  // RMSNorm folded into decode GEMMs (M <= 128, stream-K path).  Producer (needs a
  // residual epilogue): ssq_out[t * ssq_ld + m] = sum over weight tile t's 128 rows of
  // bf16(Y[m, n])^2, for ceil(N / 128) <= ssq_parts_cap tiles.  Consumer: Y[m, :] is
  // scaled by rsqrt(sum_{p < ssq_parts} ssq_in[p * ssq_ld + m] / norm_dim + norm_eps)
  // before bias / SiLU (the norm weight is folded into W's columns).
  float* ssq_out = nullptr;
  const float* ssq_in = nullptr;
  int ssq_ld = 0, ssq_parts = 0, ssq_parts_cap = 0, norm_dim = 0;
  float norm_eps = 0.f;
};

// Push half of the fused tensor-parallel all-reduce (one shot, data-polled).  Every
// rank owns a receive buffer [2 halves][world source ranks][half_floats] bf16
// (cudaMalloc + CUDA IPC, symm.cu) whose free slots hold the "empty" pattern 0x8000
// (bf16 -0.0).  The row-parallel GEMM stores its partial Y[m, n] (rounded to bf16, a
// -0.0 stored as +0.0) at m * N + n of its own slot in half (*epoch & 1) on every rank:
// plain posted stores, no fence and no flag.  ar_norm (ar_norm.cu) polls the values
// themselves until none is empty, then empties the slots again and advances *epoch.
struct ARPush {
  __nv_bfloat16* const* xbuf = nullptr;  // device array [world] of the ranks' receive buffers
  const uint32_t* epoch = nullptr;       // this rank's call counter (device, advanced by ar_norm)
  int rank = 0, world = 1;
  long long half_floats = 0;             // elements per (half, source rank) slot
  // Fused reduce (reduce != 0, stream-K bf16 / e4m3 GEMM): after its push, the same
  // kernel's warps take (token, 128-feature chunk) items of this rank's receive buffer,
  // poll until every rank's values have arrived, sum them in rank order (+ bias) into
  // the bf16 residual stream (in place) and store the chunk's sum of squares of the new
  // residual at ssq_out[chunk * ssq_ld + token] (the next GEMM applies the RMSNorm from
  // them, folded-norm consumer), empty the slots and, last warp of the launch, advance
  // *epoch.  Needs every CTA of the launch resident at once (persistent grid).
  int reduce = 0;
  const void* bias = nullptr;            // bf16 [N] or null
  void* residual = nullptr;              // bf16 [M, N] (row stride N), updated in place
  float* ssq_out = nullptr;              // [ceil(N / 128)][ssq_ld] or null
  int ssq_ld = 0;
  uint32_t* done = nullptr;              // zeroed completion counter of this rank
  unsigned long long spin_limit = 0;     // 0: the library default
};
// Prefill (M > 128) GEMM kernel choice: 0 tiled, 1 stream-K, 2 stream-K 256-token
// tiles, 3 persistent, 4 persistent 256-wide (VRM_GEMM_PREFILL sets the start value).
void gemm_set_prefill_mode(int mode);
void gemm_bf16(const GemmArgs& a, cudaStream_t stream);
// FP8 W8A8: x, w are e4m3 bytes ([M, K], [N, K], strides in bytes); y = (x w^T) *
// scale_x[m] * scale_w[n] (+ bias / residual / silu_mul as gemm_bf16).  K % 128 == 0.
void gemm_fp8(const GemmArgs& a, const float* scale_x, const float* scale_w, cudaStream_t stream);
// Per-row e4m3 quantisation: scale[r] = amax(|x[r]|) / 448, q = e4m3_rn_sat(x / scale).
void fp8_rows_quantize(const void* x, int64_t ldx, int rows, int K, uint8_t* q, float* scale, cudaStream_t stream);
// Debug: per-CTA timeline of the stream-K decode GEMM into buf ([ctas][8] u64 ns), null = off.
void gemm_set_trace(void* buf);

// ---------------------------------------------------------------- mixture of experts (moe.cu, gemm_tc.cu)
// A block of <= BN consecutive rows of the expert-grouped activations, all routed to
// one expert.
struct MoeBlock {
  int expert, row0, nrows, pad;
};
// Routing plan on the device: from expert ids [P = tokens * topk] builds counts,
// offsets, the grouped row of every (token, k) pair, the token of every grouped row and
// the list of BN-row blocks (*num_blocks of at most max_blocks).  E <= 2048.
struct MoePlanArgs {
  const int64_t* ids64 = nullptr;   // [P] expert of each (token, k), row-major [T, topk] ...
  const int* ids32 = nullptr;       // ... or as int32 (exactly one of the two)
  int P = 0, topk = 1, E = 0, BN = 16, max_blocks = 0;
  int* counts = nullptr;            // [E]
  int* offsets = nullptr;           // [E + 1]
  int* row_of = nullptr;            // [P]
  int* tok_of_row = nullptr;        // [P]
  MoeBlock* blocks = nullptr;       // [max_blocks]
  int* num_blocks = nullptr;        // [1]
};
void moe_plan(const MoePlanArgs& a, cudaStream_t stream);
// Router: per token softmax over E bf16 logits (fp32), top-k, optional renormalisation
// of the k weights; then the plan of the chosen ids (plan.ids32 = ids32).  Small
// batches do both in one kernel.
struct MoeRouteArgs {
  const void* logits = nullptr;     // bf16 [T, E], leading dimension ldl
  int64_t ldl = 0;
  int T = 0;
  bool norm_topk = true;
  int* ids32 = nullptr;             // [T, topk] out
  int64_t* ids64 = nullptr;         // [T, topk] out (optional)
  float* weights = nullptr;         // [T, topk] out
  MoePlanArgs plan;
};
void moe_route(const MoeRouteArgs& a, cudaStream_t stream);
// x_perm[r] = x[tok_of_row[r]] for r < P (bf16 rows of K elements)
void moe_gather(const void* x, int64_t ldx, const int* tok_of_row, int P, int K, void* x_perm, int64_t ld_perm,
                cudaStream_t stream);
// Grouped expert GEMM: out[row, :] = x_perm[row, :] @ W[expert(row)]^T for the rows of
// every block (SiLU(gate) * up over interleaved rows with kEpiSiluMul).
struct MoeGemmArgs {
  const void* w = nullptr;          // bf16 [E, N, K] (K-major)
  int E = 0, N = 0, K = 0;
  const void* x_perm = nullptr;     // bf16 [rows_cap, K], leading dimension ldx
  int64_t ldx = 0;
  int rows_cap = 0;
  const void* blocks = nullptr;     // MoeBlock [max_blocks]
  const int* num_blocks = nullptr;
  int max_blocks = 0, BN = 16;
  void* out = nullptr;              // bf16 [rows_cap, N or N/2]
  int64_t ldo = 0;
  int epilogue = kEpiNone;
};
void moe_grouped_gemm(const MoeGemmArgs& a, cudaStream_t stream);
// s[t, :] = sum_k w[t, k] * y_perm[row_of[t * topk + k], :] (+ add[t, :]), fp32 in k order.
// Without residual: out = s.  With residual: residual += s (in place, bf16) and, when
// norm_w is given, out = RMSNorm(residual) * norm_w (the next layer's input norm).
struct MoeCombineArgs {
  const void* y_perm = nullptr;
  int64_t ld_perm = 0;
  const int* row_of = nullptr;
  const float* weights = nullptr;
  int T = 0, topk = 1, H = 0;
  const void* add = nullptr;        // [T, H] (optional)
  void* residual = nullptr;         // [T, H] (optional)
  void* out = nullptr;              // [T, H], leading dimension ldo (may be null with residual and no norm)
  int64_t ldo = 0;
  const void* norm_w = nullptr;     // [H] (optional, needs residual)
  float eps = 1e-6f;
  // expert parallelism: row_of null = rows in pair order; wait for every rank's flag
  // in wait_flags to reach *epoch, and read the half (epoch & 1) of half_rows rows
  const uint32_t* wait_flags = nullptr;
  int wait_world = 0;
  const uint32_t* epoch = nullptr;
  long long half_rows = 0;
};
void moe_combine(const MoeCombineArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- NVFP4 x NVFP4 (nvfp4_bs.cu)
// Rows [0, valid) of x (bf16 [*, K], K % 256 == 0) to e2m1 codes q [rows, K/2] and e4m3
// block scales in 128x4 atoms; rows [valid, rows) zero.  gs_tensor: one fp32 scale for
// the tensor (weights); else a per-row scale amax / (6 * 448) is written to gs_rows.
void nvfp4_rows_quantize(const void* x, int64_t ldx, int valid, int rows, int K, const float* gs_tensor,
                         float* gs_rows, uint8_t* q, uint8_t* sf, cudaStream_t stream);
// out[m, n] = sum_k A[m, k] B[n, k] * gsa[m] * gsb on tcgen05 kind::mxf4nvf4 (bf16 out,
// rows m < M written); A padded to Mpad rows, N % 128 == 0, K % 256 == 0.
// Epilogue: + bias[n], + residual[m, n] (may alias out), or SiLU(gate) * up over
// interleaved weight-row pairs (out has N / 2 columns).
void nvfp4_bs_gemm(const uint8_t* qa, const uint8_t* sfa, const float* gsa, int M, int Mpad, const uint8_t* qb,
                   const uint8_t* sfb, const float* gsb, int N, int K, void* out, int64_t ldo, cudaStream_t stream,
                   const void* bias = nullptr, const void* residual = nullptr, int silu_mul = 0);

// ---------------------------------------------------------------- expert parallelism (moe_ep.cu)
// Expert-parallel MoE over peer memory.  Rank r owns experts [r * E_local, (r + 1) *
// E_local).  Every rank owns symmetric buffers (cudaMalloc + CUDA IPC), each in two
// halves that alternate with the parity of the layer-call epoch:
//   cnt    int  [2][world][E]            routed-pair counts per expert, one row per source rank
//   xrecv  bf16 [2][r_rows][H]           rows received for this rank's experts
//   meta   int  [2][r_rows]              source rank * p_cap + pair index of each received row
//   yback  bf16 [2][p_cap][H]            expert outputs returned for this rank's own pairs
//   flags  u32  [3][world]               count / dispatch / return phase, one word per peer
// with r_rows = world * p_cap + BN_max (the last block's TMA box reads past the rows).
struct MoeEpBuffers {
  int* const* cnt = nullptr;                  // device arrays [world] of the ranks' base pointers
  __nv_bfloat16* const* xrecv = nullptr;
  int* const* meta = nullptr;
  __nv_bfloat16* const* yback = nullptr;
  uint32_t* const* flags = nullptr;
  uint32_t* epoch = nullptr;                  // this rank's call counter (device)
  uint32_t* done = nullptr;                   // this rank's completion counters [2] (device, zero)
  int* meta_local = nullptr;                  // this rank's own meta buffer (host-visible pointer)
  __nv_bfloat16* xrecv_local = nullptr;       // this rank's own receive buffer
  __nv_bfloat16* yback_local = nullptr;       // this rank's own return buffer
  uint32_t* flags_local = nullptr;            // this rank's own flag array
  int rank = 0, world = 1, E = 0, E_local = 0, H = 0;
  int p_cap = 0;                              // pairs per rank (max tokens * topk)
  int r_rows = 0;                             // rows per half of xrecv / meta
};
// Count exchange: advances the epoch; sends this rank's per-expert counts ([E], or zeros
// when T == 0) to every rank and flags them.
void moe_ep_counts(const MoeEpBuffers& b, const int* counts, int T, cudaStream_t stream);
// Dispatch: waits for every rank's counts, then stores the rows of x routed to each
// expert into its owner's xrecv (grouped by local expert, then source rank) with their
// meta tags, and flags the owners.  ids / row_of / offsets come from this rank's plan.
void moe_ep_dispatch(const MoeEpBuffers& b, const void* x, const int* ids32, const int* row_of, const int* offsets,
                     int T, int topk, cudaStream_t stream);
// Owner plan: waits for every rank's dispatch, then builds the block list over this
// rank's experts (row0 includes the half offset).
void moe_ep_owner_plan(const MoeEpBuffers& b, int BN, MoeBlock* blocks, int* num_blocks, int max_blocks,
                       cudaStream_t stream);
// Grouped down projection whose epilogue returns each row to its source rank's yback
// (posted NVLink stores), then flags every rank when its last CTA finishes.
void moe_ep_grouped_return(const MoeEpBuffers& b, const MoeGemmArgs& g, cudaStream_t stream);
// Combine on the source rank: waits for every owner's return flag, then the weighted
// k-order sum of yback rows (+ add, residual, next RMSNorm) as moe_combine.
void moe_ep_combine(const MoeEpBuffers& b, const MoeCombineArgs& c, cudaStream_t stream);

// ---------------------------------------------------------------- norms / rope / elementwise (norm_rope.cu)
// out = norm(x [+ residual]); when residual != null the sum is stored back into it.
void rmsnorm(const void* x, int64_t ldx, void* residual, const void* w, void* out, int64_t ldo, int T, int H,
             float eps, cudaStream_t stream);
void layernorm(const void* x, int64_t ldx, void* residual, const void* w, const void* b, void* out, int64_t ldo,
               int T, int H, float eps, cudaStream_t stream);

// Reduce half of the fused all-reduce, fused with the residual update and the next
// norm.  Waits (bounded) until every peer's flag for this rank reaches *epoch, then per
// row: s = sum over source ranks in rank order of the slots (+ bias) (+ residual),
// rounded to bf16 and stored back into residual; then
//   mode kArAdd:       out = s (if out != residual)
//   mode kArRmsNorm:   out = rmsnorm(s) * w
//   mode kArLayerNorm: out = layernorm(s) * w + b
// Every rank sums the same values in the same order: identical results on all ranks.
enum ArNormMode { kArAdd = 0, kArRmsNorm = 1, kArLayerNorm = 2 };
struct ARNormArgs {
  __nv_bfloat16* xbuf = nullptr;     // this rank's receive buffer (emptied after reading)
  uint32_t* epoch = nullptr;         // this rank's call counter (advanced here)
  uint32_t* done = nullptr;          // zeroed CTA completion counter (device)
  int rank = 0, world = 1;
  long long half_floats = 0;
  int T = 0, H = 0;
  const void* bias = nullptr;        // bf16 [H] or null
  void* residual = nullptr;          // bf16 [T, H] in/out or null
  const void* w = nullptr;           // norm weight [H]
  const void* b = nullptr;           // layernorm bias [H]
  void* out = nullptr;               // bf16 [T, ldo]
  int64_t ldo = 0;
  int mode = kArAdd;
  float eps = 1e-6f;
  // clock cycles one CTA polls for missing values before it reports kErrFlagTimeout
  // (missing values count as 0); 0 = the library default (about one second)
  unsigned long long spin_limit = 0;
  uint32_t* err = nullptr;           // null = the per-device error word
};
void ar_norm(const ARNormArgs& a, cudaStream_t stream);

// ---------------------------------------------------------------- NVFP4 weights (nvfp4.cu)
// Quantises W bf16 [N, K] (N % 16 == 0, K % 64 == 0) with the per-tensor scale *gs
// (= amax / (6 * 448), on the device) into q [N * K / 2] and s [N * K / 16] bytes in
// fragment order; dequantises back to bf16 [N, K] row-major.
void nvfp4_quantize(const void* w, int64_t ldw, int N, int K, const float* gs, uint8_t* q, uint8_t* s,
                    cudaStream_t stream);
void nvfp4_dequantize(const uint8_t* q, const uint8_t* s, const float* gs, int N, int K, void* out,
                      cudaStream_t stream);
// W4A16 GEMM for decode (M <= nvfp4_gemm_max_m()): out[M, N] = x @ W'^T (+ bias)
// (+ residual), or the SiLU(gate) * up epilogue over interleaved rows (out [M, N/2]).
struct Nvfp4GemmArgs {
  const void* x = nullptr;      // bf16 [M, K]
  int64_t ldx = 0;
  const uint8_t* q = nullptr;
  const uint8_t* s = nullptr;
  const float* gs = nullptr;
  const void* bias = nullptr;
  const void* residual = nullptr;   // bf16 [M, N], leading dimension ldo
  void* out = nullptr;
  int64_t ldo = 0;
  int M = 0, N = 0, K = 0;
  int epilogue = kEpiNone;
  // fused all-reduce push (push != 0): the partial (times the per-tensor scale, no bias
  // or residual) goes to this rank's slot of every rank's receive buffer instead of out
  int push = 0;
  ARPush ar;
};
void nvfp4_gemm(const Nvfp4GemmArgs& a, cudaStream_t stream);
// W4A16 decode GEMM on tcgen05 (M <= 128) over the block-scaled layout of nvfp4_bs.cu:
// codes uint8 [N, K/2] row-major, e4m3 scale atoms (128 rows x 4 blocks of 16), fp32
// per-tensor scale.  N % 128 == 0, K % 128 == 0.  Epilogues as gemm_bf16.
struct Nvfp4TcArgs {
  const void* x = nullptr;      // bf16 [M, K]
  int64_t ldx = 0;
  const uint8_t* q_rows = nullptr;
  const uint8_t* sf = nullptr;
  const float* gs = nullptr;
  const void* bias = nullptr;
  const void* residual = nullptr;
  void* out = nullptr;
  int64_t ldo = 0;
  int M = 0, N = 0, K = 0;
  int epilogue = kEpiNone;
};
void nvfp4_tc_gemm(const Nvfp4TcArgs& a, cudaStream_t stream);
int nvfp4_gemm_max_m();

// ---------------------------------------------------------------- TurboQuant records (turboquant.cu)
// n vectors of 128 dims (bf16 or fp32) -> n 64-byte records, and back to bf16.
// signs: fp32 [128] rotation signs; jl: fp32 [64, 128] JL matrix.
void tq_compress(const void* x, bool x_bf16, int64_t n, const float* signs, const float* jl, uint8_t* out,
                 cudaStream_t stream);
void tq_decompress(const uint8_t* rec, int64_t n, const float* signs, void* out, cudaStream_t stream);
// TurboQuant KV pages: pool [pages, layers, 2, KH, 16, 64] uint8 records (D = 128).
// tq_kv_write: the rotated k / v rows of qkv [T, (Hq + 2 KH) * 128] -> records at
// slot_mapping (< 0 skips).  tq_paged_decode: decode attention scored from the records
// (asymmetric QJL estimator), values from their polar decodes; out [B, Hq * 128] bf16.
void tq_kv_write(const void* qkv, int64_t ld, int T, int Hq, int KH, const int* slot_mapping, uint8_t* pool,
                 int num_layers, int layer, int64_t num_pages, const float* signs, const float* jl,
                 cudaStream_t stream);
void tq_paged_decode(const void* q, int64_t ld_q, const uint8_t* pool, int num_layers, int layer, int KH, int Hq,
                     const int* block_tables, int bt_stride, const int* context_lens, int B, const float* signs,
                     const float* jl, float sm_scale, void* out, int64_t ld_o, int64_t num_pages,
                     cudaStream_t stream);

struct RopeKvArgs {
  void* qkv = nullptr;          // bf16 [T, (Hq + 2 KH) * D], rotated in place
  int64_t ld_qkv = 0;
  int T = 0, Hq = 0, KH = 0, D = 0;
  const int* positions = nullptr;   // [T] (null: no rotation)
  const float* cos_sin = nullptr;   // [max_pos, rot_dim] = [cos | sin]
  int rot_dim = 0;
  void* cache = nullptr;            // [pages, layers, 2, KH, page_size, row]
  bool cache_fp8 = false;
  bool cache_q4 = false;            // four-bit rows: D/2 code bytes + D/32 fp16 {scale, min}
  int num_layers = 0, layer = 0, page_size = 16;
  const int* slot_mapping = nullptr;   // [T] page * page_size + offset, < 0 skips
  const float* kv_scale = nullptr;     // [layers, 2, KH] (fp8 only)
  int64_t num_pages = 0;               // pool pages (checked in bounds-check builds)
  uint32_t* err = nullptr;             // error word (set by rope_kv_write)
};
void rope_kv_write(const RopeKvArgs& a, cudaStream_t stream);
// per-head RMSNorm of the q and k heads of qkv [T, ld] in place (Qwen3 q_norm / k_norm)
void qk_rmsnorm(void* qkv, int64_t ld, const void* wq, const void* wk, int T, int Hq, int KH, int D, float eps,
                cudaStream_t stream);

void silu_mul(const void* x, int64_t ldx, void* out, int64_t ldo, int T, int I, cudaStream_t stream);
void gelu_tanh(void* x, size_t n, cudaStream_t stream);
void embedding(const int* ids, const void* table, const int* pos, const void* pos_table, void* out, int T, int H,
               cudaStream_t stream);
void add_inplace(void* a, const void* b, size_t n, cudaStream_t stream);

// ---------------------------------------------------------------- attention (attention.cu)
struct DecodeAttnArgs {
  const void* q = nullptr;   // bf16, token b head h at q + b*ld_q + h*D
  int64_t ld_q = 0;
  const void* cache = nullptr;
  bool cache_fp8 = false;
  bool cache_q4 = false;   // four-bit rows (see RopeKvArgs)
  int num_layers = 0, layer = 0, KH = 0, D = 0, Hq = 0;
  const int* block_tables = nullptr;   // [B, bt_stride]
  int bt_stride = 0;
  const int* context_lens = nullptr;   // [B]
  const float* kv_scale = nullptr;     // [layers, 2, KH] (fp8 only)
  float sm_scale = 1.f;
  void* out = nullptr;                 // bf16, token b head h at out + b*ld_o + h*D
  int64_t ld_o = 0;
  int B = 0;
  int max_pages = 0;                   // upper bound on pages per sequence (split choice)
  int num_splits = 0;                  // 0: choose from B, KH and max_pages
  // scratch for split partials; null -> the per-device workspace is used
  float* ws = nullptr;
  size_t ws_bytes = 0;
  uint32_t* counters = nullptr;        // >= B*KH zeroed words; null -> per-device counters
  // pages in the pool (its first dimension): > 0 enables the persistent TMA kernel for
  // bf16 pages (0 keeps the per-(sequence, head, split) kernel)
  int64_t cache_pages = 0;
  // fused RoPE + KV write of this step's token (positions != null): q is the
  // unrotated qkv row [Hq q | KH k | KH v heads]; the cache is written at slot_mapping
  const int* positions = nullptr;      // [B]
  const float* cos_sin = nullptr;      // [max_pos, rot_dim] or null (no rotation)
  int rot_dim = 0;                     // must equal D when cos_sin is given
  const int* slot_mapping = nullptr;   // [B], -1 = no write
  // device word that bounds / timeout errors are OR-ed into; null -> the per-device
  // error word (error_word())
  uint32_t* err = nullptr;
  // optional L2 prefetch of the bytes the next kernel streams (the o_proj weights): the
  // CTAs issue bulk L2 prefetches of equal slices at their start, so those bytes load
  // while attention, which leaves HBM bandwidth spare at short contexts, runs
  const void* l2_prefetch = nullptr;   // 16-byte aligned
  uint64_t l2_prefetch_bytes = 0;      // multiple of 16
};
void paged_attention_decode(const DecodeAttnArgs& a, cudaStream_t stream);
// Selects the persistent TMA decode kernel for bf16 pages (default off, VRM_DECODE_TMA=1).
void set_decode_tma(bool on);
// Scratch bytes paged_attention_decode needs for a given split count.
size_t decode_attention_scratch_bytes(int B, int Hq, int D, int splits);
int decode_attention_choose_splits(int B, int KH, int max_pages);

struct PrefillAttnArgs {
  const void* q = nullptr;   // bf16 [T_total, ...], token t head h at q + t*ld_q + h*D
  int64_t ld_q = 0;
  const void* cache = nullptr;
  bool cache_fp8 = false;
  bool cache_q4 = false;   // four-bit rows (see RopeKvArgs)
  int num_layers = 0, layer = 0, KH = 0, D = 0, Hq = 0;
  const int* block_tables = nullptr;
  int bt_stride = 0;
  const int* cu_q = nullptr;           // [B + 1] query offsets
  const int* context_lens = nullptr;   // [B] total keys (prefix + new)
  const float* kv_scale = nullptr;
  float sm_scale = 1.f;
  void* out = nullptr;
  int64_t ld_o = 0;
  int B = 0, max_q_len = 0;
  int64_t cache_pages = 0;             // pool pages (checked in bounds-check builds)
  int64_t num_tokens = 0;              // rows of q (> 0 enables the tcgen05 kernel for bf16 pages)
};
void paged_attention_prefill(const PrefillAttnArgs& a, cudaStream_t stream);
// Selects the tcgen05 prefill kernel for bf16 pages (default off, VRM_PREFILL_TC=1 on).
void set_prefill_tc(bool on);

// ---------------------------------------------------------------- sampling (sampling.cu)
void argmax_rows(const void* logits, int64_t ld, int B, int V, int* out, cudaStream_t stream);
void sample_rows(const void* logits, int64_t ld, int B, int V, const float* temperature, const int* top_k,
                 const float* top_p, uint64_t seed, const int* steps, int* out, cudaStream_t stream);
// Vocabulary-parallel sampling: a rank's logits shard [B, Vs] (columns v_off.. of a
// V_total vocabulary) -> KC candidates per row (cand_val fp32, cand_idx int32, [B, KC]);
// after an all-gather of every rank's candidates (rank r's at r * rank_stride elements
// from cand_val / cand_idx) the combine picks the same token on every rank.  Rows with top-k > kmax, or top-p < 1 without top-k, need
// the full logits (sampling.cu explains the exactness conditions).
void sample_vp_local(const void* logits, int64_t ld, int B, int Vs, int v_off, int V_total, const float* temperature,
                     const int* top_k, const float* top_p, uint64_t seed, const int* steps, int KC, int kmax,
                     float* cand_val, int* cand_idx, cudaStream_t stream);
void sample_vp_combine(const float* cand_val, const int* cand_idx, int64_t rank_stride, int tp, int B, int KC,
                       int V_total, const float* temperature, const int* top_k, const float* top_p, uint64_t seed,
                       const int* steps, int kmax, int* out, cudaStream_t stream);

// ---------------------------------------------------------------- symmetric buffers (symm.cu)
void* symm_malloc(size_t bytes);
void symm_free(void* p);
// Fills count 16-bit words at p (current device) with value and waits for it.
void symm_fill_u16(void* p, size_t count, uint16_t value);

// ---------------------------------------------------------------- virtual memory regions (vmm.cpp)
// One reserved virtual range whose chunks are backed by physical memory on chosen
// devices and readable / writable from the listed devices.
size_t vmm_granularity(int device);
uint64_t vmm_reserve(size_t bytes, size_t alignment);
void vmm_map(uint64_t base, size_t offset, size_t bytes, int location_device, const std::vector<int>& access,
             bool shareable);
int vmm_export_fd(uint64_t base, size_t offset);
void vmm_map_fd(uint64_t base, size_t offset, size_t bytes, int fd, const std::vector<int>& access);
void vmm_unmap(uint64_t base, size_t offset);
void vmm_free(uint64_t base);
std::vector<uint8_t> ipc_handle(void* p);
void* ipc_open(const std::vector<uint8_t>& bytes);
void ipc_close(void* p);

// ---------------------------------------------------------------- KV page migration (migrate.cu)
// dst_pool[dst_idx[i]] <- src_pool[src_idx[i]] for whole pages of page_bytes; runs on the
// current (source) device; dst_pool may be a peer GPU's memory (peer access enabled).
// src_pages / dst_pages: the pools' page counts (checked in bounds-check builds; 0 = unknown)
void page_copy(const void* src_pool, void* dst_pool, const int* src_idx, const int* dst_idx, int n_pages,
               size_t page_bytes, cudaStream_t stream, int64_t src_pages = 0, int64_t dst_pages = 0);
// Enables device -> peer access for this process (no-op if already enabled); false if unsupported.
bool enable_peer_access(int device, int peer);

}  // namespace vrm
