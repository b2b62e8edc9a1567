// PyTorch bindings (module vramancer_b200._C): shape/dtype checks around the raw
// launchers of vrm_kernels.h.  Every op runs on the current CUDA stream.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "vrm_host.h"
#include "vrm_kernels.h"

namespace {

using torch::Tensor;
using OptT = c10::optional<Tensor>;

cudaStream_t cur_stream() { return at::cuda::getCurrentCUDAStream(); }

bool has(const OptT& t) { return t.has_value() && t->defined(); }

// Every tensor argument of one launch must live on the same device as `ref`: a kernel
// given another GPU's pointer would fault instead of failing here.
void same_device(const Tensor& ref, std::initializer_list<const Tensor*> ts, const char* op) {
  for (const Tensor* t : ts)
    if (t && t->defined())
      TORCH_CHECK(t->device() == ref.device(), op, ": all tensors must be on ", ref.device(), ", got one on ",
                  t->device());
}
void same_device_opt(const Tensor& ref, std::initializer_list<const OptT*> ts, const char* op) {
  for (const OptT* t : ts)
    if (t && has(*t))
      TORCH_CHECK((*t)->device() == ref.device(), op, ": all tensors must be on ", ref.device(), ", got one on ",
                  (*t)->device());
}

void check_bf16_2d(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, ": must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kBFloat16, name, ": must be bf16");
  TORCH_CHECK(t.dim() == 2 && t.stride(1) == 1, name, ": must be 2-D with unit inner stride");
}

bool is_fp8_cache(const Tensor& cache) { return cache.scalar_type() == torch::kFloat8_e4m3fn; }

// uint8 pools hold four-bit rows: head_dim/2 code bytes + head_dim/8 bytes of fp16
// {scale, min} pairs, so the last dimension is head_dim * 5 / 8
bool is_q4_cache(const Tensor& cache) { return cache.scalar_type() == torch::kUInt8; }

int64_t cache_head_dim(const Tensor& cache) { return is_q4_cache(cache) ? cache.size(5) * 8 / 5 : cache.size(5); }

void check_cache(const Tensor& cache) {
  TORCH_CHECK(cache.is_cuda() && cache.dim() == 6 && cache.is_contiguous(),
              "kv cache must be a contiguous [pages, layers, 2, kv_heads, page_size, row] CUDA tensor");
  TORCH_CHECK(cache.size(2) == 2, "kv cache dim 2 must be 2 (k, v)");
  TORCH_CHECK(is_fp8_cache(cache) || is_q4_cache(cache) || cache.scalar_type() == torch::kBFloat16,
              "kv cache dtype must be bf16, fp8 or uint8 (four-bit rows)");
  if (is_q4_cache(cache))
    TORCH_CHECK(cache.size(5) == 80 || cache.size(5) == 40,
                "four-bit kv cache rows must be 80 (head_dim 128) or 40 (head_dim 64) bytes");
}

// ---------------------------------------------------------------- GEMM
void gemm_out(const Tensor& x, const Tensor& w, const OptT& bias, Tensor& out, int64_t force_splits, int64_t epilogue,
              const OptT& residual, const OptT& ssq_out, const OptT& ssq_in, int64_t ssq_parts, double norm_eps) {
  check_bf16_2d(x, "gemm x");
  check_bf16_2d(w, "gemm w");
  check_bf16_2d(out, "gemm out");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm: K mismatch (", K, " vs ", w.size(1), ")");
  same_device(x, {&w, &out}, "gemm");
  same_device_opt(x, {&bias, &residual}, "gemm");
  const int64_t n_out = epilogue == vrm::kEpiSiluMul ? N / 2 : N;
  TORCH_CHECK(out.size(0) == M && out.size(1) == n_out, "gemm: out must be [", M, ", ", n_out, "]");
  vrm::GemmArgs a;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  if (has(bias)) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
                "gemm: bias must be contiguous bf16 [N]");
    a.bias = bias->data_ptr();
  }
  if (has(residual)) {
    check_bf16_2d(*residual, "gemm residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(0) == out.stride(0),
                "gemm: residual must match out");
    a.residual = residual->data_ptr();
  }
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  for (const OptT* t : {&ssq_out, &ssq_in}) {
    if (has(*t)) {
      TORCH_CHECK((*t)->scalar_type() == torch::kFloat32 && (*t)->is_contiguous() && (*t)->dim() == 2,
                  "gemm: norm sums must be contiguous fp32 [parts, tokens]");
      same_device(x, {&**t}, "gemm");
    }
  }
  if (has(ssq_out)) {
    a.ssq_out = ssq_out->data_ptr<float>();
    a.ssq_ld = (int)ssq_out->size(1);
    a.ssq_parts_cap = (int)ssq_out->size(0);
  }
  if (has(ssq_in)) {
    TORCH_CHECK(ssq_parts > 0 && ssq_parts <= ssq_in->size(0), "gemm: ssq_parts out of range");
    a.ssq_in = ssq_in->data_ptr<float>();
    a.ssq_ld = (int)ssq_in->size(1);
    a.ssq_parts = (int)ssq_parts;
    a.norm_dim = (int)K;
    a.norm_eps = (float)norm_eps;
  }
  a.K = (int)K;
  a.force_splits = (int)force_splits;
  a.epilogue = (int)epilogue;
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::gemm_bf16(a, cur_stream());
}

Tensor gemm(const Tensor& x, const Tensor& w, const OptT& bias, int64_t force_splits, int64_t epilogue) {
  const int64_t n_out = epilogue == vrm::kEpiSiluMul ? w.size(0) / 2 : w.size(0);
  auto out = torch::empty({x.size(0), n_out}, x.options());
  gemm_out(x, w, bias, out, force_splits, epilogue, c10::nullopt, c10::nullopt, c10::nullopt, 0, 0.0);
  return out;
}

// ---------------------------------------------------------------- norms
void rmsnorm(const Tensor& x, const OptT& residual, const Tensor& w, Tensor& out, double eps) {
  check_bf16_2d(x, "rmsnorm x");
  check_bf16_2d(out, "rmsnorm out");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.numel() == x.size(1), "rmsnorm: weight");
  TORCH_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "rmsnorm: row strides must be multiples of 8");
  same_device(x, {&w, &out}, "rmsnorm");
  same_device_opt(x, {&residual}, "rmsnorm");
  void* rp = nullptr;
  if (has(residual)) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes() &&
                    residual->scalar_type() == torch::kBFloat16,
                "rmsnorm: residual must be contiguous bf16 like x");
    rp = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::rmsnorm(x.data_ptr(), x.stride(0), rp, w.data_ptr(), out.data_ptr(), out.stride(0), (int)x.size(0),
               (int)x.size(1), (float)eps, cur_stream());
}

void layernorm(const Tensor& x, const OptT& residual, const Tensor& w, const Tensor& b, Tensor& out, double eps) {
  check_bf16_2d(x, "layernorm x");
  check_bf16_2d(out, "layernorm out");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.is_contiguous() && w.numel() == x.size(1), "layernorm: weight");
  TORCH_CHECK(b.scalar_type() == torch::kBFloat16 && b.is_contiguous() && b.numel() == x.size(1), "layernorm: bias");
  TORCH_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 8 == 0, "layernorm: row strides must be multiples of 8");
  same_device(x, {&w, &b, &out}, "layernorm");
  same_device_opt(x, {&residual}, "layernorm");
  void* rp = nullptr;
  if (has(residual)) {
    TORCH_CHECK(residual->is_contiguous() && residual->sizes() == x.sizes() &&
                    residual->scalar_type() == torch::kBFloat16,
                "layernorm: residual must be contiguous bf16 like x");
    rp = residual->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::layernorm(x.data_ptr(), x.stride(0), rp, w.data_ptr(), b.data_ptr(), out.data_ptr(), out.stride(0),
                 (int)x.size(0), (int)x.size(1), (float)eps, cur_stream());
}

// ---------------------------------------------------------------- rope + kv write
void rope_kv_write(Tensor& qkv, const OptT& positions, const OptT& cos_sin, Tensor& cache, const OptT& slot_mapping,
                   const OptT& kv_scale, int64_t layer, int64_t Hq, int64_t KH, int64_t D) {
  check_bf16_2d(qkv, "rope qkv");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * KH) * D, "rope: qkv width must be (Hq + 2 KH) * D");
  check_cache(cache);
  TORCH_CHECK(cache.size(3) == KH && cache_head_dim(cache) == D, "rope: cache kv_heads/head_dim mismatch");
  TORCH_CHECK(layer >= 0 && layer < cache.size(1), "rope: layer out of range");
  same_device(qkv, {&cache}, "rope_kv_write");
  same_device_opt(qkv, {&positions, &cos_sin, &slot_mapping, &kv_scale}, "rope_kv_write");
  vrm::RopeKvArgs a;
  a.qkv = qkv.data_ptr();
  a.ld_qkv = qkv.stride(0);
  a.T = (int)qkv.size(0);
  a.Hq = (int)Hq;
  a.KH = (int)KH;
  a.D = (int)D;
  if (has(cos_sin)) {
    TORCH_CHECK(has(positions) && positions->scalar_type() == torch::kInt32 && positions->numel() >= a.T,
                "rope: int32 positions required");
    TORCH_CHECK(cos_sin->scalar_type() == torch::kFloat32 && cos_sin->is_contiguous() && cos_sin->dim() == 2,
                "rope: cos_sin must be contiguous fp32 [max_pos, rot_dim]");
    TORCH_CHECK(cos_sin->size(1) <= D && cos_sin->size(1) % 2 == 0, "rope: rot_dim");
    a.positions = positions->data_ptr<int>();
    a.cos_sin = cos_sin->data_ptr<float>();
    a.rot_dim = (int)cos_sin->size(1);
  }
  a.cache = cache.data_ptr();
  a.cache_fp8 = is_fp8_cache(cache);
  a.cache_q4 = is_q4_cache(cache);
  a.num_pages = cache.size(0);
  a.num_layers = (int)cache.size(1);
  a.layer = (int)layer;
  a.page_size = (int)cache.size(4);
  if (has(slot_mapping)) {
    TORCH_CHECK(slot_mapping->scalar_type() == torch::kInt32 && slot_mapping->numel() >= a.T, "rope: int32 slots");
    a.slot_mapping = slot_mapping->data_ptr<int>();
  }
  if (has(kv_scale)) {
    TORCH_CHECK(kv_scale->scalar_type() == torch::kFloat32 && kv_scale->is_contiguous() &&
                    kv_scale->numel() == cache.size(1) * 2 * KH,
                "rope: kv_scale must be fp32 [layers, 2, kv_heads]");
    a.kv_scale = kv_scale->data_ptr<float>();
  }
  TORCH_CHECK(!a.cache_fp8 || a.kv_scale, "rope: fp8 cache needs kv_scale");
  const c10::cuda::CUDAGuard guard(qkv.device());
  vrm::rope_kv_write(a, cur_stream());
}

void qk_rmsnorm(Tensor& qkv, const Tensor& wq, const Tensor& wk, int64_t Hq, int64_t KH, int64_t D, double eps) {
  check_bf16_2d(qkv, "qk_rmsnorm qkv");
  TORCH_CHECK(qkv.size(1) == (Hq + 2 * KH) * D, "qk_rmsnorm: qkv width must be (Hq + 2 KH) * D");
  for (const Tensor* w : {&wq, &wk})
    TORCH_CHECK(w->scalar_type() == torch::kBFloat16 && w->is_contiguous() && w->numel() == D,
                "qk_rmsnorm: norm weights must be contiguous bf16 [head_dim]");
  same_device(qkv, {&wq, &wk}, "qk_rmsnorm");
  const c10::cuda::CUDAGuard guard(qkv.device());
  vrm::qk_rmsnorm(qkv.data_ptr(), qkv.stride(0), wq.data_ptr(), wk.data_ptr(), (int)qkv.size(0), (int)Hq, (int)KH,
                  (int)D, (float)eps, cur_stream());
}

// ---------------------------------------------------------------- elementwise
void silu_mul(const Tensor& x, Tensor& out) {
  check_bf16_2d(x, "silu_mul x");
  check_bf16_2d(out, "silu_mul out");
  TORCH_CHECK(out.size(0) == x.size(0) && out.size(1) * 2 == x.size(1), "silu_mul: out must be [T, I] for x [T, 2I]");
  same_device(x, {&out}, "silu_mul");
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::silu_mul(x.data_ptr(), x.stride(0), out.data_ptr(), out.stride(0), (int)x.size(0), (int)out.size(1),
                cur_stream());
}

void gelu_tanh_(Tensor& x) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kBFloat16 && x.is_contiguous(), "gelu: contiguous bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::gelu_tanh(x.data_ptr(), x.numel(), cur_stream());
}

void embedding(const Tensor& ids, const Tensor& table, const OptT& pos, const OptT& pos_table, Tensor& out) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == torch::kInt32 && ids.is_contiguous(), "embedding: int32 ids");
  TORCH_CHECK(table.scalar_type() == torch::kBFloat16 && table.is_contiguous() && table.dim() == 2, "embedding: table");
  TORCH_CHECK(out.is_contiguous() && out.size(0) == ids.numel() && out.size(1) == table.size(1), "embedding: out");
  same_device(ids, {&table, &out}, "embedding");
  same_device_opt(ids, {&pos, &pos_table}, "embedding");
  const int* pp = nullptr;
  const void* pt = nullptr;
  if (has(pos_table)) {
    TORCH_CHECK(has(pos) && pos->scalar_type() == torch::kInt32 && pos->is_contiguous(), "embedding: int32 positions");
    TORCH_CHECK(pos_table->scalar_type() == torch::kBFloat16 && pos_table->is_contiguous(), "embedding: pos table");
    pp = pos->data_ptr<int>();
    pt = pos_table->data_ptr();
  }
  const c10::cuda::CUDAGuard guard(ids.device());
  vrm::embedding(ids.data_ptr<int>(), table.data_ptr(), pp, pt, out.data_ptr(), (int)ids.numel(), (int)table.size(1),
                 cur_stream());
}

void add_(Tensor& a, const Tensor& b) {
  TORCH_CHECK(a.is_contiguous() && b.is_contiguous() && a.numel() == b.numel() &&
                  a.scalar_type() == torch::kBFloat16 && b.scalar_type() == torch::kBFloat16,
              "add_: contiguous bf16 of equal size");
  same_device(a, {&b}, "add_");
  const c10::cuda::CUDAGuard guard(a.device());
  vrm::add_inplace(a.data_ptr(), b.data_ptr(), a.numel(), cur_stream());
}

// ---------------------------------------------------------------- attention
void attn_decode(const Tensor& q, const Tensor& cache, int64_t layer, const Tensor& block_tables,
                 const Tensor& context_lens, const OptT& kv_scale, double sm_scale, Tensor& out, int64_t num_splits,
                 int64_t num_q_heads, const OptT& positions, const OptT& cos_sin, const OptT& slot_mapping,
                 const OptT& l2_prefetch) {
  check_cache(cache);
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 2 && q.stride(1) == 1 &&
                  q.stride(0) % 2 == 0,
              "decode: q must be bf16 [B, >= Hq*D] with unit inner stride");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "decode: out");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 && block_tables.stride(1) == 1,
              "decode: block_tables must be int32 [B, max_pages]");
  TORCH_CHECK(context_lens.scalar_type() == torch::kInt32 && context_lens.is_contiguous(), "decode: int32 context_lens");
  const int64_t B = q.size(0);
  TORCH_CHECK(block_tables.size(0) >= B && context_lens.numel() >= B && out.size(0) >= B, "decode: batch sizes");
  TORCH_CHECK(layer >= 0 && layer < cache.size(1), "decode: layer out of range");
  same_device(q, {&cache, &block_tables, &context_lens, &out}, "paged_attention_decode");
  same_device_opt(q, {&kv_scale}, "paged_attention_decode");
  vrm::DecodeAttnArgs a;
  a.q = q.data_ptr();
  a.ld_q = q.stride(0);
  a.cache = cache.data_ptr();
  a.cache_fp8 = is_fp8_cache(cache);
  a.cache_q4 = is_q4_cache(cache);
  a.num_layers = (int)cache.size(1);
  a.layer = (int)layer;
  a.KH = (int)cache.size(3);
  a.D = (int)cache_head_dim(cache);
  a.Hq = (int)num_q_heads;
  TORCH_CHECK(q.size(1) >= a.Hq * a.D && out.size(1) >= a.Hq * a.D, "decode: q/out width");
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.context_lens = context_lens.data_ptr<int>();
  if (has(kv_scale)) {
    TORCH_CHECK(kv_scale->scalar_type() == torch::kFloat32 && kv_scale->is_contiguous(), "decode: fp32 kv_scale");
    a.kv_scale = kv_scale->data_ptr<float>();
  }
  a.sm_scale = (float)sm_scale;
  a.out = out.data_ptr();
  a.ld_o = out.stride(0);
  a.B = (int)B;
  a.max_pages = (int)block_tables.size(1);
  a.num_splits = (int)num_splits;
  a.cache_pages = cache.size(0);
  if (has(l2_prefetch)) {
    same_device_opt(q, {&l2_prefetch}, "paged_attention_decode");
    TORCH_CHECK(l2_prefetch->is_contiguous(), "decode: l2_prefetch must be contiguous");
    const uint64_t bytes = (uint64_t)l2_prefetch->numel() * l2_prefetch->element_size();
    if (reinterpret_cast<uintptr_t>(l2_prefetch->data_ptr()) % 16 == 0 && bytes >= 16) {
      a.l2_prefetch = l2_prefetch->data_ptr();
      a.l2_prefetch_bytes = bytes & ~uint64_t(15);
    }
  }
  if (has(positions)) {
    // fused RoPE + KV write: q is the whole qkv row
    TORCH_CHECK(has(slot_mapping), "decode: fused KV write needs slot_mapping");
    TORCH_CHECK(positions->scalar_type() == torch::kInt32 && positions->is_contiguous() && positions->numel() >= B,
                "decode: int32 positions [B]");
    TORCH_CHECK(slot_mapping->scalar_type() == torch::kInt32 && slot_mapping->is_contiguous() &&
                    slot_mapping->numel() >= B, "decode: int32 slot_mapping [B]");
    TORCH_CHECK(q.size(1) >= (a.Hq + 2 * a.KH) * a.D, "decode: fused KV write needs the qkv row");
    same_device_opt(q, {&positions, &cos_sin, &slot_mapping}, "paged_attention_decode");
    a.positions = positions->data_ptr<int>();
    a.slot_mapping = slot_mapping->data_ptr<int>();
    if (has(cos_sin)) {
      TORCH_CHECK(cos_sin->scalar_type() == torch::kFloat32 && cos_sin->is_contiguous() && cos_sin->dim() == 2,
                  "decode: fp32 cos_sin [max_pos, rot_dim]");
      a.cos_sin = cos_sin->data_ptr<float>();
      a.rot_dim = (int)cos_sin->size(1);
    }
  }
  const c10::cuda::CUDAGuard guard(q.device());
  vrm::paged_attention_decode(a, cur_stream());
}

void attn_prefill(const Tensor& q, const Tensor& cache, int64_t layer, const Tensor& block_tables, const Tensor& cu_q,
                  const Tensor& context_lens, const OptT& kv_scale, double sm_scale, Tensor& out, int64_t max_q_len,
                  int64_t num_q_heads) {
  check_cache(cache);
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 2 && q.stride(1) == 1, "prefill: q");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "prefill: out");
  TORCH_CHECK(cu_q.scalar_type() == torch::kInt32 && cu_q.is_contiguous() && context_lens.scalar_type() == torch::kInt32 &&
                  block_tables.scalar_type() == torch::kInt32 && block_tables.stride(1) == 1,
              "prefill: int32 metadata");
  TORCH_CHECK(layer >= 0 && layer < cache.size(1), "prefill: layer out of range");
  same_device(q, {&cache, &block_tables, &cu_q, &context_lens, &out}, "paged_attention_prefill");
  same_device_opt(q, {&kv_scale}, "paged_attention_prefill");
  vrm::PrefillAttnArgs a;
  a.q = q.data_ptr();
  a.ld_q = q.stride(0);
  a.cache = cache.data_ptr();
  a.cache_fp8 = is_fp8_cache(cache);
  a.cache_q4 = is_q4_cache(cache);
  a.cache_pages = cache.size(0);
  a.num_tokens = q.size(0);
  a.num_layers = (int)cache.size(1);
  a.layer = (int)layer;
  a.KH = (int)cache.size(3);
  a.D = (int)cache_head_dim(cache);
  a.Hq = (int)num_q_heads;
  a.block_tables = block_tables.data_ptr<int>();
  a.bt_stride = (int)block_tables.stride(0);
  a.cu_q = cu_q.data_ptr<int>();
  a.context_lens = context_lens.data_ptr<int>();
  if (has(kv_scale)) {
    TORCH_CHECK(kv_scale->scalar_type() == torch::kFloat32 && kv_scale->is_contiguous(), "prefill: fp32 kv_scale");
    a.kv_scale = kv_scale->data_ptr<float>();
  }
  a.sm_scale = (float)sm_scale;
  a.out = out.data_ptr();
  a.ld_o = out.stride(0);
  a.B = (int)cu_q.numel() - 1;
  a.max_q_len = (int)max_q_len;
  const c10::cuda::CUDAGuard guard(q.device());
  vrm::paged_attention_prefill(a, cur_stream());
}

// ---------------------------------------------------------------- sampling
void argmax(const Tensor& logits, Tensor& out) {
  check_bf16_2d(logits, "argmax logits");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.numel() >= logits.size(0), "argmax: int32 out");
  same_device(logits, {&out}, "argmax");
  const c10::cuda::CUDAGuard guard(logits.device());
  vrm::argmax_rows(logits.data_ptr(), logits.stride(0), (int)logits.size(0), (int)logits.size(1),
                   out.data_ptr<int>(), cur_stream());
}

void sample(const Tensor& logits, const Tensor& temperature, const Tensor& top_k, const Tensor& top_p, int64_t seed,
            const Tensor& steps, Tensor& out) {
  check_bf16_2d(logits, "sample logits");
  const int64_t B = logits.size(0);
  TORCH_CHECK(temperature.scalar_type() == torch::kFloat32 && temperature.numel() >= B, "sample: fp32 temperature");
  TORCH_CHECK(top_k.scalar_type() == torch::kInt32 && top_k.numel() >= B, "sample: int32 top_k");
  TORCH_CHECK(top_p.scalar_type() == torch::kFloat32 && top_p.numel() >= B, "sample: fp32 top_p");
  TORCH_CHECK(steps.scalar_type() == torch::kInt32 && steps.numel() >= B, "sample: int32 steps");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.numel() >= B, "sample: int32 out");
  same_device(logits, {&temperature, &top_k, &top_p, &steps, &out}, "sample");
  const c10::cuda::CUDAGuard guard(logits.device());
  vrm::sample_rows(logits.data_ptr(), logits.stride(0), (int)B, (int)logits.size(1), temperature.data_ptr<float>(),
                   top_k.data_ptr<int>(), top_p.data_ptr<float>(), (uint64_t)seed, steps.data_ptr<int>(),
                   out.data_ptr<int>(), cur_stream());
}

// cand: int32 [2, B, KC]: [0] the candidates' fp32 values (bit patterns), [1] their
// vocabulary indices (-1 = empty), one buffer so that a single all-gather moves both
void sample_vp_local(const Tensor& logits, int64_t v_off, int64_t vocab, const Tensor& temperature,
                     const Tensor& top_k, const Tensor& top_p, int64_t seed, const Tensor& steps, int64_t kmax,
                     Tensor& cand) {
  check_bf16_2d(logits, "sample_vp logits");
  const int64_t B = logits.size(0);
  TORCH_CHECK(temperature.scalar_type() == torch::kFloat32 && temperature.numel() >= B, "sample_vp: fp32 temperature");
  TORCH_CHECK(top_k.scalar_type() == torch::kInt32 && top_k.numel() >= B, "sample_vp: int32 top_k");
  TORCH_CHECK(top_p.scalar_type() == torch::kFloat32 && top_p.numel() >= B, "sample_vp: fp32 top_p");
  TORCH_CHECK(steps.scalar_type() == torch::kInt32 && steps.numel() >= B, "sample_vp: int32 steps");
  TORCH_CHECK(cand.scalar_type() == torch::kInt32 && cand.is_contiguous() && cand.dim() == 3 && cand.size(0) == 2 &&
                  cand.size(1) == B, "sample_vp: int32 cand [2, B, KC]");
  same_device(logits, {&temperature, &top_k, &top_p, &steps, &cand}, "sample_vp_local");
  const c10::cuda::CUDAGuard guard(logits.device());
  int* base = cand.data_ptr<int>();
  const int64_t KC = cand.size(2);
  vrm::sample_vp_local(logits.data_ptr(), logits.stride(0), (int)B, (int)logits.size(1), (int)v_off, (int)vocab,
                       temperature.data_ptr<float>(), top_k.data_ptr<int>(), top_p.data_ptr<float>(), (uint64_t)seed,
                       steps.data_ptr<int>(), (int)KC, (int)kmax, reinterpret_cast<float*>(base), base + B * KC,
                       cur_stream());
}

// gathered: int32 [tp, 2, B, KC], every rank's sample_vp_local output
void sample_vp_combine(const Tensor& gathered, int64_t vocab, const Tensor& temperature, const Tensor& top_k,
                       const Tensor& top_p, int64_t seed, const Tensor& steps, int64_t kmax, Tensor& out) {
  TORCH_CHECK(gathered.is_cuda() && gathered.scalar_type() == torch::kInt32 && gathered.is_contiguous() &&
                  gathered.dim() == 4 && gathered.size(1) == 2, "sample_vp: int32 candidates [tp, 2, B, KC]");
  const int64_t B = gathered.size(2), KC = gathered.size(3);
  TORCH_CHECK(temperature.numel() >= B && top_k.numel() >= B && top_p.numel() >= B && steps.numel() >= B &&
                  out.numel() >= B && out.scalar_type() == torch::kInt32, "sample_vp: per-row inputs");
  same_device(gathered, {&temperature, &top_k, &top_p, &steps, &out}, "sample_vp_combine");
  const c10::cuda::CUDAGuard guard(gathered.device());
  const int* base = gathered.data_ptr<int>();
  vrm::sample_vp_combine(reinterpret_cast<const float*>(base), base + B * KC, 2 * B * KC, (int)gathered.size(0),
                         (int)B, (int)KC, (int)vocab, temperature.data_ptr<float>(), top_k.data_ptr<int>(),
                         top_p.data_ptr<float>(), (uint64_t)seed, steps.data_ptr<int>(), (int)kmax,
                         out.data_ptr<int>(), cur_stream());
}

// ---------------------------------------------------------------- fused GEMM + all-reduce
// Push half: row-parallel GEMM (bf16, or e4m3 with its scales) whose epilogue stores the
// partial into this rank's slot of every rank's receive buffer (ARPush).  Nothing is
// written to a tensor here.
void gemm_ar_push(const Tensor& x, const Tensor& w, const Tensor& xbuf_ptrs, const Tensor& epoch, int64_t rank,
                  int64_t world, int64_t half_floats, const OptT& scale_x, const OptT& scale_w,
                  const OptT& residual, const OptT& bias, const OptT& ssq_out, const OptT& done,
                  int64_t spin_limit) {
  const bool f8 = w.scalar_type() == torch::kFloat8_e4m3fn || w.scalar_type() == torch::kByte;
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && x.dim() == 2 && w.dim() == 2 && x.stride(1) == 1 && w.stride(1) == 1,
              "gemm_ar: 2-D CUDA operands with unit inner stride");
  TORCH_CHECK(f8 ? (x.scalar_type() == torch::kFloat8_e4m3fn || x.scalar_type() == torch::kByte)
                 : (x.scalar_type() == torch::kBFloat16 && w.scalar_type() == torch::kBFloat16),
              "gemm_ar: bf16 x bf16 or e4m3 x e4m3 operands");
  TORCH_CHECK(!f8 || (has(scale_x) && has(scale_w)), "gemm_ar: e4m3 operands need scale_x and scale_w");
  const int64_t M = x.size(0), K = x.size(1), N = w.size(0);
  TORCH_CHECK(w.size(1) == K, "gemm_ar: shapes");
  TORCH_CHECK(M <= 128, "gemm_ar: fused all-reduce is for decode shapes (M <= 128)");
  TORCH_CHECK(M * N <= half_floats, "gemm_ar: output larger than the receive buffer");
  same_device(x, {&w, &xbuf_ptrs, &epoch}, "gemm_ar");
  TORCH_CHECK(xbuf_ptrs.scalar_type() == torch::kInt64 && xbuf_ptrs.numel() == world,
              "gemm_ar: pointer array must be int64 [world]");
  vrm::ARPush ar;
  ar.xbuf = reinterpret_cast<__nv_bfloat16* const*>(xbuf_ptrs.data_ptr());
  ar.epoch = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  ar.rank = (int)rank;
  ar.world = (int)world;
  ar.half_floats = half_floats;
  if (has(residual)) {
    // fused reduce: sum of every rank's partial (+ bias) into the residual stream, norm sums
    same_device_opt(x, {&residual, &bias, &ssq_out, &done}, "gemm_ar");
    TORCH_CHECK(residual->scalar_type() == torch::kBFloat16 && residual->is_contiguous() &&
                    residual->numel() == M * N,
                "gemm_ar: residual must be contiguous bf16 [M, N]");
    TORCH_CHECK(has(done) && done->scalar_type() == torch::kInt32, "gemm_ar: fused reduce needs its done counter");
    if (has(bias))
      TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->numel() == N && bias->is_contiguous(),
                  "gemm_ar: bias bf16 [N]");
    if (has(ssq_out))
      TORCH_CHECK(ssq_out->scalar_type() == torch::kFloat32 && ssq_out->dim() == 2 &&
                      ssq_out->size(0) >= (N + 127) / 128 && ssq_out->size(1) >= M && ssq_out->is_contiguous(),
                  "gemm_ar: ssq_out fp32 [>= ceil(N / 128), >= M]");
    ar.reduce = 1;
    ar.residual = residual->data_ptr();
    ar.bias = has(bias) ? bias->data_ptr() : nullptr;
    ar.ssq_out = has(ssq_out) ? ssq_out->data_ptr<float>() : nullptr;
    ar.ssq_ld = has(ssq_out) ? (int)ssq_out->size(1) : 0;
    ar.done = reinterpret_cast<uint32_t*>(done->data_ptr());
    ar.spin_limit = spin_limit > 0 ? (unsigned long long)spin_limit : 0ull;
  }
  vrm::GemmArgs a;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);   // elements (bf16) or bytes (e4m3)
  a.w = w.data_ptr();
  a.ldw = w.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.allreduce = &ar;
  const c10::cuda::CUDAGuard guard(x.device());
  if (f8) {
    same_device_opt(x, {&scale_x, &scale_w}, "gemm_ar");
    TORCH_CHECK(scale_x->scalar_type() == torch::kFloat32 && scale_w->scalar_type() == torch::kFloat32 &&
                    scale_x->numel() >= M && scale_w->numel() >= N,
                "gemm_ar: fp32 scales [M] and [N]");
    vrm::gemm_fp8(a, scale_x->data_ptr<float>(), scale_w->data_ptr<float>(), cur_stream());
  } else {
    vrm::gemm_bf16(a, cur_stream());
  }
}

// Reduce half fused with bias + residual + norm (ARNormArgs).  xbuf / epoch / done are
// this rank's own device buffers.
void ar_norm(int64_t xbuf, const Tensor& epoch, const Tensor& done, int64_t rank, int64_t world, int64_t half_floats,
             int64_t T, int64_t H, const OptT& bias, const OptT& residual, const OptT& w, const OptT& b,
             const OptT& out, int64_t mode, double eps, int64_t spin_limit, const OptT& err) {
  TORCH_CHECK(epoch.is_cuda() && done.is_cuda(), "ar_norm: epoch and done must be CUDA tensors");
  same_device_opt(epoch, {&bias, &residual, &w, &b, &out, &err}, "ar_norm");
  same_device(epoch, {&done}, "ar_norm");
  for (const OptT* t : {&bias, &residual, &w, &b, &out})
    if (has(*t)) TORCH_CHECK((*t)->scalar_type() == torch::kBFloat16, "ar_norm: bf16 tensors");
  if (has(residual)) TORCH_CHECK(residual->is_contiguous() && residual->numel() == T * H, "ar_norm: residual [T, H]");
  if (has(out)) TORCH_CHECK(out->dim() == 2 && out->size(0) == T && out->size(1) == H && out->stride(1) == 1,
                            "ar_norm: out [T, H]");
  if (has(bias)) TORCH_CHECK(bias->numel() == H && bias->is_contiguous(), "ar_norm: bias [H]");
  if (has(w)) TORCH_CHECK(w->numel() == H && w->is_contiguous(), "ar_norm: weight [H]");
  if (has(b)) TORCH_CHECK(b->numel() == H && b->is_contiguous(), "ar_norm: norm bias [H]");
  if (has(err)) TORCH_CHECK(err->scalar_type() == torch::kInt32 && err->numel() >= 1, "ar_norm: err int32 [1]");
  vrm::ARNormArgs a;
  a.xbuf = reinterpret_cast<__nv_bfloat16*>(xbuf);
  a.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr());
  a.done = reinterpret_cast<uint32_t*>(done.data_ptr());
  a.rank = (int)rank;
  a.world = (int)world;
  a.half_floats = half_floats;
  a.T = (int)T;
  a.H = (int)H;
  a.bias = has(bias) ? bias->data_ptr() : nullptr;
  a.residual = has(residual) ? residual->data_ptr() : nullptr;
  a.w = has(w) ? w->data_ptr() : nullptr;
  a.b = has(b) ? b->data_ptr() : nullptr;
  a.out = has(out) ? out->data_ptr() : nullptr;
  a.ldo = has(out) ? out->stride(0) : H;
  a.mode = (int)mode;
  a.eps = (float)eps;
  a.spin_limit = spin_limit > 0 ? (unsigned long long)spin_limit : 0ull;
  a.err = has(err) ? reinterpret_cast<uint32_t*>(err->data_ptr()) : nullptr;
  const c10::cuda::CUDAGuard guard(epoch.device());
  vrm::ar_norm(a, cur_stream());
}

// ---------------------------------------------------------------- NVFP4 weights
void check_nvfp4(const Tensor& q, const Tensor& sc, const Tensor& gs, int64_t N, int64_t K, const char* op) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kUInt8 && q.is_contiguous() && q.numel() == N * K / 2, op,
              ": q must be contiguous uint8 [N * K / 2]");
  TORCH_CHECK(sc.scalar_type() == torch::kUInt8 && sc.is_contiguous() && sc.numel() == N * K / 16, op,
              ": s must be contiguous uint8 [N * K / 16]");
  TORCH_CHECK(gs.scalar_type() == torch::kFloat32 && gs.numel() == 1, op, ": gs must be one fp32 value");
  TORCH_CHECK(N % 16 == 0 && K % 64 == 0, op, ": N must be a multiple of 16 and K of 64");
  same_device(q, {&sc, &gs}, op);
}

std::vector<Tensor> nvfp4_quantize(const Tensor& w, const Tensor& gs) {
  check_bf16_2d(w, "nvfp4_quantize w");
  const int64_t N = w.size(0), K = w.size(1);
  auto q = torch::empty({N * K / 2}, w.options().dtype(torch::kUInt8));
  auto sc = torch::empty({N * K / 16}, w.options().dtype(torch::kUInt8));
  check_nvfp4(q, sc, gs, N, K, "nvfp4_quantize");
  same_device(w, {&gs}, "nvfp4_quantize");
  const c10::cuda::CUDAGuard guard(w.device());
  vrm::nvfp4_quantize(w.data_ptr(), w.stride(0), (int)N, (int)K, gs.data_ptr<float>(), q.data_ptr<uint8_t>(),
                      sc.data_ptr<uint8_t>(), cur_stream());
  return {q, sc};
}

Tensor nvfp4_dequantize(const Tensor& q, const Tensor& sc, const Tensor& gs, int64_t N, int64_t K) {
  check_nvfp4(q, sc, gs, N, K, "nvfp4_dequantize");
  auto out = torch::empty({N, K}, q.options().dtype(torch::kBFloat16));
  const c10::cuda::CUDAGuard guard(q.device());
  vrm::nvfp4_dequantize(q.data_ptr<uint8_t>(), sc.data_ptr<uint8_t>(), gs.data_ptr<float>(), (int)N, (int)K,
                        out.data_ptr(), cur_stream());
  return out;
}

// W4A16 decode on tcgen05 over the block-scaled layout (q_rows [N, K/2], scale atoms)
void nvfp4_tc_gemm_out(const Tensor& x, const Tensor& q_rows, const Tensor& sf, const Tensor& gs, const OptT& bias,
                       Tensor& out, int64_t epilogue, const OptT& residual) {
  check_bf16_2d(x, "nvfp4_tc x");
  check_bf16_2d(out, "nvfp4_tc out");
  const int64_t M = x.size(0), K = x.size(1);
  TORCH_CHECK(q_rows.is_cuda() && q_rows.scalar_type() == torch::kUInt8 && q_rows.is_contiguous() &&
                  q_rows.dim() == 2 && q_rows.size(1) * 2 == K, "nvfp4_tc: q_rows must be uint8 [N, K/2]");
  const int64_t N = q_rows.size(0);
  TORCH_CHECK(sf.scalar_type() == torch::kUInt8 && sf.is_contiguous() && sf.numel() >= N * K / 16,
              "nvfp4_tc: scale atoms");
  TORCH_CHECK(gs.scalar_type() == torch::kFloat32 && gs.numel() >= 1, "nvfp4_tc: fp32 gs");
  same_device(x, {&q_rows, &sf, &gs, &out}, "nvfp4_tc_gemm");
  same_device_opt(x, {&bias, &residual}, "nvfp4_tc_gemm");
  const int64_t n_out = epilogue == vrm::kEpiSiluMul ? N / 2 : N;
  TORCH_CHECK(out.size(0) == M && out.size(1) == n_out, "nvfp4_tc: out must be [", M, ", ", n_out, "]");
  vrm::Nvfp4TcArgs a;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.q_rows = q_rows.data_ptr<uint8_t>();
  a.sf = sf.data_ptr<uint8_t>();
  a.gs = gs.data_ptr<float>();
  if (has(bias)) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
                "nvfp4_tc: bias must be contiguous bf16 [N]");
    a.bias = bias->data_ptr();
  }
  if (has(residual)) {
    check_bf16_2d(*residual, "nvfp4_tc residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(0) == out.stride(0),
                "nvfp4_tc: residual must match out");
    a.residual = residual->data_ptr();
  }
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.epilogue = (int)epilogue;
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::nvfp4_tc_gemm(a, cur_stream());
}

void nvfp4_gemm_out(const Tensor& x, const Tensor& q, const Tensor& sc, const Tensor& gs, int64_t N,
                    const OptT& bias, Tensor& out, int64_t epilogue, const OptT& residual) {
  check_bf16_2d(x, "nvfp4_gemm x");
  check_bf16_2d(out, "nvfp4_gemm out");
  const int64_t M = x.size(0), K = x.size(1);
  check_nvfp4(q, sc, gs, N, K, "nvfp4_gemm");
  same_device(x, {&q, &out}, "nvfp4_gemm");
  same_device_opt(x, {&bias, &residual}, "nvfp4_gemm");
  const int64_t n_out = epilogue == vrm::kEpiSiluMul ? N / 2 : N;
  TORCH_CHECK(out.size(0) == M && out.size(1) == n_out, "nvfp4_gemm: out must be [", M, ", ", n_out, "]");
  vrm::Nvfp4GemmArgs a;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.q = q.data_ptr<uint8_t>();
  a.s = sc.data_ptr<uint8_t>();
  a.gs = gs.data_ptr<float>();
  if (has(bias)) {
    TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->is_contiguous() && bias->numel() == N,
                "nvfp4_gemm: bias must be contiguous bf16 [N]");
    a.bias = bias->data_ptr();
  }
  if (has(residual)) {
    check_bf16_2d(*residual, "nvfp4_gemm residual");
    TORCH_CHECK(residual->size(0) == M && residual->size(1) == N && residual->stride(0) == out.stride(0),
                "nvfp4_gemm: residual must match out");
    a.residual = residual->data_ptr();
  }
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.epilogue = (int)epilogue;
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::nvfp4_gemm(a, cur_stream());
}

// Fused all-reduce push of the W4A16 decode GEMM: the partial goes to this rank's slot
// of every rank's receive buffer (ARPush); nothing is written to a tensor here.
void nvfp4_gemm_ar_push(const Tensor& x, const Tensor& q, const Tensor& sc, const Tensor& gs, int64_t N,
                        const Tensor& xbuf_ptrs, const Tensor& epoch, int64_t rank, int64_t world,
                        int64_t half_floats) {
  check_bf16_2d(x, "nvfp4_gemm_ar x");
  const int64_t M = x.size(0), K = x.size(1);
  check_nvfp4(q, sc, gs, N, K, "nvfp4_gemm_ar");
  same_device(x, {&q, &xbuf_ptrs, &epoch}, "nvfp4_gemm_ar");
  TORCH_CHECK(xbuf_ptrs.scalar_type() == torch::kInt64 && xbuf_ptrs.numel() == world,
              "nvfp4_gemm_ar: pointer array must be int64 [world]");
  TORCH_CHECK(M * N <= half_floats, "nvfp4_gemm_ar: output larger than the receive buffer");
  vrm::Nvfp4GemmArgs a;
  a.x = x.data_ptr();
  a.ldx = x.stride(0);
  a.q = q.data_ptr<uint8_t>();
  a.s = sc.data_ptr<uint8_t>();
  a.gs = gs.data_ptr<float>();
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.push = 1;
  a.ar.xbuf = reinterpret_cast<__nv_bfloat16* const*>(xbuf_ptrs.data_ptr());
  a.ar.epoch = reinterpret_cast<const uint32_t*>(epoch.data_ptr());
  a.ar.rank = (int)rank;
  a.ar.world = (int)world;
  a.ar.half_floats = half_floats;
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::nvfp4_gemm(a, cur_stream());
}

// ---------------------------------------------------------------- TurboQuant KV records
Tensor tq_compress(const Tensor& x, const Tensor& signs, const Tensor& jl) {
  TORCH_CHECK(x.is_cuda() && x.is_contiguous() && x.size(-1) == 128, "tq_compress: contiguous CUDA [..., 128]");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat32, "tq_compress: bf16 or fp32");
  TORCH_CHECK(signs.scalar_type() == torch::kFloat32 && signs.numel() == 128 && signs.is_contiguous(), "tq_compress: signs");
  TORCH_CHECK(jl.scalar_type() == torch::kFloat32 && jl.numel() == 64 * 128 && jl.is_contiguous(), "tq_compress: jl [64, 128]");
  same_device(x, {&signs, &jl}, "tq_compress");
  auto sizes = x.sizes().vec();
  sizes.back() = 64;
  auto out = torch::empty(sizes, x.options().dtype(torch::kUInt8));
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::tq_compress(x.data_ptr(), x.scalar_type() == torch::kBFloat16, x.numel() / 128, signs.data_ptr<float>(),
                   jl.data_ptr<float>(), out.data_ptr<uint8_t>(), cur_stream());
  return out;
}

// TurboQuant KV pages: pool int8 [pages, layers, 2, KH, 16, 64] (records as bytes)
static void check_tq_pool(const Tensor& pool, int64_t layer, const char* what) {
  TORCH_CHECK(pool.is_cuda() && pool.is_contiguous() && pool.dim() == 6 && pool.size(2) == 2 && pool.size(5) == 64 &&
                  (pool.scalar_type() == torch::kInt8 || pool.scalar_type() == torch::kUInt8),
              what, ": TurboQuant pool must be a contiguous int8 [pages, layers, 2, kv_heads, 16, 64] CUDA tensor");
  TORCH_CHECK(pool.size(4) == 16, what, ": 16-token pages");
  TORCH_CHECK(layer >= 0 && layer < pool.size(1), what, ": layer out of range");
}
static void check_tq_params(const Tensor& signs, const Tensor& jl, const char* what) {
  TORCH_CHECK(signs.scalar_type() == torch::kFloat32 && signs.is_contiguous() && signs.numel() == 128, what,
              ": fp32 signs [128]");
  TORCH_CHECK(jl.scalar_type() == torch::kFloat32 && jl.is_contiguous() && jl.numel() == 64 * 128, what,
              ": fp32 jl [64, 128]");
}

void tq_kv_write(const Tensor& qkv, const Tensor& slot_mapping, Tensor& pool, int64_t layer, int64_t Hq, int64_t KH,
                 const Tensor& signs, const Tensor& jl) {
  check_bf16_2d(qkv, "tq_kv_write qkv");
  check_tq_pool(pool, layer, "tq_kv_write");
  check_tq_params(signs, jl, "tq_kv_write");
  TORCH_CHECK(pool.size(3) == KH && qkv.size(1) >= (Hq + 2 * KH) * 128 && qkv.stride(0) % 4 == 0,
              "tq_kv_write: qkv must hold (Hq + 2 KH) heads of 128 dims");
  TORCH_CHECK(slot_mapping.scalar_type() == torch::kInt32 && slot_mapping.numel() >= qkv.size(0),
              "tq_kv_write: int32 slot_mapping");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(qkv.data_ptr()) & 7) == 0 &&
                  (reinterpret_cast<uintptr_t>(pool.data_ptr()) & 63) == 0,
              "tq_kv_write: qkv 8-byte and pool 64-byte aligned");
  same_device(qkv, {&slot_mapping, &pool, &signs, &jl}, "tq_kv_write");
  const c10::cuda::CUDAGuard guard(qkv.device());
  vrm::tq_kv_write(qkv.data_ptr(), qkv.stride(0), (int)qkv.size(0), (int)Hq, (int)KH, slot_mapping.data_ptr<int>(),
                   reinterpret_cast<uint8_t*>(pool.data_ptr()), (int)pool.size(1), (int)layer, pool.size(0),
                   signs.data_ptr<float>(), jl.data_ptr<float>(), cur_stream());
}

void tq_paged_decode(const Tensor& q, const Tensor& pool, int64_t layer, const Tensor& block_tables,
                     const Tensor& context_lens, const Tensor& signs, const Tensor& jl, double sm_scale, Tensor& out,
                     int64_t num_q_heads) {
  check_tq_pool(pool, layer, "tq_paged_decode");
  check_tq_params(signs, jl, "tq_paged_decode");
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 2 && q.stride(1) == 1 &&
                  q.stride(0) % 4 == 0 && q.size(1) >= num_q_heads * 128,
              "tq_paged_decode: q must be bf16 [B, >= Hq * 128] with unit inner stride");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.dim() == 2 && out.stride(1) == 1 &&
                  out.size(1) >= num_q_heads * 128 && out.stride(0) % 4 == 0, "tq_paged_decode: out");
  TORCH_CHECK(block_tables.scalar_type() == torch::kInt32 && block_tables.dim() == 2 && block_tables.stride(1) == 1,
              "tq_paged_decode: int32 block_tables [B, max_pages]");
  TORCH_CHECK(context_lens.scalar_type() == torch::kInt32 && context_lens.numel() >= q.size(0),
              "tq_paged_decode: int32 context_lens");
  TORCH_CHECK((reinterpret_cast<uintptr_t>(q.data_ptr()) & 7) == 0 && (reinterpret_cast<uintptr_t>(out.data_ptr()) & 7) == 0 &&
                  (reinterpret_cast<uintptr_t>(pool.data_ptr()) & 63) == 0,
              "tq_paged_decode: q / out 8-byte and pool 64-byte aligned");
  same_device(q, {&pool, &block_tables, &context_lens, &signs, &jl, &out}, "tq_paged_decode");
  const c10::cuda::CUDAGuard guard(q.device());
  vrm::tq_paged_decode(q.data_ptr(), q.stride(0), reinterpret_cast<const uint8_t*>(pool.data_ptr()),
                       (int)pool.size(1), (int)layer, (int)pool.size(3), (int)num_q_heads,
                       block_tables.data_ptr<int>(), (int)block_tables.stride(0), context_lens.data_ptr<int>(),
                       (int)q.size(0), signs.data_ptr<float>(), jl.data_ptr<float>(), (float)sm_scale,
                       out.data_ptr(), out.stride(0), pool.size(0), cur_stream());
}

Tensor tq_decompress(const Tensor& rec, const Tensor& signs) {
  TORCH_CHECK(rec.is_cuda() && rec.is_contiguous() && rec.scalar_type() == torch::kUInt8 && rec.size(-1) == 64,
              "tq_decompress: contiguous CUDA uint8 [..., 64]");
  TORCH_CHECK(signs.scalar_type() == torch::kFloat32 && signs.numel() == 128, "tq_decompress: signs");
  same_device(rec, {&signs}, "tq_decompress");
  auto sizes = rec.sizes().vec();
  sizes.back() = 128;
  auto out = torch::empty(sizes, rec.options().dtype(torch::kBFloat16));
  const c10::cuda::CUDAGuard guard(rec.device());
  vrm::tq_decompress(rec.data_ptr<uint8_t>(), rec.numel() / 64, signs.data_ptr<float>(), out.data_ptr(),
                     cur_stream());
  return out;
}

// ---------------------------------------------------------------- mixture of experts
// Routed experts of one MoE layer on the device: plan, gather, grouped gate/up GEMM with
// the SiLU*up epilogue, grouped down GEMM, weighted combine (+ add, e.g. the shared
// expert).  x [T, H], ids int64 [T, topk], weights fp32 [T, topk], gate_up [E, 2I, H]
// (interleaved gate / up rows), down [E, H, I].  No host synchronisation.
// FP8 rows: e4m3 codes [rows, K] and per-row scales.
std::vector<Tensor> fp8_rows_quantize(const Tensor& x) {
  check_bf16_2d(x, "fp8 rows x");
  const c10::cuda::CUDAGuard guard(x.device());
  auto q = torch::empty({x.size(0), x.size(1)}, x.options().dtype(torch::kUInt8));
  auto sc = torch::empty({x.size(0)}, x.options().dtype(torch::kFloat32));
  vrm::fp8_rows_quantize(x.data_ptr(), x.stride(0), (int)x.size(0), (int)x.size(1), q.data_ptr<uint8_t>(),
                         sc.data_ptr<float>(), cur_stream());
  return {q, sc};
}

// y = (x_q w_q^T) * sx[m] * sw[n] (+ bias, + residual, or silu_mul) into out.
void gemm_fp8_out(const Tensor& xq, const Tensor& sx, const Tensor& wq, const Tensor& sw, const OptT& bias,
                  Tensor& out, int64_t epilogue, const OptT& residual) {
  for (const Tensor* t : {&xq, &wq})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kUInt8 && t->dim() == 2 && t->stride(1) == 1,
                "gemm fp8: uint8 (e4m3) [rows, K] operands");
  TORCH_CHECK(sx.scalar_type() == torch::kFloat32 && sw.scalar_type() == torch::kFloat32 &&
                  sx.numel() >= xq.size(0) && sw.numel() >= wq.size(0),
              "gemm fp8: fp32 scales");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.stride(1) == 1, "gemm fp8: bf16 out");
  same_device(xq, {&sx, &wq, &sw, &out}, "gemm fp8");
  same_device_opt(xq, {&bias, &residual}, "gemm fp8");
  const int64_t M = xq.size(0), K = xq.size(1), N = wq.size(0);
  TORCH_CHECK(wq.size(1) == K, "gemm fp8: K mismatch");
  TORCH_CHECK(out.size(0) == M && out.size(1) == (epilogue == vrm::kEpiSiluMul ? N / 2 : N), "gemm fp8: out shape");
  const c10::cuda::CUDAGuard guard(xq.device());
  vrm::GemmArgs a;
  a.x = xq.data_ptr();
  a.ldx = xq.stride(0);
  a.w = wq.data_ptr();
  a.ldw = wq.stride(0);
  a.bias = has(bias) ? bias->data_ptr() : nullptr;
  a.out = out.data_ptr();
  a.ldo = out.stride(0);
  a.M = (int)M;
  a.N = (int)N;
  a.K = (int)K;
  a.epilogue = (int)epilogue;
  a.residual = has(residual) ? residual->data_ptr() : nullptr;
  vrm::gemm_fp8(a, sx.data_ptr<float>(), sw.data_ptr<float>(), cur_stream());
}

// NVFP4 rows (block-scaled format of nvfp4_bs.cu): returns q [rows, K/2], the scale
// atoms, and the per-row scales (empty when gs_tensor is given).
std::vector<Tensor> nvfp4_rows_quantize(const Tensor& x, int64_t rows, const OptT& gs_tensor) {
  check_bf16_2d(x, "nvfp4 rows x");
  const int64_t valid = x.size(0), K = x.size(1);
  TORCH_CHECK(rows >= valid && rows % 128 == 0 && K % 256 == 0, "nvfp4 rows: rows % 128, K % 256");
  const c10::cuda::CUDAGuard guard(x.device());
  auto o8 = x.options().dtype(torch::kUInt8);
  auto q = torch::empty({rows, K / 2}, o8);
  auto sf = torch::empty({rows / 128 * (K / 64) * 512}, o8);
  Tensor gs_rows;
  const float* gt = nullptr;
  if (has(gs_tensor)) {
    TORCH_CHECK(gs_tensor->scalar_type() == torch::kFloat32 && gs_tensor->numel() == 1, "nvfp4 rows: gs fp32 [1]");
    same_device_opt(x, {&gs_tensor}, "nvfp4 rows");
    gt = gs_tensor->data_ptr<float>();
    gs_rows = torch::empty({0}, x.options().dtype(torch::kFloat32));
  } else {
    gs_rows = torch::empty({rows}, x.options().dtype(torch::kFloat32));
  }
  vrm::nvfp4_rows_quantize(x.data_ptr(), x.stride(0), (int)valid, (int)rows, (int)K, gt,
                           gt ? nullptr : gs_rows.data_ptr<float>(), q.data_ptr<uint8_t>(), sf.data_ptr<uint8_t>(),
                           cur_stream());
  return {q, sf, gs_rows};
}

Tensor nvfp4_bs_gemm(const Tensor& qa, const Tensor& sfa, const Tensor& gsa, int64_t M, const Tensor& qb,
                     const Tensor& sfb, const Tensor& gsb, const OptT& bias, const OptT& residual, int64_t epilogue,
                     const OptT& out_opt) {
  for (const Tensor* t : {&qa, &sfa, &qb, &sfb})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kUInt8 && t->is_contiguous(), "nvfp4 bs gemm: uint8 tensors");
  TORCH_CHECK(gsa.scalar_type() == torch::kFloat32 && gsb.scalar_type() == torch::kFloat32 && gsb.numel() == 1,
              "nvfp4 bs gemm: fp32 scales");
  same_device(qa, {&sfa, &gsa, &qb, &sfb, &gsb}, "nvfp4 bs gemm");
  const int64_t Mpad = qa.size(0), K = qa.size(1) * 2, N = qb.size(0);
  TORCH_CHECK(qb.size(1) * 2 == K && gsa.numel() >= M && M <= Mpad, "nvfp4 bs gemm: shapes");
  const c10::cuda::CUDAGuard guard(qa.device());
  const int64_t No = epilogue == vrm::kEpiSiluMul ? N / 2 : N;
  Tensor out = has(out_opt) ? *out_opt : torch::empty({M, No}, qa.options().dtype(torch::kBFloat16));
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.is_contiguous() && out.size(0) == M && out.size(1) == No,
              "nvfp4 bs gemm: out bf16 [M, N or N/2]");
  if (has(bias)) TORCH_CHECK(bias->scalar_type() == torch::kBFloat16 && bias->numel() == N, "nvfp4 bs gemm: bias");
  if (has(residual))
    TORCH_CHECK(residual->scalar_type() == torch::kBFloat16 && residual->is_contiguous() && residual->sizes() == out.sizes(),
                "nvfp4 bs gemm: residual [M, N]");
  same_device_opt(qa, {&bias, &residual, &out_opt}, "nvfp4 bs gemm");
  vrm::nvfp4_bs_gemm(qa.data_ptr<uint8_t>(), sfa.data_ptr<uint8_t>(), gsa.data_ptr<float>(), (int)M, (int)Mpad,
                     qb.data_ptr<uint8_t>(), sfb.data_ptr<uint8_t>(), gsb.data_ptr<float>(), (int)N, (int)K,
                     out.data_ptr(), No, cur_stream(), has(bias) ? bias->data_ptr() : nullptr,
                     has(residual) ? residual->data_ptr() : nullptr, epilogue == vrm::kEpiSiluMul ? 1 : 0);
  return out;
}

// Expert plan of a MoE layer: per-expert counts and row offsets, the grouped row of every
// (token, k) pair, the token of every grouped row and the list of token blocks
// (expert, first row, rows, 0) that drives the grouped GEMM.
struct MoePlanT {
  Tensor counts, offsets, row_of, tok, blocks, nblk;
  int64_t max_blocks;
};

MoePlanT moe_plan_alloc(const torch::TensorOptions& o, int64_t E, int64_t P, int64_t BN) {
  MoePlanT t;
  t.max_blocks = std::min<int64_t>(E, P) + (P + BN - 1) / BN;
  auto oi = o.dtype(torch::kInt32);
  t.counts = torch::empty({E}, oi);
  t.offsets = torch::empty({E + 1}, oi);
  t.row_of = torch::empty({std::max<int64_t>(P, 1)}, oi);
  t.tok = torch::empty({std::max<int64_t>(P, 1)}, oi);
  t.blocks = torch::empty({std::max<int64_t>(1, t.max_blocks), 4}, oi);
  t.nblk = torch::zeros({1}, oi);
  return t;
}

vrm::MoePlanArgs moe_plan_args(MoePlanT& t, int64_t P, int64_t topk, int64_t E, int64_t BN) {
  vrm::MoePlanArgs pa;
  pa.P = (int)P;
  pa.topk = (int)topk;
  pa.E = (int)E;
  pa.BN = (int)BN;
  pa.max_blocks = (int)t.max_blocks;
  pa.counts = t.counts.data_ptr<int>();
  pa.offsets = t.offsets.data_ptr<int>();
  pa.row_of = t.row_of.data_ptr<int>();
  pa.tok_of_row = t.tok.data_ptr<int>();
  pa.blocks = reinterpret_cast<vrm::MoeBlock*>(t.blocks.data_ptr<int>());
  pa.num_blocks = t.nblk.data_ptr<int>();
  return pa;
}

std::vector<Tensor> moe_plan_op(const Tensor& ids, int64_t E, int64_t BN) {
  TORCH_CHECK(ids.is_cuda() && ids.scalar_type() == torch::kInt64 && ids.dim() == 2 && ids.is_contiguous(),
              "moe: ids int64 [T, topk]");
  const int64_t P = ids.numel();
  const c10::cuda::CUDAGuard guard(ids.device());
  auto t = moe_plan_alloc(ids.options(), E, P, BN);
  auto pa = moe_plan_args(t, P, ids.size(1), E, BN);
  pa.ids64 = ids.data_ptr<int64_t>();
  vrm::moe_plan(pa, cur_stream());
  return {t.counts, t.offsets, t.row_of, t.tok, t.blocks, t.nblk};
}

// Router on the device: softmax / top-k / renormalisation of bf16 logits [T, E] and the
// plan.  Returns ids (int64), weights (fp32) and the plan tensors.
std::vector<Tensor> moe_route_op(const Tensor& logits, int64_t topk, bool norm_topk, int64_t BN) {
  check_bf16_2d(logits, "moe logits");
  const int64_t T = logits.size(0), E = logits.size(1), P = T * topk;
  const c10::cuda::CUDAGuard guard(logits.device());
  auto t = moe_plan_alloc(logits.options(), E, P, BN);
  auto ids32 = torch::empty({T, topk}, logits.options().dtype(torch::kInt32));
  auto ids64 = torch::empty({T, topk}, logits.options().dtype(torch::kInt64));
  auto w = torch::empty({T, topk}, logits.options().dtype(torch::kFloat32));
  vrm::MoeRouteArgs ra;
  ra.logits = logits.data_ptr();
  ra.ldl = logits.stride(0);
  ra.T = (int)T;
  ra.norm_topk = norm_topk;
  ra.ids32 = ids32.data_ptr<int>();
  ra.ids64 = ids64.data_ptr<int64_t>();
  ra.weights = w.data_ptr<float>();
  ra.plan = moe_plan_args(t, P, topk, E, BN);
  ra.plan.ids32 = ra.ids32;
  vrm::moe_route(ra, cur_stream());
  return {ids64, w, t.counts, t.offsets, t.row_of, t.tok, t.blocks, t.nblk};
}

// Grouped expert GEMM over a plan: out[r] = x_perm[r] @ w[expert(r)].T for every row r
// of every block (epilogue 1: SiLU(gate)*up over interleaved weight-row pairs).
Tensor moe_grouped_linear(const Tensor& x_perm, const Tensor& w, const Tensor& blocks, const Tensor& nblk, int64_t BN,
                          int64_t epilogue) {
  check_bf16_2d(x_perm, "moe x_perm");
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16 && w.dim() == 3 && w.is_contiguous() && w.size(2) == x_perm.size(1),
              "moe: w bf16 [E, N, K]");
  TORCH_CHECK(blocks.scalar_type() == torch::kInt32 && blocks.dim() == 2 && blocks.size(1) == 4 && blocks.is_contiguous(),
              "moe: blocks int32 [max_blocks, 4]");
  same_device(x_perm, {&w, &blocks, &nblk}, "moe");
  const int64_t N = epilogue == vrm::kEpiSiluMul ? w.size(1) / 2 : w.size(1);
  auto out = torch::empty({x_perm.size(0), N}, x_perm.options());
  const c10::cuda::CUDAGuard guard(x_perm.device());
  vrm::MoeGemmArgs g;
  g.w = w.data_ptr();
  g.E = (int)w.size(0);
  g.N = (int)w.size(1);
  g.K = (int)w.size(2);
  g.x_perm = x_perm.data_ptr();
  g.ldx = x_perm.stride(0);
  g.rows_cap = (int)x_perm.size(0);
  g.blocks = blocks.data_ptr<int>();
  g.num_blocks = nblk.data_ptr<int>();
  g.max_blocks = (int)blocks.size(0);
  g.BN = (int)BN;
  g.out = out.data_ptr();
  g.ldo = N;
  g.epilogue = (int)epilogue;
  vrm::moe_grouped_gemm(g, cur_stream());
  return out;
}

void check_moe_weights(const Tensor& x, const Tensor& gate_up, const Tensor& down) {
  check_bf16_2d(x, "moe x");
  TORCH_CHECK(x.is_contiguous(), "moe: x must be contiguous");
  TORCH_CHECK(gate_up.scalar_type() == torch::kBFloat16 && gate_up.dim() == 3 && gate_up.is_contiguous(),
              "moe: gate_up bf16 [E, 2I, H]");
  TORCH_CHECK(down.scalar_type() == torch::kBFloat16 && down.dim() == 3 && down.is_contiguous(), "moe: down bf16 [E, H, I]");
  const int64_t H = x.size(1), E = gate_up.size(0), I = gate_up.size(1) / 2;
  TORCH_CHECK(gate_up.size(2) == H && down.size(0) == E && down.size(1) == H && down.size(2) == I, "moe: shapes");
  same_device(x, {&gate_up, &down}, "moe");
}

// gather -> grouped gate/up -> grouped down -> combine over a finished plan.  Returns
// the layer output, or (with residual) updates it in place and returns the fused
// norm's output (undefined without norm_w).
Tensor moe_run_experts(const Tensor& x, MoePlanT& plan, const Tensor& weights, int64_t topk, const Tensor& gate_up,
                       const Tensor& down, int64_t BN, const OptT& add, const OptT& residual, const OptT& norm_w,
                       double eps) {
  const int64_t T = x.size(0), H = x.size(1), P = T * topk;
  same_device_opt(x, {&add, &residual, &norm_w}, "moe");
  for (const OptT* o : {&add, &residual})
    if (has(*o)) TORCH_CHECK((*o)->scalar_type() == torch::kBFloat16 && (*o)->is_contiguous() && (*o)->sizes() == x.sizes(),
                             "moe: add / residual must be bf16 [T, H]");
  if (has(norm_w)) TORCH_CHECK(has(residual) && norm_w->scalar_type() == torch::kBFloat16 && norm_w->numel() == H,
                               "moe: norm_w bf16 [H] with a residual");
  cudaStream_t st = cur_stream();
  // rows past the last block are read by the last block's TMA box (BN rows) and discarded
  auto x_perm = torch::empty({P + BN, H}, x.options());
  vrm::moe_gather(x.data_ptr(), H, plan.tok.data_ptr<int>(), (int)P, (int)H, x_perm.data_ptr(), H, st);
  auto h_perm = moe_grouped_linear(x_perm, gate_up, plan.blocks, plan.nblk, BN, vrm::kEpiSiluMul);
  auto y_perm = moe_grouped_linear(h_perm, down, plan.blocks, plan.nblk, BN, vrm::kEpiNone);
  Tensor out;
  if (!has(residual) || has(norm_w)) out = torch::empty({T, H}, x.options());
  vrm::MoeCombineArgs c;
  c.y_perm = y_perm.data_ptr();
  c.ld_perm = H;
  c.row_of = plan.row_of.data_ptr<int>();
  c.weights = weights.data_ptr<float>();
  c.T = (int)T;
  c.topk = (int)topk;
  c.H = (int)H;
  c.add = has(add) ? add->data_ptr() : nullptr;
  c.residual = has(residual) ? residual->data_ptr() : nullptr;
  c.out = out.defined() ? out.data_ptr() : nullptr;
  c.ldo = H;
  c.norm_w = has(norm_w) ? norm_w->data_ptr() : nullptr;
  c.eps = (float)eps;
  vrm::moe_combine(c, st);
  return out;
}

// Routed experts with explicit routing (ids int64 [T, topk], weights fp32 [T, topk]).
Tensor moe_experts(const Tensor& x, const Tensor& ids, const Tensor& weights, const Tensor& gate_up,
                   const Tensor& down, int64_t BN, const OptT& add) {
  check_moe_weights(x, gate_up, down);
  TORCH_CHECK(ids.scalar_type() == torch::kInt64 && ids.dim() == 2 && ids.is_contiguous() && ids.size(0) == x.size(0),
              "moe: ids int64 [T, topk]");
  TORCH_CHECK(weights.scalar_type() == torch::kFloat32 && weights.sizes() == ids.sizes() && weights.is_contiguous(),
              "moe: weights fp32 [T, topk]");
  same_device(x, {&ids, &weights}, "moe");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t topk = ids.size(1), E = gate_up.size(0), P = x.size(0) * topk;
  auto plan = moe_plan_alloc(x.options(), E, P, BN);
  auto pa = moe_plan_args(plan, P, topk, E, BN);
  pa.ids64 = ids.data_ptr<int64_t>();
  vrm::moe_plan(pa, cur_stream());
  return moe_run_experts(x, plan, weights, topk, gate_up, down, BN, add, c10::nullopt, c10::nullopt, 0.0);
}

// Expert-parallel MoE layer (moe_ep.cu).  `ptrs` (CUDA int64 [5 * world]) holds the
// ranks' cnt, xrecv, meta, yback and flag buffers; `desc` = {rank, world, E, H, p_cap,
// r_rows, cnt_local, xrecv_local, meta_local, yback_local, flags_local}; gate_up / down
// hold this rank's experts [E_local, ...].  Same return convention as moe_layer.
Tensor moe_ep_layer(const Tensor& x, const Tensor& logits, int64_t topk, bool norm_topk, const Tensor& gate_up,
                    const Tensor& down, int64_t BN, const Tensor& ptrs, std::vector<int64_t> desc, const Tensor& epoch,
                    const Tensor& done, const OptT& add, const OptT& residual, const OptT& norm_w, double eps) {
  TORCH_CHECK(desc.size() == 11, "moe_ep: desc has 11 entries");
  check_moe_weights(x, gate_up, down);
  check_bf16_2d(logits, "moe logits");
  same_device(x, {&logits, &ptrs, &epoch, &done}, "moe_ep");
  const int world = (int)desc[1];
  TORCH_CHECK(ptrs.scalar_type() == torch::kInt64 && ptrs.numel() == 5 * world, "moe_ep: ptrs int64 [5 * world]");
  TORCH_CHECK(epoch.scalar_type() == torch::kInt32 && done.scalar_type() == torch::kInt32 && done.numel() >= 2,
              "moe_ep: epoch / done int32");
  const c10::cuda::CUDAGuard guard(x.device());
  vrm::MoeEpBuffers b;
  const int64_t* P64 = ptrs.data_ptr<int64_t>();
  b.cnt = reinterpret_cast<int* const*>(P64);
  b.xrecv = reinterpret_cast<__nv_bfloat16* const*>(P64 + world);
  b.meta = reinterpret_cast<int* const*>(P64 + 2 * world);
  b.yback = reinterpret_cast<__nv_bfloat16* const*>(P64 + 3 * world);
  b.flags = reinterpret_cast<uint32_t* const*>(P64 + 4 * world);
  b.epoch = reinterpret_cast<uint32_t*>(epoch.data_ptr<int>());
  b.done = reinterpret_cast<uint32_t*>(done.data_ptr<int>());
  b.rank = (int)desc[0];
  b.world = world;
  b.E = (int)desc[2];
  b.E_local = b.E / world;
  b.H = (int)desc[3];
  b.p_cap = (int)desc[4];
  b.r_rows = (int)desc[5];
  b.xrecv_local = reinterpret_cast<__nv_bfloat16*>(desc[7]);
  b.meta_local = reinterpret_cast<int*>(desc[8]);
  b.yback_local = reinterpret_cast<__nv_bfloat16*>(desc[9]);
  b.flags_local = reinterpret_cast<uint32_t*>(desc[10]);
  const int64_t T = x.size(0), H = x.size(1), E = b.E, P = T * topk;
  TORCH_CHECK(gate_up.size(0) == b.E_local && logits.size(1) == E && H == b.H && P <= b.p_cap,
              "moe_ep: shapes / capacity (tokens * topk <= p_cap)");
  cudaStream_t st = cur_stream();
  // local routing and plan over all E experts (its counts, offsets and row_of drive the dispatch)
  auto plan = moe_plan_alloc(x.options(), E, P, 128);
  auto ids32 = torch::empty({std::max<int64_t>(P, 1)}, x.options().dtype(torch::kInt32));
  auto w = torch::empty({std::max<int64_t>(P, 1)}, x.options().dtype(torch::kFloat32));
  if (T > 0) {
    vrm::MoeRouteArgs ra;
    ra.logits = logits.data_ptr();
    ra.ldl = logits.stride(0);
    ra.T = (int)T;
    ra.norm_topk = norm_topk;
    ra.ids32 = ids32.data_ptr<int>();
    ra.weights = w.data_ptr<float>();
    ra.plan = moe_plan_args(plan, P, topk, E, 128);
    ra.plan.ids32 = ra.ids32;
    vrm::moe_route(ra, st);
  }
  vrm::moe_ep_counts(b, plan.counts.data_ptr<int>(), (int)T, st);
  vrm::moe_ep_dispatch(b, x.data_ptr(), ids32.data_ptr<int>(), plan.row_of.data_ptr<int>(),
                       plan.offsets.data_ptr<int>(), (int)T, (int)topk, st);
  // owner side: blocks over this rank's experts, rows of every source rank
  const int64_t max_blocks = b.E_local + ((int64_t)world * b.p_cap + BN - 1) / BN;
  auto blocks = torch::empty({max_blocks, 4}, x.options().dtype(torch::kInt32));
  auto nblk = torch::zeros({1}, x.options().dtype(torch::kInt32));
  vrm::moe_ep_owner_plan(b, (int)BN, reinterpret_cast<vrm::MoeBlock*>(blocks.data_ptr<int>()), nblk.data_ptr<int>(),
                         (int)max_blocks, st);
  const int64_t I = gate_up.size(1) / 2;
  auto h = torch::empty({2 * (int64_t)b.r_rows, I}, x.options());
  vrm::MoeGemmArgs g;
  g.w = gate_up.data_ptr();
  g.E = (int)b.E_local;
  g.N = (int)gate_up.size(1);
  g.K = (int)H;
  g.x_perm = b.xrecv_local;
  g.ldx = H;
  g.rows_cap = 2 * b.r_rows;
  g.blocks = blocks.data_ptr<int>();
  g.num_blocks = nblk.data_ptr<int>();
  g.max_blocks = (int)max_blocks;
  g.BN = (int)BN;
  g.out = h.data_ptr();
  g.ldo = I;
  g.epilogue = vrm::kEpiSiluMul;
  vrm::moe_grouped_gemm(g, st);
  g.w = down.data_ptr();
  g.N = (int)H;
  g.K = (int)I;
  g.x_perm = h.data_ptr();
  g.ldx = I;
  g.out = nullptr;
  g.ldo = H;
  g.epilogue = vrm::kEpiNone;
  vrm::moe_ep_grouped_return(b, g, st);
  for (const OptT* o : {&add, &residual})
    if (has(*o)) TORCH_CHECK((*o)->scalar_type() == torch::kBFloat16 && (*o)->is_contiguous() && (*o)->sizes() == x.sizes(),
                             "moe: add / residual must be bf16 [T, H]");
  Tensor out;
  if (!has(residual) || has(norm_w)) out = torch::empty({T, H}, x.options());
  vrm::MoeCombineArgs c;
  c.weights = w.data_ptr<float>();
  c.T = (int)T;
  c.topk = (int)topk;
  c.H = (int)H;
  c.add = has(add) ? add->data_ptr() : nullptr;
  c.residual = has(residual) ? residual->data_ptr() : nullptr;
  c.out = out.defined() ? out.data_ptr() : nullptr;
  c.ldo = H;
  c.norm_w = has(norm_w) ? norm_w->data_ptr() : nullptr;
  c.eps = (float)eps;
  vrm::moe_ep_combine(b, c, st);
  return out;
}

// A whole MoE layer from the router logits (bf16 [T, E]): device routing, plan, experts,
// combine (+ add, + residual in place, + the next RMSNorm when norm_w is given).
Tensor moe_layer(const Tensor& x, const Tensor& logits, int64_t topk, bool norm_topk, const Tensor& gate_up,
                 const Tensor& down, int64_t BN, const OptT& add, const OptT& residual, const OptT& norm_w,
                 double eps) {
  check_moe_weights(x, gate_up, down);
  check_bf16_2d(logits, "moe logits");
  TORCH_CHECK(logits.size(0) == x.size(0) && logits.size(1) == gate_up.size(0), "moe: logits [T, E]");
  same_device(x, {&logits}, "moe");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t T = x.size(0), E = gate_up.size(0), P = T * topk;
  auto plan = moe_plan_alloc(x.options(), E, P, BN);
  auto ids32 = torch::empty({std::max<int64_t>(P, 1)}, x.options().dtype(torch::kInt32));
  auto w = torch::empty({std::max<int64_t>(P, 1)}, x.options().dtype(torch::kFloat32));
  vrm::MoeRouteArgs ra;
  ra.logits = logits.data_ptr();
  ra.ldl = logits.stride(0);
  ra.T = (int)T;
  ra.norm_topk = norm_topk;
  ra.ids32 = ids32.data_ptr<int>();
  ra.weights = w.data_ptr<float>();
  ra.plan = moe_plan_args(plan, P, topk, E, BN);
  ra.plan.ids32 = ra.ids32;
  vrm::moe_route(ra, cur_stream());
  return moe_run_experts(x, plan, w, topk, gate_up, down, BN, add, residual, norm_w, eps);
}

// ---------------------------------------------------------------- page migration
void page_copy(const Tensor& src_pool, Tensor& dst_pool, const Tensor& src_idx, const Tensor& dst_idx) {
  TORCH_CHECK(src_pool.is_cuda() && dst_pool.is_cuda() && src_pool.is_contiguous() && dst_pool.is_contiguous(),
              "page_copy: contiguous CUDA pools");
  TORCH_CHECK(src_pool.dim() >= 1 && dst_pool.dim() >= 1 && src_pool.nbytes() / src_pool.size(0) ==
                  dst_pool.nbytes() / dst_pool.size(0), "page_copy: pools must have the same page size");
  TORCH_CHECK(src_idx.scalar_type() == torch::kInt32 && dst_idx.scalar_type() == torch::kInt32 &&
                  src_idx.numel() == dst_idx.numel() && src_idx.device() == src_pool.device() &&
                  dst_idx.device() == src_pool.device(),
              "page_copy: int32 index tensors on the source device");
  const size_t page_bytes = src_pool.nbytes() / src_pool.size(0);
  const c10::cuda::CUDAGuard guard(src_pool.device());
  if (src_pool.device() != dst_pool.device()) {
    TORCH_CHECK(vrm::enable_peer_access(src_pool.device().index(), dst_pool.device().index()),
                "page_copy: no peer access between the two GPUs");
  }
  vrm::page_copy(src_pool.data_ptr(), dst_pool.data_ptr(), src_idx.data_ptr<int>(), dst_idx.data_ptr<int>(),
                 (int)src_idx.numel(), page_bytes, cur_stream(), src_pool.size(0), dst_pool.size(0));
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "vramancer_b200 sm_100a kernels";
  m.attr("EPI_NONE") = (int)vrm::kEpiNone;
  m.attr("EPI_SILU_MUL") = (int)vrm::kEpiSiluMul;
  m.def("gemm", &gemm, py::arg("x"), py::arg("w"), py::arg("bias") = py::none(), py::arg("force_splits") = 0,
        py::arg("epilogue") = 0);
  m.def("gemm_out", &gemm_out, py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("out"),
        py::arg("force_splits") = 0, py::arg("epilogue") = 0, py::arg("residual") = py::none(),
        py::arg("ssq_out") = py::none(), py::arg("ssq_in") = py::none(), py::arg("ssq_parts") = 0,
        py::arg("norm_eps") = 0.0);
  m.def("rmsnorm", &rmsnorm, py::arg("x"), py::arg("residual"), py::arg("w"), py::arg("out"), py::arg("eps"));
  m.def("layernorm", &layernorm, py::arg("x"), py::arg("residual"), py::arg("w"), py::arg("b"), py::arg("out"),
        py::arg("eps"));
  m.def("qk_rmsnorm", &qk_rmsnorm, py::arg("qkv"), py::arg("wq"), py::arg("wk"), py::arg("num_q_heads"),
        py::arg("num_kv_heads"), py::arg("head_dim"), py::arg("eps"));
  m.def("rope_kv_write", &rope_kv_write, py::arg("qkv"), py::arg("positions"), py::arg("cos_sin"), py::arg("cache"),
        py::arg("slot_mapping"), py::arg("kv_scale"), py::arg("layer"), py::arg("num_q_heads"),
        py::arg("num_kv_heads"), py::arg("head_dim"));
  m.def("silu_mul", &silu_mul, py::arg("x"), py::arg("out"));
  m.def("gelu_tanh_", &gelu_tanh_, py::arg("x"));
  m.def("embedding", &embedding, py::arg("ids"), py::arg("table"), py::arg("pos"), py::arg("pos_table"),
        py::arg("out"));
  m.def("add_", &add_, py::arg("a"), py::arg("b"));
  m.def("paged_attention_decode", &attn_decode, py::arg("q"), py::arg("cache"), py::arg("layer"),
        py::arg("block_tables"), py::arg("context_lens"), py::arg("kv_scale"), py::arg("sm_scale"), py::arg("out"),
        py::arg("num_splits"), py::arg("num_q_heads"), py::arg("positions") = py::none(),
        py::arg("cos_sin") = py::none(), py::arg("slot_mapping") = py::none(),
        py::arg("l2_prefetch") = py::none());
  m.def("paged_attention_prefill", &attn_prefill, py::arg("q"), py::arg("cache"), py::arg("layer"),
        py::arg("block_tables"), py::arg("cu_q"), py::arg("context_lens"), py::arg("kv_scale"), py::arg("sm_scale"),
        py::arg("out"), py::arg("max_q_len"), py::arg("num_q_heads"));
  m.def("decode_attention_splits", [](int64_t B, int64_t KH, int64_t max_pages) {
    return vrm::decode_attention_choose_splits((int)B, (int)KH, (int)max_pages);
  });
  m.def("argmax", &argmax, py::arg("logits"), py::arg("out"));
  m.def("sample_vp_local", &sample_vp_local, py::arg("logits"), py::arg("v_off"), py::arg("vocab"),
        py::arg("temperature"), py::arg("top_k"), py::arg("top_p"), py::arg("seed"), py::arg("steps"),
        py::arg("kmax"), py::arg("cand"));
  m.def("sample_vp_combine", &sample_vp_combine, py::arg("gathered"), py::arg("vocab"), py::arg("temperature"),
        py::arg("top_k"), py::arg("top_p"), py::arg("seed"), py::arg("steps"), py::arg("kmax"), py::arg("out"));
  m.def("sample", &sample, py::arg("logits"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"),
        py::arg("seed"), py::arg("steps"), py::arg("out"));
  m.def("set_prefill_tc", [](bool on) { vrm::set_prefill_tc(on); });
  m.def("gemm_set_prefill_mode", [](int64_t mode) { vrm::gemm_set_prefill_mode((int)mode); });
  m.def("gemm_set_trace", [](c10::optional<Tensor> buf) {
    vrm::gemm_set_trace(buf.has_value() && buf->defined() ? buf->data_ptr() : nullptr);
  });
  m.def("nvfp4_quantize", &nvfp4_quantize, py::arg("w"), py::arg("gs"),
        "bf16 [N, K] -> (q, s) NVFP4 bytes in fragment order, per-tensor scale gs on the device");
  m.def("nvfp4_dequantize", &nvfp4_dequantize, py::arg("q"), py::arg("s"), py::arg("gs"), py::arg("N"), py::arg("K"));
  m.def("nvfp4_tc_gemm_out", &nvfp4_tc_gemm_out, py::arg("x"), py::arg("q_rows"), py::arg("sf"), py::arg("gs"),
        py::arg("bias"), py::arg("out"), py::arg("epilogue"), py::arg("residual"));
  m.def("nvfp4_gemm_out", &nvfp4_gemm_out, py::arg("x"), py::arg("q"), py::arg("s"), py::arg("gs"), py::arg("N"),
        py::arg("bias"), py::arg("out"), py::arg("epilogue"), py::arg("residual"),
        "W4A16 decode GEMM (M <= 32) over NVFP4 weights");
  m.def("nvfp4_gemm_ar_push", &nvfp4_gemm_ar_push, py::arg("x"), py::arg("q"), py::arg("s"), py::arg("gs"),
        py::arg("N"), py::arg("xbuf_ptrs"), py::arg("epoch"), py::arg("rank"), py::arg("world"),
        py::arg("half_floats"), "W4A16 decode GEMM pushing its partial into every rank's receive buffer");
  m.def("nvfp4_gemm_max_m", &vrm::nvfp4_gemm_max_m);
  m.def("tq_compress", &tq_compress, py::arg("x"), py::arg("signs"), py::arg("jl"),
        "TurboQuant: [..., 128] -> 64-byte records (Hadamard + PolarQuant + QJL)");
  m.def("tq_kv_write", &tq_kv_write, py::arg("qkv"), py::arg("slot_mapping"), py::arg("pool"), py::arg("layer"),
        py::arg("num_q_heads"), py::arg("num_kv_heads"), py::arg("signs"), py::arg("jl"));
  m.def("tq_paged_decode", &tq_paged_decode, py::arg("q"), py::arg("pool"), py::arg("layer"),
        py::arg("block_tables"), py::arg("context_lens"), py::arg("signs"), py::arg("jl"), py::arg("sm_scale"),
        py::arg("out"), py::arg("num_q_heads"));
  m.def("tq_decompress", &tq_decompress, py::arg("rec"), py::arg("signs"),
        "TurboQuant: 64-byte records -> bf16 [..., 128]");
  m.def("set_decode_tma", &vrm::set_decode_tma, py::arg("on"),
        "use the persistent TMA decode-attention kernel for bf16 pages (default off)");
  m.def("fp8_rows_quantize", &fp8_rows_quantize, py::arg("x"), "e4m3 rows with per-row scales");
  m.def("gemm_fp8_out", &gemm_fp8_out, py::arg("xq"), py::arg("sx"), py::arg("wq"), py::arg("sw"), py::arg("bias"),
        py::arg("out"), py::arg("epilogue"), py::arg("residual"),
        "FP8 W8A8 GEMM (stream-K tcgen05 kind::f8f6f4, per-token x per-channel scales)");
  m.def("nvfp4_rows_quantize", &nvfp4_rows_quantize, py::arg("x"), py::arg("rows"), py::arg("gs_tensor"),
        "NVFP4 rows for the block-scaled GEMM: codes, 128x4 scale atoms, per-row scales");
  m.def("nvfp4_bs_gemm", &nvfp4_bs_gemm, py::arg("qa"), py::arg("sfa"), py::arg("gsa"), py::arg("M"), py::arg("qb"),
        py::arg("sfb"), py::arg("gsb"), py::arg("bias") = py::none(), py::arg("residual") = py::none(),
        py::arg("epilogue") = 0, py::arg("out") = py::none(),
        "NVFP4 x NVFP4 GEMM on tcgen05 kind::mxf4nvf4 (bf16 out, bias / residual / silu_mul epilogue)");
  m.def("moe_route", &moe_route_op, py::arg("logits"), py::arg("topk"), py::arg("norm_topk"), py::arg("BN"),
        "MoE router on the device: ids, weights, counts, offsets, row_of, tok_of_row, blocks, num_blocks");
  m.def("moe_layer", &moe_layer, py::arg("x"), py::arg("logits"), py::arg("topk"), py::arg("norm_topk"),
        py::arg("gate_up"), py::arg("down"), py::arg("BN"), py::arg("add"), py::arg("residual"), py::arg("norm_w"),
        py::arg("eps"), "MoE layer from router logits (device routing, grouped GEMMs, fused combine)");
  m.def("moe_ep_layer", &moe_ep_layer, py::arg("x"), py::arg("logits"), py::arg("topk"), py::arg("norm_topk"),
        py::arg("gate_up"), py::arg("down"), py::arg("BN"), py::arg("ptrs"), py::arg("desc"), py::arg("epoch"),
        py::arg("done"), py::arg("add"), py::arg("residual"), py::arg("norm_w"), py::arg("eps"),
        "expert-parallel MoE layer: peer-memory dispatch, grouped GEMMs with the return fused into the epilogue");
  m.def("moe_plan", &moe_plan_op, py::arg("ids"), py::arg("E"), py::arg("BN"),
        "MoE expert plan: counts, offsets, row_of, tok_of_row, blocks [max_blocks, 4], num_blocks");
  m.def("moe_grouped_linear", &moe_grouped_linear, py::arg("x_perm"), py::arg("w"), py::arg("blocks"),
        py::arg("num_blocks"), py::arg("BN"), py::arg("epilogue"), "grouped expert GEMM over a MoE plan");
  m.def("moe_experts", &moe_experts, py::arg("x"), py::arg("ids"), py::arg("weights"), py::arg("gate_up"),
        py::arg("down"), py::arg("BN"), py::arg("add"),
        "routed experts of a MoE layer on the device (plan, gather, grouped tcgen05 GEMMs, combine)");
  m.def("gemm_ar_push", &gemm_ar_push, py::arg("x"), py::arg("w"), py::arg("xbuf_ptrs"), py::arg("epoch"),
        py::arg("rank"), py::arg("world"), py::arg("half_floats"), py::arg("scale_x") = py::none(),
        py::arg("scale_w") = py::none(), py::arg("residual") = py::none(), py::arg("bias") = py::none(),
        py::arg("ssq_out") = py::none(), py::arg("done") = py::none(), py::arg("spin_limit") = 0,
        "row-parallel GEMM storing its partial into every rank's receive buffer (fused all-reduce, push); with "
        "residual, the same kernel also reduces into the residual stream and stores the RMSNorm sums");
  m.def("ar_norm", &ar_norm, py::arg("xbuf"), py::arg("epoch"), py::arg("done"), py::arg("rank"), py::arg("world"),
        py::arg("half_floats"), py::arg("T"), py::arg("H"), py::arg("bias"), py::arg("residual"), py::arg("w"),
        py::arg("b"), py::arg("out"), py::arg("mode"), py::arg("eps"), py::arg("spin_limit") = 0,
        py::arg("err") = py::none(),
        "fused all-reduce, reduce half: poll the slots, sum in rank order, + bias + residual, optional norm");
  m.def("vmm_granularity", [](int64_t device) { return (int64_t)vrm::vmm_granularity((int)device); });
  m.def("vmm_reserve", [](int64_t bytes, int64_t align) { return (int64_t)vrm::vmm_reserve(bytes, align); });
  m.def("vmm_map", [](int64_t base, int64_t offset, int64_t bytes, int64_t location, std::vector<int64_t> access,
                      bool shareable) {
    std::vector<int> acc(access.begin(), access.end());
    vrm::vmm_map((uint64_t)base, offset, bytes, (int)location, acc, shareable);
  });
  m.def("vmm_export_fd", [](int64_t base, int64_t offset) { return vrm::vmm_export_fd((uint64_t)base, offset); });
  m.def("vmm_map_fd", [](int64_t base, int64_t offset, int64_t bytes, int64_t fd, std::vector<int64_t> access) {
    std::vector<int> acc(access.begin(), access.end());
    vrm::vmm_map_fd((uint64_t)base, offset, bytes, (int)fd, acc);
  });
  m.def("vmm_unmap", [](int64_t base, int64_t offset) { vrm::vmm_unmap((uint64_t)base, offset); });
  m.def("vmm_free", [](int64_t base) { vrm::vmm_free((uint64_t)base); });
  m.def("tensor_from_ptr", [](int64_t ptr, std::vector<int64_t> shape, std::string dtype, int64_t device) {
    // a tensor view of device memory this library manages (no ownership: the caller
    // keeps the region alive for the tensor's lifetime)
    at::ScalarType st;
    if (dtype == "bfloat16") st = torch::kBFloat16;
    else if (dtype == "float8_e4m3fn") st = torch::kFloat8_e4m3fn;
    else if (dtype == "float32") st = torch::kFloat32;
    else if (dtype == "uint8") st = torch::kByte;
    else if (dtype == "float16") st = torch::kHalf;
    else TORCH_CHECK(false, "tensor_from_ptr: unsupported dtype ", dtype);
    auto opts = torch::TensorOptions().dtype(st).device(torch::kCUDA, (int)device);
    return torch::from_blob(reinterpret_cast<void*>(ptr), shape, opts);
  });
  m.def("symm_fill_u16", [](int64_t p, int64_t count, int64_t value) {
    vrm::symm_fill_u16(reinterpret_cast<void*>(p), (size_t)count, (uint16_t)value);
  });
  m.def("symm_malloc", [](int64_t bytes) { return (int64_t)reinterpret_cast<uintptr_t>(vrm::symm_malloc(bytes)); });
  m.def("symm_free", [](int64_t p) { vrm::symm_free(reinterpret_cast<void*>(p)); });
  m.def("ipc_handle", [](int64_t p) {
    auto v = vrm::ipc_handle(reinterpret_cast<void*>(p));
    return py::bytes(reinterpret_cast<const char*>(v.data()), v.size());
  });
  m.def("ipc_open", [](py::bytes b) {
    std::string s = b;
    std::vector<uint8_t> v(s.begin(), s.end());
    return (int64_t)reinterpret_cast<uintptr_t>(vrm::ipc_open(v));
  });
  m.def("ipc_close", [](int64_t p) { vrm::ipc_close(reinterpret_cast<void*>(p)); });
  m.def("page_copy", &page_copy, py::arg("src_pool"), py::arg("dst_pool"), py::arg("src_idx"), py::arg("dst_idx"),
        "copy whole KV pages between pools (peer GPU allowed), runs on the source device");
  m.def("enable_peer_access", &vrm::enable_peer_access, py::arg("device"), py::arg("peer"));
  m.def("read_and_clear_errors", &vrm::read_and_clear_errors, "device error word (bounded-wait timeouts)");
  m.def("reserve_workspace", [](int64_t bytes) { vrm::workspace_reserve((size_t)bytes, cur_stream()); },
        "pre-allocate split-K / split-KV scratch before CUDA graph capture");
  m.def("workspace_size", []() { return (int64_t)vrm::workspace_size(); });
}
