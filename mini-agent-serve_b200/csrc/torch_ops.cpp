// torch_ops.cpp -- the `mas_b200::*` PyTorch operators, implemented in C++ over the C ABI.
//
// Each operator unpacks its tensors into the plain pointers, sizes and strides of the matching
// include/mas_b200.h entry point and launches on the tensor's device and current stream. Doing this in
// C++ keeps a call at dispatcher cost (a few microseconds): the serving loop issues several of these
// ops per layer, and a Python-level operator body would make short steps CPU-bound. The fake (meta)
// kernels that torch.compile traces with are registered from Python (ops.py); the argument checks
// that must raise flashinfer's Python exception types stay in the Python wrappers, and the checks
// here are the last line (TORCH_CHECK -> RuntimeError).
#include <ATen/ATen.h>
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/library.h>

#include "../../include/mas_b200.h"

namespace {

int act_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kBFloat16) return MAS_DTYPE_BF16;
  if (t.scalar_type() == at::kHalf) return MAS_DTYPE_FP16;
  TORCH_CHECK(false, "mas_b200: unsupported dtype ", t.scalar_type(), "; expected bfloat16 or float16");
}

int id_code(const at::Tensor& t) {
  if (t.scalar_type() == at::kInt) return MAS_DTYPE_INT32;
  if (t.scalar_type() == at::kLong) return MAS_DTYPE_INT64;
  TORCH_CHECK(false, "mas_b200: indices must be int32 or int64, got ", t.scalar_type());
}

void check(int rc, const char* fn) {
  TORCH_CHECK(rc == MAS_OK, fn, " failed with status ", rc, ": ", mas_status_string(rc));
}

// [rows, cols] view of a tensor whose last dimension is contiguous and whose leading dimensions
// collapse into one: returns (rows, row stride in elements).
struct Rows {
  int64_t rows;
  int64_t cols;
  int64_t stride;
};

Rows rows_of(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.dim() >= 1, "mas_b200: ", name, " must have at least one dimension");
  const int64_t cols = t.size(-1);
  TORCH_CHECK(t.stride(-1) == 1 || cols <= 1, "mas_b200: ", name, " must be contiguous in its last dimension");
  if (t.dim() == 1) return {1, cols, cols};
  int64_t rows = 1;
  for (int64_t d = 0; d < t.dim() - 1; ++d) rows *= t.size(d);
  const int64_t stride = t.stride(-2);
  for (int64_t d = 0; d + 2 < t.dim(); ++d) {
    TORCH_CHECK(t.size(d + 1) == 1 || t.stride(d) == t.stride(d + 1) * t.size(d + 1),
                "mas_b200: ", name, "'s leading dimensions must be collapsible into one");
  }
  return {rows, cols, rows > 1 ? stride : cols};
}

void* stream_of(const at::Tensor& t) {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream(t.device().index()).stream());
}

// The weight is read as `cols` contiguous elements of the activation dtype.
void check_norm_operands(const at::Tensor& input, const at::Tensor& residual, const at::Tensor& weight,
                         int64_t cols) {
  TORCH_CHECK(residual.scalar_type() == input.scalar_type() && weight.scalar_type() == input.scalar_type(),
              "mas_b200: input, residual and weight must share one dtype");
  TORCH_CHECK(weight.dim() == 1 && weight.numel() == cols && weight.is_contiguous(),
              "mas_b200: weight must be a contiguous (hidden_size,) vector");
}

void fused_add_rmsnorm(at::Tensor input, at::Tensor residual, at::Tensor weight, double eps, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(input.device());
  const Rows x = rows_of(input, "input"), r = rows_of(residual, "residual");
  TORCH_CHECK(x.rows == r.rows && x.cols == r.cols, "mas_b200: input and residual shapes differ");
  check_norm_operands(input, residual, weight, x.cols);
  check(mas_fused_add_rmsnorm(input.data_ptr(), residual.data_ptr(), weight.data_ptr(), x.rows, x.cols, x.stride,
                              r.stride, static_cast<float>(eps), act_code(input), enable_pdl, stream_of(input)),
        "mas_fused_add_rmsnorm");
}

void fused_add_rmsnorm_quant(at::Tensor out, at::Tensor input, at::Tensor residual, at::Tensor weight,
                             at::Tensor scale, double eps, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(input.device());
  const Rows o = rows_of(out, "out"), x = rows_of(input, "input"), r = rows_of(residual, "residual");
  TORCH_CHECK(o.rows == x.rows && x.rows == r.rows && o.cols == x.cols && x.cols == r.cols,
              "mas_b200: out, input and residual shapes differ");
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn, "mas_b200: out must be float8_e4m3fn");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() == 1, "mas_b200: scale must be one fp32 value");
  check_norm_operands(input, residual, weight, x.cols);
  check(mas_fused_add_rmsnorm_quant(out.data_ptr(), input.data_ptr(), residual.data_ptr(), weight.data_ptr(),
                                    scale.data_ptr<float>(), x.rows, x.cols, o.stride, x.stride, r.stride,
                                    static_cast<float>(eps), act_code(input), MAS_DTYPE_FP8_E4M3, enable_pdl,
                                    stream_of(input)),
        "mas_fused_add_rmsnorm_quant");
}

void silu_and_mul(at::Tensor out, at::Tensor input, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(input.device());
  const Rows o = rows_of(out, "out"), x = rows_of(input, "input");
  TORCH_CHECK(o.rows == x.rows && x.cols == 2 * o.cols, "mas_b200: out must be input[..., :d]-shaped");
  check(mas_silu_and_mul(out.data_ptr(), input.data_ptr(), x.rows, o.cols, o.stride, x.stride, act_code(input),
                         enable_pdl, stream_of(input)),
        "mas_silu_and_mul");
}

void silu_and_mul_quant(at::Tensor out, at::Tensor input, at::Tensor scale, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(input.device());
  const Rows o = rows_of(out, "out"), x = rows_of(input, "input");
  TORCH_CHECK(o.rows == x.rows && x.cols == 2 * o.cols, "mas_b200: out must be input[..., :d]-shaped");
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn, "mas_b200: out must be float8_e4m3fn");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() == 1, "mas_b200: scale must be one fp32 value");
  check(mas_silu_and_mul_quant(out.data_ptr(), input.data_ptr(), scale.data_ptr<float>(), x.rows, o.cols, o.stride,
                               x.stride, act_code(input), MAS_DTYPE_FP8_E4M3, enable_pdl, stream_of(input)),
        "mas_silu_and_mul_quant");
}

// q and k as (tokens, heads, head_size) views, contiguous within a head; one contiguous position per
// token; an fp32 cache. The kernels read positions[0 .. tokens) with unit stride.
void check_rope_operands(const at::Tensor& q, const at::Tensor& k, const at::Tensor& cos_sin_cache,
                         const at::Tensor& pos_ids) {
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3, "mas_b200: q and k must be (tokens, heads, head_size) views");
  TORCH_CHECK(q.size(0) == k.size(0) && q.size(2) == k.size(2), "mas_b200: q and k token counts or head sizes differ");
  TORCH_CHECK(q.stride(2) == 1 && k.stride(2) == 1, "mas_b200: q and k must be contiguous within a head");
  TORCH_CHECK(q.scalar_type() == k.scalar_type(), "mas_b200: q and k must share one dtype");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous() && cos_sin_cache.scalar_type() == at::kFloat,
              "mas_b200: cos_sin_cache must be a contiguous fp32 (max_positions, rotary_dim) tensor");
  TORCH_CHECK(pos_ids.is_contiguous() && pos_ids.numel() == q.size(0),
              "mas_b200: positions must be contiguous with one entry per token");
}

void apply_rope_pos_ids_cos_sin_cache(at::Tensor q, at::Tensor k, at::Tensor cos_sin_cache, at::Tensor pos_ids,
                                      bool interleave, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(q.device());
  check_rope_operands(q, k, cos_sin_cache, pos_ids);
  check(mas_rope_cos_sin_cache_inplace(pos_ids.data_ptr(), id_code(pos_ids), q.data_ptr(), k.data_ptr(),
                                       cos_sin_cache.data_ptr<float>(), q.size(0), q.size(1), k.size(1), q.size(2),
                                       cos_sin_cache.size(1), cos_sin_cache.size(0), q.stride(0), q.stride(1),
                                       k.stride(0), k.stride(1), interleave ? 0 : 1, act_code(q), nullptr, enable_pdl,
                                       stream_of(q)),
        "mas_rope_cos_sin_cache_inplace");
}

void apply_rope_q_scale(at::Tensor q, at::Tensor k, at::Tensor cos_sin_cache, at::Tensor pos_ids, bool interleave,
                        double beta, int64_t original_max, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(q.device());
  check_rope_operands(q, k, cos_sin_cache, pos_ids);
  check(mas_rope_cos_sin_cache_q_scale_inplace(
            pos_ids.data_ptr(), id_code(pos_ids), q.data_ptr(), k.data_ptr(), cos_sin_cache.data_ptr<float>(),
            q.size(0), q.size(1), k.size(1), q.size(2), cos_sin_cache.size(1), cos_sin_cache.size(0), q.stride(0),
            q.stride(1), k.stride(0), k.stride(1), interleave ? 0 : 1, static_cast<float>(beta), original_max,
            act_code(q), nullptr, enable_pdl, stream_of(q)),
        "mas_rope_cos_sin_cache_q_scale_inplace");
}

// One layer's paged cache as the C ABI describes it: 4-D k/v caches with identical strides, NHD
// ([pages, page_size, heads, head_size]) or HND ([pages, heads, page_size, head_size]).
MasPagedKVCache paged_cache(const at::Tensor& k_cache, const at::Tensor& v_cache, const at::Tensor& kv_indices,
                            const at::Tensor& kv_indptr, bool hnd) {
  TORCH_CHECK(k_cache.dim() == 4 && v_cache.dim() == 4, "mas_b200: k_cache and v_cache must be 4-D");
  TORCH_CHECK(k_cache.sizes() == v_cache.sizes() && k_cache.strides() == v_cache.strides(),
              "mas_b200: k/v cache shapes and strides must be identical");
  TORCH_CHECK(k_cache.stride(3) == 1, "mas_b200: the cache's last dimension must be contiguous");
  TORCH_CHECK(kv_indices.scalar_type() == at::kInt && kv_indptr.scalar_type() == at::kInt &&
                  kv_indices.is_contiguous() && kv_indptr.is_contiguous() && kv_indptr.dim() == 1 &&
                  kv_indptr.numel() >= 1,
              "mas_b200: kv_indices and kv_indptr must be contiguous int32 vectors");
  MasPagedKVCache c = {};
  c.k_cache = k_cache.data_ptr();
  c.v_cache = v_cache.data_ptr();
  c.num_pages = k_cache.size(0);
  c.page_size = hnd ? k_cache.size(2) : k_cache.size(1);
  c.stride_page = k_cache.stride(0);
  c.stride_entry = hnd ? k_cache.stride(2) : k_cache.stride(1);
  c.stride_head = hnd ? k_cache.stride(1) : k_cache.stride(2);
  c.kv_indices = kv_indices.data_ptr<int32_t>();
  c.num_indices = kv_indices.numel();
  c.kv_indptr = kv_indptr.data_ptr<int32_t>();
  c.batch_size = kv_indptr.numel() - 1;
  return c;
}

void append_paged_kv_cache(at::Tensor k, at::Tensor v, at::Tensor batch_indices, at::Tensor positions,
                           at::Tensor k_cache, at::Tensor v_cache, at::Tensor kv_indices, at::Tensor kv_indptr,
                           bool hnd, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(k.device());
  TORCH_CHECK(k.dim() == 3 && v.dim() == 3 && k.sizes() == v.sizes(), "mas_b200: k and v must be (tokens, heads, head_size)");
  TORCH_CHECK(k.stride(2) == 1 && v.stride(2) == 1, "mas_b200: k and v must be contiguous in head_size");
  TORCH_CHECK(batch_indices.scalar_type() == at::kInt && batch_indices.is_contiguous() &&
                  batch_indices.numel() == k.size(0) && positions.is_contiguous() && positions.numel() == k.size(0),
              "mas_b200: batch_indices (int32) and positions must be contiguous, one per token");
  TORCH_CHECK(k_cache.scalar_type() == k.scalar_type() && v.scalar_type() == k.scalar_type(),
              "mas_b200: k, v and the caches must share one dtype");
  const MasPagedKVCache c = paged_cache(k_cache, v_cache, kv_indices, kv_indptr, hnd);
  TORCH_CHECK((hnd ? k_cache.size(1) : k_cache.size(2)) == k.size(1) && k_cache.size(3) == k.size(2),
              "mas_b200: the cache's heads/head_size differ from k's");
  check(mas_append_paged_kv_cache(k.data_ptr(), v.data_ptr(), batch_indices.data_ptr<int32_t>(), positions.data_ptr(),
                                  id_code(positions), &c, k.size(0), k.size(1), k.size(2), k.stride(0), k.stride(1),
                                  v.stride(0), v.stride(1), act_code(k), nullptr, enable_pdl, stream_of(k)),
        "mas_append_paged_kv_cache");
}

void rope_append_paged_kv_cache(at::Tensor q, at::Tensor k, at::Tensor v, at::Tensor cos_sin_cache,
                                at::Tensor pos_ids, at::Tensor batch_indices, at::Tensor k_cache, at::Tensor v_cache,
                                at::Tensor kv_indices, at::Tensor kv_indptr, bool interleave, bool hnd, double beta,
                                int64_t original_max, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(q.device());
  TORCH_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "mas_b200: q, k and v must be (tokens, heads, head_size) views");
  TORCH_CHECK(k.sizes() == v.sizes() && q.size(2) == k.size(2) && q.size(0) == k.size(0),
              "mas_b200: q, k and v shapes disagree");
  TORCH_CHECK(cos_sin_cache.dim() == 2 && cos_sin_cache.is_contiguous(), "mas_b200: cos_sin_cache must be contiguous");
  TORCH_CHECK(batch_indices.scalar_type() == at::kInt && batch_indices.is_contiguous() &&
                  batch_indices.numel() == q.size(0) && pos_ids.is_contiguous() && pos_ids.numel() == q.size(0),
              "mas_b200: batch_indices (int32) and positions must be contiguous, one per token");
  TORCH_CHECK(k_cache.scalar_type() == k.scalar_type() && v.scalar_type() == k.scalar_type() &&
                  q.scalar_type() == k.scalar_type(),
              "mas_b200: q, k, v and the caches must share one dtype");
  const MasPagedKVCache c = paged_cache(k_cache, v_cache, kv_indices, kv_indptr, hnd);
  TORCH_CHECK((hnd ? k_cache.size(1) : k_cache.size(2)) == k.size(1) && k_cache.size(3) == k.size(2),
              "mas_b200: the cache's heads/head_size differ from k's");
  check(mas_rope_append_paged_kv_cache(
            pos_ids.data_ptr(), id_code(pos_ids), q.data_ptr(), k.data_ptr(), v.data_ptr(),
            cos_sin_cache.data_ptr<float>(), batch_indices.data_ptr<int32_t>(), &c, q.size(0), q.size(1), k.size(1),
            q.size(2), cos_sin_cache.size(1), cos_sin_cache.size(0), q.stride(0), q.stride(1), k.stride(0), k.stride(1),
            v.stride(0), v.stride(1), interleave ? 0 : 1, static_cast<float>(beta), original_max, act_code(q), nullptr,
            enable_pdl, stream_of(q)),
        "mas_rope_append_paged_kv_cache");
}

void gather(at::Tensor& out, const at::Tensor& ids, const at::Tensor& weight, bool enable_pdl) {
  TORCH_CHECK(weight.dim() == 2 && weight.stride(1) == 1, "mas_b200: weight must be (num_embeddings, dim)");
  TORCH_CHECK(ids.is_contiguous(), "mas_b200: input_ids must be contiguous");
  TORCH_CHECK(out.is_contiguous(), "mas_b200: out must be contiguous");
  check(mas_embedding_gather(out.data_ptr(), weight.data_ptr(), ids.data_ptr(), id_code(ids), ids.numel(),
                             weight.size(1), weight.size(0), weight.size(1), weight.stride(0),
                             static_cast<int>(weight.element_size()), nullptr, enable_pdl, stream_of(weight)),
        "mas_embedding_gather");
}

at::Tensor embedding(at::Tensor input_ids, at::Tensor weight, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(weight.device());
  std::vector<int64_t> shape(input_ids.sizes().begin(), input_ids.sizes().end());
  shape.push_back(weight.size(1));
  at::Tensor out = at::empty(shape, weight.options());
  gather(out, input_ids.contiguous(), weight, enable_pdl);
  return out;
}

at::Tensor embedding_fill(at::Tensor input_ids, at::Tensor weight, at::Tensor last_tokens, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(weight.device());
  TORCH_CHECK(weight.dim() == 2 && weight.stride(1) == 1, "mas_b200: weight must be (num_embeddings, dim)");
  TORCH_CHECK(input_ids.is_contiguous(), "mas_b200: input_ids must be contiguous (it is updated in place)");
  TORCH_CHECK(last_tokens.is_contiguous(), "mas_b200: last_tokens must be contiguous");
  std::vector<int64_t> shape(input_ids.sizes().begin(), input_ids.sizes().end());
  shape.push_back(weight.size(1));
  at::Tensor out = at::empty(shape, weight.options());
  check(mas_embedding_gather_fill_placeholders(
            out.data_ptr(), weight.data_ptr(), input_ids.data_ptr(), id_code(input_ids), last_tokens.data_ptr(),
            id_code(last_tokens), last_tokens.numel(), input_ids.numel(), weight.size(1), weight.size(0),
            weight.size(1), weight.stride(0), static_cast<int>(weight.element_size()), nullptr, enable_pdl,
            stream_of(weight)),
        "mas_embedding_gather_fill_placeholders");
  return out;
}

void embedding_out(at::Tensor out, at::Tensor input_ids, at::Tensor weight, bool enable_pdl) {
  const c10::cuda::CUDAGuard guard(weight.device());
  gather(out, input_ids, weight, enable_pdl);
}

}  // namespace

TORCH_LIBRARY(mas_b200, m) {
  m.def("fused_add_rmsnorm(Tensor(a!) input, Tensor(b!) residual, Tensor weight, float eps, bool enable_pdl) -> ()");
  m.def("fused_add_rmsnorm_quant(Tensor(a!) out, Tensor input, Tensor(b!) residual, Tensor weight, Tensor scale, "
        "float eps, bool enable_pdl) -> ()");
  m.def("silu_and_mul(Tensor(a!) out, Tensor input, bool enable_pdl) -> ()");
  m.def("silu_and_mul_quant(Tensor(a!) out, Tensor input, Tensor scale, bool enable_pdl) -> ()");
  m.def("apply_rope_pos_ids_cos_sin_cache(Tensor(a!) q, Tensor(b!) k, Tensor cos_sin_cache, Tensor pos_ids, "
        "bool interleave, bool enable_pdl) -> ()");
  m.def("apply_rope_q_scale(Tensor(a!) q, Tensor(b!) k, Tensor cos_sin_cache, Tensor pos_ids, bool interleave, "
        "float beta, int original_max, bool enable_pdl) -> ()");
  m.def("append_paged_kv_cache(Tensor k, Tensor v, Tensor batch_indices, Tensor positions, Tensor(a!) k_cache, "
        "Tensor(b!) v_cache, Tensor kv_indices, Tensor kv_indptr, bool hnd, bool enable_pdl) -> ()");
  m.def("rope_append_paged_kv_cache(Tensor(a!) q, Tensor(b!) k, Tensor v, Tensor cos_sin_cache, Tensor pos_ids, "
        "Tensor batch_indices, Tensor(c!) k_cache, Tensor(d!) v_cache, Tensor kv_indices, Tensor kv_indptr, "
        "bool interleave, bool hnd, float beta, int original_max, bool enable_pdl) -> ()");
  m.def("embedding(Tensor input_ids, Tensor weight, bool enable_pdl) -> Tensor");
  m.def("embedding_out(Tensor(a!) out, Tensor input_ids, Tensor weight, bool enable_pdl) -> ()");
  m.def("embedding_fill(Tensor(a!) input_ids, Tensor weight, Tensor last_tokens, bool enable_pdl) -> Tensor");
}

TORCH_LIBRARY_IMPL(mas_b200, CUDA, m) {
  m.impl("fused_add_rmsnorm", &fused_add_rmsnorm);
  m.impl("fused_add_rmsnorm_quant", &fused_add_rmsnorm_quant);
  m.impl("silu_and_mul", &silu_and_mul);
  m.impl("silu_and_mul_quant", &silu_and_mul_quant);
  m.impl("apply_rope_pos_ids_cos_sin_cache", &apply_rope_pos_ids_cos_sin_cache);
  m.impl("apply_rope_q_scale", &apply_rope_q_scale);
  m.impl("append_paged_kv_cache", &append_paged_kv_cache);
  m.impl("rope_append_paged_kv_cache", &rope_append_paged_kv_cache);
  m.impl("embedding", &embedding);
  m.impl("embedding_out", &embedding_out);
  m.impl("embedding_fill", &embedding_fill);
}
