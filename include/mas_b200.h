/*
 * mas_b200.h -- C ABI of the B200-native per-token layer ops of mini-agent-serve.
 *
 * Every entry point takes raw device pointers, element counts and element strides, plus the CUDA
 * stream to launch on (a cudaStream_t passed as void*; NULL is the legacy default stream). No entry
 * point allocates, synchronises the host or reads device data on the host, so every one of them can
 * be captured into a CUDA graph once mas_prepare_device() has run for the device (the first call of
 * any entry point on a device runs it too).
 *
 * Return value: 0 on success; a negative MAS_ERR_* code when the arguments are rejected (nothing is
 * launched); a positive cudaError_t when the launch itself failed.
 *
 * Dtype codes (MAS_DTYPE_*) name the element type of the activation tensors.
 *
 * The reference interface each function replaces is cited beside it. Paths are relative to the
 * mini-agent-serve source tree, or (prefix FI/) to flashinfer-python 0.6.11.post2, the third-party
 * package whose kernels the reference calls for these ops.
 */
#ifndef MAS_B200_H_
#define MAS_B200_H_

#include <stdint.h>

#if defined(__GNUC__)
#define MAS_API __attribute__((visibility("default")))
#else
#define MAS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Element types. */
#define MAS_DTYPE_BF16 0
#define MAS_DTYPE_FP16 1
#define MAS_DTYPE_FP32 2
#define MAS_DTYPE_FP8_E4M3 3
#define MAS_DTYPE_INT32 4
#define MAS_DTYPE_INT64 5

/* Host-side status codes (returned). */
#define MAS_OK 0
#define MAS_ERR_INVALID_ARGUMENT (-1) /* null pointer, negative size, stride shorter than a row */
#define MAS_ERR_UNSUPPORTED_DTYPE (-2)
#define MAS_ERR_UNSUPPORTED_SHAPE (-3) /* e.g. odd rotary_dim, head_size < rotary_dim */
#define MAS_ERR_NO_DEVICE (-4)         /* no current CUDA device could be queried */

/* Device-side status bits, OR-ed (atomicOr) into the int32 `status` word the gather, rope and
 * paged-append kernels take. A NULL `status` selects the library's own status word of the current
 * device (mas_read_status_word), so a data error is always recorded somewhere, including in calls
 * traced by torch.compile or replayed from a CUDA graph. No word is ever cleared by the kernels; the
 * caller zeroes and reads it when it chooses (reading is a host sync, so the ops never do). */
#define MAS_STATUS_EMBED_ID_OUT_OF_RANGE 1 /* an id outside [0, vocab): its output row is zeroed */
#define MAS_STATUS_ROPE_POS_OUT_OF_RANGE 2 /* a position outside [0, max_positions): token left as is */
#define MAS_STATUS_COPY_TIMEOUT 4          /* a bulk-copy wait ran past its time limit; outputs undefined */
#define MAS_STATUS_KV_SLOT_OUT_OF_RANGE 8  /* a paged-KV slot index out of range: that token not appended */

/* Library version, (major << 16) | minor. */
MAS_API int mas_version(void);

/* Human-readable text for a return code of any entry point (never NULL). */
MAS_API const char* mas_status_string(int code);

/* One-time per-device set-up: shared-memory opt-in for every kernel and the SM count. Idempotent and
 * thread-safe. Call it for each device before the first stream capture that uses the library. */
MAS_API int mas_prepare_device(int device);

/* Reads (and, if `clear` is nonzero, zeroes) the library fault word of `device`: the OR of the
 * MAS_STATUS_* bits raised by kernels that have no caller status word (bulk-copy wait timeouts of
 * the RMSNorm kernels, for instance). This synchronises the host with the device: a diagnostic,
 * never called by the ops themselves, not for use during stream capture. The reference has no such
 * facility (flashinfer kernels have no bounded waits to report). */
MAS_API int mas_read_fault_word(int device, int32_t* value, int clear);

/* Reads (and, if `clear` is nonzero, zeroes) the library status word of `device`: the OR of the
 * MAS_STATUS_* data-error bits of every call on that device made with a NULL `status` (an
 * out-of-range token id, rope position or paged-KV slot). Host-synchronising, like
 * mas_read_fault_word. It stands in for the device-side index checks by which aten's embedding and
 * flashinfer's kernels would raise or fault (miniagentserve/models/devstral2/devstral2.py:282). */
MAS_API int mas_read_status_word(int device, int32_t* value, int clear);

/*
 * Self-test of failure detection (no counterpart in the reference): launches one thread that waits
 * on an mbarrier nothing completes, bounded by limit_ns nanoseconds (0 < limit_ns <= 2 s, the limit
 * every kernel's own waits use), then sets MAS_STATUS_COPY_TIMEOUT in the library fault word, as a
 * kernel whose bulk copy never landed does. The device stays usable; read the word with
 * mas_read_fault_word. Used by the tests to show that a wait that runs out ends in a status the
 * host can read, without faulting or hanging the GPU.
 */
MAS_API int mas_selftest_bounded_wait(int64_t limit_ns, void* stream);

/*
 * Fused residual add + RMSNorm, in place, bf16/fp16:
 *   h = f32(input) + f32(residual);  residual <- round(h);
 *   input <- round(h * rsqrt(mean(h^2) + eps) * weight)      (mean over hidden_size, h unrounded)
 * Replaces flashinfer.norm.fused_add_rmsnorm (FI/norm/__init__.py:236-274; kernel semantics
 * FI/norm/kernels/fused_add_rmsnorm.py:380-406, FI/data/include/flashinfer/norm.cuh:387-480), called
 * by Devstral2Model.forward for the final norm (miniagentserve/models/devstral2/devstral2.py:305-307).
 * Strides are in elements between consecutive tokens; the hidden dimension is contiguous.
 */
MAS_API int mas_fused_add_rmsnorm(void* input, void* residual, const void* weight, int64_t num_tokens,
                          int64_t hidden_size, int64_t input_stride, int64_t residual_stride,
                          float eps, int dtype, int enable_pdl, void* stream);

/*
 * Fused residual add + RMSNorm + FP8 (e4m3) quantisation:
 *   h as above; residual <- round(h); input unchanged;
 *   out <- e4m3_rn(clamp(h * rstd * weight * (1 / scale[0]), -448, 448))
 * Replaces flashinfer.norm.fused_add_rmsnorm_quant (FI/norm/__init__.py:288-344; kernel semantics
 * FI/norm/kernels/fused_add_rmsnorm.py:700-728, FI/data/include/flashinfer/norm.cuh:517-600), called
 * twice per decoder layer (miniagentserve/models/devstral2/devstral2.py:241-252). `scale` is a
 * device pointer to one float. out_dtype must be MAS_DTYPE_FP8_E4M3.
 */
MAS_API int mas_fused_add_rmsnorm_quant(void* out, const void* input, void* residual, const void* weight,
                                const float* scale, int64_t num_tokens, int64_t hidden_size,
                                int64_t out_stride, int64_t input_stride, int64_t residual_stride,
                                float eps, int dtype, int out_dtype, int enable_pdl, void* stream);

/*
 * SiLU-and-mul gating: out[t, i] = round(silu(f32(in[t, i])) * f32(in[t, d + i])), i < d,
 * silu(v) = v / (1 + exp(-v)).
 * Replaces flashinfer.activation.silu_and_mul (FI/activation.py:77-118; kernel
 * FI/data/include/flashinfer/activation.cuh:29-65, activation FI/jit/activation.py:77-80), called by
 * Devstral2MLP.forward (miniagentserve/models/devstral2/devstral2.py:223-224).
 */
MAS_API int mas_silu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                     int64_t out_stride, int64_t input_stride, int dtype, int enable_pdl,
                     void* stream);

/*
 * SiLU-and-mul fused with the activation quantisation of the down projection that consumes it:
 *   act = round(silu(gate) * up) as mas_silu_and_mul stores it;
 *   out[t * out_stride + i] = e4m3_rn(clamp(f32(act) / scale[0], -448, 448))   (IEEE quotient)
 * Replaces the pair silu_and_mul (miniagentserve/models/devstral2/devstral2.py:224) ->
 * FP8Linear.forward's quantize_fp8(x, activation_scale) (devstral2.py:93-95, :110-111), so the
 * bf16 activation never goes to memory. `scale` is a device pointer to one float; out_dtype must
 * be MAS_DTYPE_FP8_E4M3; out_stride is in bytes (= elements).
 */
MAS_API int mas_silu_and_mul_quant(void* out, const void* input, const float* scale, int64_t num_tokens,
                           int64_t d, int64_t out_stride, int64_t input_stride, int dtype,
                           int out_dtype, int enable_pdl, void* stream);

/*
 * Rotary embedding applied in place to q and k from an fp32 cos|sin cache
 * ([max_positions, rotary_dim]: cos in columns [0, rotary_dim/2), sin in [rotary_dim/2, rotary_dim)).
 * Neox (is_neox=1): for i < rotary_dim/2, with c = cache[pos, i], s = cache[pos, rotary_dim/2 + i]:
 *   x[i] <- x[i]*c - x[i + rotary_dim/2]*s;   x[i + rotary_dim/2] <- x[i + rotary_dim/2]*c + x[i]*s
 * Interleaved (is_neox=0): the pairs are (x[2i], x[2i+1]) with the same c, s.
 * Elements [rotary_dim, head_size) are left untouched. fp32 math, one rounding per element.
 * q is [num_tokens, num_q_heads, head_size] with element strides (q_stride_token, q_stride_head),
 * and likewise k; both may be strided views of one fused qkv row.
 * positions: int32 (positions_dtype MAS_DTYPE_INT32) or int64 (MAS_DTYPE_INT64).
 * A position outside [0, max_positions) leaves that token unchanged and sets
 * MAS_STATUS_ROPE_POS_OUT_OF_RANGE in *status (the library status word when status is NULL).
 * Replaces flashinfer.rope.apply_rope_with_cos_sin_cache_inplace (FI/rope.py:1223-1272; kernels
 * FI/data/include/flashinfer/pos_enc.cuh:129-147, 294-420, dispatch 1295-1372), called by
 * Devstral2Attention.forward (miniagentserve/models/devstral2/devstral2.py:163-166).
 */
MAS_API int mas_rope_cos_sin_cache_inplace(const void* positions, int positions_dtype, void* query,
                                   void* key, const float* cos_sin_cache, int64_t num_tokens,
                                   int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                   int64_t rotary_dim, int64_t max_positions,
                                   int64_t q_stride_token, int64_t q_stride_head,
                                   int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                   int dtype, int32_t* status, int enable_pdl, void* stream);

/*
 * Rotary embedding as mas_rope_cos_sin_cache_inplace, fused with the llama-4 query scale that
 * Devstral2Attention.forward applies after it (miniagentserve/models/devstral2/devstral2.py:175-179):
 *   scale = round(1 + beta * log1p(floor(pos * (1 / original_max))))   (fp32 steps, each rounded)
 *   q <- round(round(rotated q) * scale)            for every element of every q head
 * k is rotated only. The reference computes the scale as a separate tensor and multiplies q out of
 * place; here q is scaled in place (its unscaled value is not used after the scale in the reference).
 * `1 / original_max` is the fp32 reciprocal, as torch evaluates `tensor / host_scalar` on CUDA.
 * q_scale_original_max must be positive; q_scale_beta == 0 gives mas_rope_cos_sin_cache_inplace.
 */
MAS_API int mas_rope_cos_sin_cache_q_scale_inplace(const void* positions, int positions_dtype, void* query,
                                                   void* key, const float* cos_sin_cache, int64_t num_tokens,
                                                   int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                                   int64_t rotary_dim, int64_t max_positions,
                                                   int64_t q_stride_token, int64_t q_stride_head,
                                                   int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                                   float q_scale_beta, int64_t q_scale_original_max, int dtype,
                                                   int32_t* status, int enable_pdl, void* stream);

/*
 * Token-embedding gather: out[t, :] = table[ids[t], :] (a bit copy of hidden_size elements of
 * elem_size bytes). ids: int32 or int64 (ids_dtype). An id outside [0, vocab_size) zeroes its output
 * row and sets MAS_STATUS_EMBED_ID_OUT_OF_RANGE in *status (the library status word when status is NULL).
 * Replaces the aten/inductor embedding behind nn.Embedding.forward, Devstral2Model.embed_tokens
 * (miniagentserve/models/devstral2/devstral2.py:260, :282).
 */
MAS_API int mas_embedding_gather(void* out, const void* table, const void* ids, int ids_dtype,
                         int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                         int64_t out_stride, int64_t table_stride, int elem_size,
                         int32_t* status, int enable_pdl, void* stream);

/*
 * Token-embedding gather fused with ModelRunner.fill_placeholders
 * (miniagentserve/engine/model_runner.py:149-154): an id -1-r (r >= 0) is a placeholder for
 * last_tokens[r], the previous step's sample of row r. Each placeholder is resolved, the resolved id
 * is written back into `ids` (as fill_placeholders does), and the row of the resolved id is gathered,
 * all in one launch. last_tokens: int32 or int64 (last_dtype), num_last entries. A placeholder whose r
 * is not below num_last is an out-of-range id (zero row, MAS_STATUS_EMBED_ID_OUT_OF_RANGE).
 */
MAS_API int mas_embedding_gather_fill_placeholders(void* out, const void* table, void* ids, int ids_dtype,
                                                   const void* last_tokens, int last_dtype, int64_t num_last,
                                                   int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                                                   int64_t out_stride, int64_t table_stride, int elem_size,
                                                   int32_t* status, int enable_pdl, void* stream);

/*
 * The paged KV cache of one attention layer, as flashinfer's paged_kv_t describes it
 * (FI/data/include/flashinfer/page.cuh:161-165): k and v element [page, entry, head, feature] at
 * page * stride_page + entry * stride_entry + head * stride_head + feature (elements; the NHD layout
 * [num_pages, page_size, heads, head_size] has stride_entry = heads * head_size, stride_head =
 * head_size; HND swaps them). kv_indices (int32, num_indices entries) lists the pages of every
 * sequence back to back, sequence b's starting at kv_indptr[b] (int32, batch_size + 1 entries).
 * Devstral2Model.forward passes block_tables.flatten() and arange(batch + 1) * max_blocks
 * (miniagentserve/models/devstral2/devstral2.py:172, :289).
 */
typedef struct MasPagedKVCache {
  void* k_cache;
  void* v_cache;
  int64_t num_pages;
  int64_t page_size;
  int64_t stride_page;
  int64_t stride_entry;
  int64_t stride_head;
  const int32_t* kv_indices;
  int64_t num_indices;
  const int32_t* kv_indptr;
  int64_t batch_size;
} MasPagedKVCache;

/*
 * Appends token t's k and v rows to the paged cache: with b = batch_indices[t] (int32) and
 * p = positions[t] (int32 or int64, positions_dtype), flat = kv_indptr[b] * page_size + p,
 * page = kv_indices[flat / page_size], entry = flat % page_size, then k_cache[page, entry, h, :] =
 * key[t, h, :] and the same for v (byte-exact copies). k/v element (t, h, f) at
 * t * stride_token + h * stride_head + f. A token whose batch index, position, page slot or page id
 * is out of range is not appended and sets MAS_STATUS_KV_SLOT_OUT_OF_RANGE in *status (the library
 * status word when status is NULL).
 * Replaces flashinfer.page.append_paged_kv_cache (FI/page.py:280-406; kernel
 * FI/data/include/flashinfer/page.cuh:259-284), called once per attention layer
 * (miniagentserve/models/devstral2/devstral2.py:170-173). dtype: BF16 or FP16 for k, v and the cache.
 */
MAS_API int mas_append_paged_kv_cache(const void* key, const void* value, const int32_t* batch_indices,
                                      const void* positions, int positions_dtype, const MasPagedKVCache* cache,
                                      int64_t num_tokens, int64_t num_kv_heads, int64_t head_size,
                                      int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_token,
                                      int64_t v_stride_head, int dtype, int32_t* status, int enable_pdl,
                                      void* stream);

/*
 * Rope (and, when q_scale_beta != 0, the llama-4 query scale) on q and k in place, fused with the
 * paged KV append of the rotated k and of v: one launch where the layout allows it (q, k and v heads
 * contiguous within a token, 16-byte aligned rows and cache strides), otherwise the rope launch
 * followed by the append launch. Equal to mas_rope_cos_sin_cache_q_scale_inplace (or
 * mas_rope_cos_sin_cache_inplace when q_scale_beta == 0) followed by mas_append_paged_kv_cache,
 * except that a token whose position is outside [0, max_positions) is neither rotated nor appended
 * (MAS_STATUS_ROPE_POS_OUT_OF_RANGE). Replaces the sequence apply_rope_with_cos_sin_cache_inplace
 * -> append_paged_kv_cache -> llama-4 query scaling of Devstral2Attention.forward
 * (miniagentserve/models/devstral2/devstral2.py:163-179); q_scale_original_max must be > 0 when
 * q_scale_beta != 0.
 */
MAS_API int mas_rope_append_paged_kv_cache(const void* positions, int positions_dtype, void* query, void* key,
                                           const void* value, const float* cos_sin_cache,
                                           const int32_t* batch_indices, const MasPagedKVCache* cache,
                                           int64_t num_tokens, int64_t num_q_heads, int64_t num_kv_heads,
                                           int64_t head_size, int64_t rotary_dim, int64_t max_positions,
                                           int64_t q_stride_token, int64_t q_stride_head, int64_t k_stride_token,
                                           int64_t k_stride_head, int64_t v_stride_token, int64_t v_stride_head,
                                           int is_neox, float q_scale_beta, int64_t q_scale_original_max,
                                           int dtype, int32_t* status, int enable_pdl, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MAS_B200_H_ */
