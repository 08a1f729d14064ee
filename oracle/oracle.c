/*
 * oracle.c -- CPU restatement of the per-token layer ops, for TESTS ONLY.
 *
 * This file is test infrastructure: the parity tests, __graft_entry__.smoke() and the CPU-baseline
 * legs of bench.py call it as the checker. The product path (mini-agent-serve_b200/) never links,
 * loads or calls it.
 *
 * What it restates. The reference (mini-agent-serve) computes these ops through flashinfer-python
 * 0.6.11.post2 (not vendored in the reference; the reference pins no version) and through aten for
 * the embedding. Each function below follows the flashinfer source it cites (paths prefixed FI/ are
 * relative to the installed flashinfer package):
 *   - every op does its arithmetic in fp32 and rounds once to the output type (RNE);
 *   - transcendental and reduction steps are evaluated more accurately here (double sum of squares,
 *     double exp and rsqrt) than on the GPU (fp32 tree sums, __expf, rsqrt.approx); the parity bar
 *     (<= 1 bf16 ulp, or 1 e4m3 step) absorbs the difference.
 * Compiled with -ffp-contract=off so no multiply-add is fused behind the C source's back.
 *
 * Every entry point mirrors the argument order of the matching C-ABI function in
 * include/mas_b200.h (prefix orc_ instead of mas_), minus the stream and PDL flag; the paged-cache
 * functions take the fields of MasPagedKVCache as separate arguments.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORC_BF16 0
#define ORC_FP16 1
#define ORC_INT32 4
#define ORC_INT64 5

/* ---------------------------------------------------------------------------------------------
 * Number formats.
 * --------------------------------------------------------------------------------------------- */
static inline float u32_as_f32(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static inline uint32_t f32_as_u32(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* bfloat16 is the upper half of an IEEE binary32. */
static inline float bf16_to_f32(uint16_t h) { return u32_as_f32((uint32_t)h << 16); }

/* binary32 -> bfloat16, round to nearest even; NaN stays a (quiet) NaN. */
static inline uint16_t f32_to_bf16(float f) {
  uint32_t u = f32_as_u32(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x0040u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

/* binary16 <-> binary32 through the compiler's _Float16 (IEEE conversions, RNE). */
static inline float f16_to_f32(uint16_t h) { _Float16 v; memcpy(&v, &h, 2); return (float)v; }
static inline uint16_t f32_to_f16(float f) { _Float16 v = (_Float16)f; uint16_t h; memcpy(&h, &v, 2); return h; }

static inline float ld_act(const uint16_t* p, int dtype) { return dtype == ORC_BF16 ? bf16_to_f32(*p) : f16_to_f32(*p); }
static inline float ld_act_from(uint16_t h, int dtype) { return dtype == ORC_BF16 ? bf16_to_f32(h) : f16_to_f32(h); }
static inline uint16_t to_act(float f, int dtype) { return dtype == ORC_BF16 ? f32_to_bf16(f) : f32_to_f16(f); }

/* binary32 -> float8 e4m3fn (bias 7, no infinities, max finite 448 = 0x7e, NaN = 0x7f), round to
 * nearest even, saturating: |f| >= 448 (and +-inf) gives +-448, NaN gives NaN. This is the format's
 * definition worked through directly: subnormals step by 2^-9, a normal with unbiased exponent E
 * steps by 2^(E-3). */
uint8_t orc_f32_to_e4m3(float f) {
  if (isnan(f)) return 0x7f;
  const uint8_t sign = signbit(f) ? 0x80 : 0x00;
  const float a = fabsf(f);
  if (a >= 448.0f) return sign | 0x7e;
  if (a < 0.015625f) {                                /* below 2^-6: subnormal (or zero) */
    const float q = rintf(a * 512.0f);                /* exact scaling, then RNE to the 2^-9 grid */
    return sign | (uint8_t)q;                         /* q == 8 is the smallest normal, code 0x08 */
  }
  int e;
  (void)frexpf(a, &e);                                /* a = m * 2^e, m in [0.5, 1) */
  int E = e - 1;                                      /* a in [2^E, 2^(E+1)) */
  float q = rintf(ldexpf(a, 3 - E));                  /* significand in eighths: [8, 16] */
  if (q >= 16.0f) { q = 8.0f; E += 1; }
  const int code = ((E + 7) << 3) | ((int)q - 8);
  return sign | (uint8_t)(code > 0x7e ? 0x7e : code);
}

float orc_e4m3_to_f32(uint8_t b) {
  const float s = (b & 0x80) ? -1.0f : 1.0f;
  const int e = (b >> 3) & 0xf, m = b & 0x7;
  if (e == 0xf && m == 0x7) return NAN;
  if (e == 0) return s * ldexpf((float)m, -9);
  return s * ldexpf((float)(8 + m), e - 10);
}

uint16_t orc_f32_to_bf16(float f) { return f32_to_bf16(f); }
float orc_bf16_to_f32(uint16_t h) { return bf16_to_f32(h); }
uint16_t orc_f32_to_f16(float f) { return f32_to_f16(f); }

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

int orc_get_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------------------------------------
 * Fused add RMSNorm. FI/norm/kernels/fused_add_rmsnorm.py:380-406 (bf16 out) and :700-728 (fp8
 * out); FI/data/include/flashinfer/norm.cuh:405-479 and :537-600:
 *   h = f32(x) + f32(r);  r <- round(h);  rstd = 1/sqrt(sum(h^2)/H + eps);
 *   y = h * rstd * w   (left to right, fp32);  x <- round(y)   or   out <- e4m3(y * (1/scale)).
 * The norm uses the unrounded fp32 h, not round(h).
 * --------------------------------------------------------------------------------------------- */
static void norm_rows(void* out, void* input, void* residual, const void* weight, const float* scale,
                      int64_t T, int64_t H, int64_t out_stride, int64_t in_stride,
                      int64_t res_stride, float eps, int dtype, int quant) {
  const uint16_t* w = (const uint16_t*)weight;
  const float inv_scale = quant ? 1.0f / scale[0] : 1.0f;
#pragma omp parallel
  {
    float* h = (float*)malloc((size_t)H * sizeof(float));
#pragma omp for schedule(static)
    for (int64_t t = 0; t < T; ++t) {
      uint16_t* x = (uint16_t*)input + t * in_stride;
      uint16_t* r = (uint16_t*)residual + t * res_stride;
      double ss = 0.0;
      for (int64_t j = 0; j < H; ++j) {
        const float v = ld_act(&x[j], dtype) + ld_act(&r[j], dtype);
        h[j] = v;
        ss += (double)v * (double)v;
      }
      const float rstd = (float)(1.0 / sqrt(ss / (double)H + (double)eps));
      for (int64_t j = 0; j < H; ++j) {
        r[j] = to_act(h[j], dtype);
        const float y = h[j] * rstd * ld_act(&w[j], dtype);
        if (quant)
          ((uint8_t*)out)[t * out_stride + j] = orc_f32_to_e4m3(y * inv_scale);
        else
          x[j] = to_act(y, dtype);
      }
    }
    free(h);
  }
}

int orc_fused_add_rmsnorm(void* input, void* residual, const void* weight, int64_t num_tokens,
                          int64_t hidden_size, int64_t input_stride, int64_t residual_stride,
                          float eps, int dtype) {
  if (num_tokens < 0 || hidden_size <= 0 || (dtype != ORC_BF16 && dtype != ORC_FP16)) return -1;
  norm_rows(NULL, input, residual, weight, NULL, num_tokens, hidden_size, 0, input_stride,
            residual_stride, eps, dtype, 0);
  return 0;
}

int orc_fused_add_rmsnorm_quant(void* out, const void* input, void* residual, const void* weight,
                                const float* scale, int64_t num_tokens, int64_t hidden_size,
                                int64_t out_stride, int64_t input_stride, int64_t residual_stride,
                                float eps, int dtype) {
  if (num_tokens < 0 || hidden_size <= 0 || (dtype != ORC_BF16 && dtype != ORC_FP16)) return -1;
  norm_rows(out, (void*)input, residual, weight, scale, num_tokens, hidden_size, out_stride,
            input_stride, residual_stride, eps, dtype, 1);
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * SiLU and mul. FI/data/include/flashinfer/activation.cuh:43-49 with FI/jit/activation.py:77-80:
 *   out = round(silu(g) * u),  silu(g) = g / (1 + exp(-g)),  all fp32.
 * exp is evaluated in double and rounded to fp32. flashinfer compiles the quotient with fast math
 * (the approximate divide, g times the reciprocal of the divisor), whose reciprocal is 0 for a
 * divisor of 2^126 or more: silu is then g * 0 (= -0 for the negative g concerned), which the
 * B200 fixtures confirm (gate below about -87.3). Elsewhere the exact quotient is used.
 * --------------------------------------------------------------------------------------------- */
int orc_silu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                     int64_t out_stride, int64_t input_stride, int dtype) {
  if (num_tokens < 0 || d < 0 || (dtype != ORC_BF16 && dtype != ORC_FP16)) return -1;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < num_tokens; ++t) {
    const uint16_t* g = (const uint16_t*)input + t * input_stride;
    const uint16_t* u = g + d;
    uint16_t* o = (uint16_t*)out + t * out_stride;
    for (int64_t i = 0; i < d; ++i) {
      const float gv = ld_act(&g[i], dtype);
      const float e = (float)exp(-(double)gv);
      const float den = 1.0f + e;
      const float s = den >= 0x1p126f ? gv * 0.0f : gv / den;
      o[i] = to_act(s * ld_act(&u[i], dtype), dtype);
    }
  }
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * SiLU-and-mul followed by FP8Linear's activation quantisation, one pass: the reference computes
 *   act = silu_and_mul(gate_up)                 (devstral2.py:224, rounded to bf16/fp16 as above)
 *   x   = quantize_fp8(act, activation_scale)  (devstral2.py:93-95 via FP8Linear.forward :110-111)
 *       = (act / scale).clamp(-448, 448).to(float8_e4m3fn)
 * where torch.compile computes the quotient in fp32 from the upcast activation (IEEE divide, no
 * intermediate rounding to the activation type), clamps (NaN passes through) and converts with
 * round-to-nearest-even. The e4m3 bytes go to out[t * out_stride + i].
 * --------------------------------------------------------------------------------------------- */
int orc_silu_and_mul_quant(void* out, const void* input, const float* scale, int64_t num_tokens,
                           int64_t d, int64_t out_stride, int64_t input_stride, int dtype) {
  if (num_tokens < 0 || d < 0 || (dtype != ORC_BF16 && dtype != ORC_FP16) || !scale) return -1;
  const float sc = *scale;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < num_tokens; ++t) {
    const uint16_t* g = (const uint16_t*)input + t * input_stride;
    const uint16_t* u = g + d;
    uint8_t* o = (uint8_t*)out + t * out_stride;
    for (int64_t i = 0; i < d; ++i) {
      const float gv = ld_act(&g[i], dtype);
      const float e = (float)exp(-(double)gv);
      const float den = 1.0f + e;
      const float s = den >= 0x1p126f ? gv * 0.0f : gv / den;
      const float act = ld_act_from(to_act(s * ld_act(&u[i], dtype), dtype), dtype);
      float q = act / sc;
      if (q == q) q = q < -448.0f ? -448.0f : (q > 448.0f ? 448.0f : q);
      o[i] = orc_f32_to_e4m3(q);
    }
  }
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Rotary embedding from the fp32 cos|sin cache. FI/data/include/flashinfer/pos_enc.cuh:129-147
 * (neox: element i pairs with i + rotary_dim/2), :218-234 (interleaved: 2i pairs with 2i+1), cache
 * row layout :375-391 (cos = cache[pos, i], sin = cache[pos, rotary_dim/2 + i]):
 *   a' = a*cos - b*sin,  b' = b*cos + a*sin,  rounded once to the output type,
 * each evaluated as flashinfer's compiled kernel evaluates `x*cos + (+-y)*sin`: the second product
 * rounded to fp32, then one fused multiply-add (fmaf, exact before its single rounding).
 * Out-of-range positions leave the token as is and set bit 2 of *status.
 * --------------------------------------------------------------------------------------------- */
int orc_rope_cos_sin_cache_inplace(const void* positions, int positions_dtype, void* query,
                                   void* key, const float* cache, int64_t num_tokens,
                                   int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                   int64_t rotary_dim, int64_t max_positions,
                                   int64_t q_stride_token, int64_t q_stride_head,
                                   int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                   int dtype, int32_t* status) {
  if (num_tokens < 0 || rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > head_size) return -1;
  if (dtype != ORC_BF16 && dtype != ORC_FP16) return -1;
  const int64_t half = rotary_dim / 2;
  int32_t flags = 0;
#pragma omp parallel for schedule(static) reduction(| : flags)
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t pos = positions_dtype == ORC_INT64 ? ((const int64_t*)positions)[t]
                                                     : (int64_t)((const int32_t*)positions)[t];
    if (pos < 0 || pos >= max_positions) { flags |= 2; continue; }
    const float* c = cache + pos * rotary_dim;
    const float* s = c + half;
    for (int64_t h = 0; h < num_q_heads + num_kv_heads; ++h) {
      uint16_t* p = h < num_q_heads
                        ? (uint16_t*)query + t * q_stride_token + h * q_stride_head
                        : (uint16_t*)key + t * k_stride_token + (h - num_q_heads) * k_stride_head;
      for (int64_t i = 0; i < half; ++i) {
        const int64_t i0 = is_neox ? i : 2 * i;
        const int64_t i1 = is_neox ? i + half : 2 * i + 1;
        const float a = ld_act(&p[i0], dtype), b = ld_act(&p[i1], dtype);
        const float bs = b * s[i], as = a * s[i];
        p[i0] = to_act(fmaf(a, c[i], -bs), dtype);
        p[i1] = to_act(fmaf(b, c[i], as), dtype);
      }
    }
  }
  if (status) *status |= flags;
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Rotary embedding followed by the llama-4 query scale of Devstral2Attention.forward
 * (miniagentserve/models/devstral2/devstral2.py:163-166 then :175-179), as eager torch evaluates it on
 * CUDA: scale = to_act(1 + beta * log1p(floor(pos_f32 * (1 / original_max)))), each fp32 step rounded
 * on its own (`tensor / host_scalar` is a multiplication by the fp32 reciprocal there); every q
 * element (rotated or not) becomes to_act(to_act(q) * scale). k is rotated only.
 * --------------------------------------------------------------------------------------------- */
static inline float llama4_q_scale(int64_t pos, float beta, float inv_orig, int dtype) {
  const float k = floorf((float)pos * inv_orig);
  const float s = 1.0f + beta * log1pf(k);
  return ld_act_from(to_act(s, dtype), dtype);
}

int orc_rope_cos_sin_cache_q_scale_inplace(const void* positions, int positions_dtype, void* query,
                                           void* key, const float* cache, int64_t num_tokens,
                                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                           int64_t rotary_dim, int64_t max_positions,
                                           int64_t q_stride_token, int64_t q_stride_head,
                                           int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                           float beta, int64_t original_max, int dtype, int32_t* status) {
  if (original_max <= 0) return -1;
  const int rc = orc_rope_cos_sin_cache_inplace(positions, positions_dtype, query, key, cache, num_tokens,
                                                num_q_heads, num_kv_heads, head_size, rotary_dim,
                                                max_positions, q_stride_token, q_stride_head,
                                                k_stride_token, k_stride_head, is_neox, dtype, status);
  if (rc != 0 || beta == 0.0f) return rc;
  const float inv_orig = 1.0f / (float)original_max;
#pragma omp parallel for schedule(static)
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t pos = positions_dtype == ORC_INT64 ? ((const int64_t*)positions)[t]
                                                     : (int64_t)((const int32_t*)positions)[t];
    if (pos < 0 || pos >= max_positions) continue;
    const float sc = llama4_q_scale(pos, beta, inv_orig, dtype);
    for (int64_t h = 0; h < num_q_heads; ++h) {
      uint16_t* p = (uint16_t*)query + t * q_stride_token + h * q_stride_head;
      for (int64_t i = 0; i < head_size; ++i) p[i] = to_act(ld_act(&p[i], dtype) * sc, dtype);
    }
  }
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Paged KV append. FI/data/include/flashinfer/page.cuh:259-284 (kernel) with the element offsets of
 * :161-165: token t of sequence b = batch_indices[t] at position p goes to
 *   flat = kv_indptr[b] * page_size + p, page = kv_indices[flat / page_size], entry = flat % page_size
 * and k_cache[page*stride_page + entry*stride_entry + h*stride_head + f] = k[t, h, f] (same for v),
 * a byte copy. Indices are checked here (the reference kernel trusts them): a batch index outside
 * [0, batch_size), a negative position, flat / page_size outside kv_indices or a page id outside
 * [0, num_pages) skips the token and sets bit 8 of *status. pos_limit > 0 (used by the fused form
 * below) skips tokens at positions outside [0, pos_limit) without flagging them.
 * --------------------------------------------------------------------------------------------- */
static int append_impl(const void* key, const void* value, const int32_t* batch_indices, const void* positions,
                       int positions_dtype, void* k_cache, void* v_cache, int64_t num_pages, int64_t page_size,
                       int64_t stride_page, int64_t stride_entry, int64_t stride_head, const int32_t* kv_indices,
                       int64_t num_indices, const int32_t* kv_indptr, int64_t batch_size, int64_t num_tokens,
                       int64_t num_kv_heads, int64_t head_size, int64_t k_stride_token, int64_t k_stride_head,
                       int64_t v_stride_token, int64_t v_stride_head, int64_t pos_limit, int32_t* status) {
  if (num_tokens < 0 || num_kv_heads < 0 || head_size <= 0 || page_size <= 0) return -1;
  int32_t flags = 0;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t p = positions_dtype == ORC_INT64 ? ((const int64_t*)positions)[t]
                                                   : (int64_t)((const int32_t*)positions)[t];
    if (pos_limit > 0 && (p < 0 || p >= pos_limit)) continue;
    const int64_t b = batch_indices[t];
    if (b < 0 || b >= batch_size || p < 0) { flags |= 8; continue; }
    const int64_t flat = (int64_t)kv_indptr[b] * page_size + p;
    const int64_t page_iter = flat / page_size, entry = flat % page_size;
    if (flat < 0 || page_iter >= num_indices) { flags |= 8; continue; }
    const int64_t page = kv_indices[page_iter];
    if (page < 0 || page >= num_pages) { flags |= 8; continue; }
    for (int64_t h = 0; h < num_kv_heads; ++h) {
      const int64_t dst = page * stride_page + entry * stride_entry + h * stride_head;
      memcpy((uint16_t*)k_cache + dst, (const uint16_t*)key + t * k_stride_token + h * k_stride_head,
             (size_t)head_size * 2);
      memcpy((uint16_t*)v_cache + dst, (const uint16_t*)value + t * v_stride_token + h * v_stride_head,
             (size_t)head_size * 2);
    }
  }
  if (status) *status |= flags;
  return 0;
}

int orc_append_paged_kv_cache(const void* key, const void* value, const int32_t* batch_indices,
                              const void* positions, int positions_dtype, void* k_cache, void* v_cache,
                              int64_t num_pages, int64_t page_size, int64_t stride_page, int64_t stride_entry,
                              int64_t stride_head, const int32_t* kv_indices, int64_t num_indices,
                              const int32_t* kv_indptr, int64_t batch_size, int64_t num_tokens,
                              int64_t num_kv_heads, int64_t head_size, int64_t k_stride_token,
                              int64_t k_stride_head, int64_t v_stride_token, int64_t v_stride_head,
                              int32_t* status) {
  return append_impl(key, value, batch_indices, positions, positions_dtype, k_cache, v_cache, num_pages,
                     page_size, stride_page, stride_entry, stride_head, kv_indices, num_indices, kv_indptr,
                     batch_size, num_tokens, num_kv_heads, head_size, k_stride_token, k_stride_head,
                     v_stride_token, v_stride_head, 0, status);
}

/* Devstral2Attention.forward's sequence (devstral2.py:163-179): rope on q and k, the paged append of
 * the rotated k and of v, then (beta != 0) the llama-4 query scale. A token whose position is
 * outside [0, max_positions) is neither rotated nor appended (bit 2 of *status). */
int orc_rope_append_paged_kv_cache(const void* positions, int positions_dtype, void* query, void* key,
                                   const void* value, const float* cache, const int32_t* batch_indices,
                                   void* k_cache, void* v_cache, int64_t num_pages, int64_t page_size,
                                   int64_t stride_page, int64_t stride_entry, int64_t stride_head,
                                   const int32_t* kv_indices, int64_t num_indices, const int32_t* kv_indptr,
                                   int64_t batch_size, int64_t num_tokens, int64_t num_q_heads,
                                   int64_t num_kv_heads, int64_t head_size, int64_t rotary_dim,
                                   int64_t max_positions, int64_t q_stride_token, int64_t q_stride_head,
                                   int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_token,
                                   int64_t v_stride_head, int is_neox, float beta, int64_t original_max,
                                   int dtype, int32_t* status) {
  int rc = orc_rope_cos_sin_cache_inplace(positions, positions_dtype, query, key, cache, num_tokens, num_q_heads,
                                          num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token,
                                          q_stride_head, k_stride_token, k_stride_head, is_neox, dtype, status);
  if (rc != 0) return rc;
  if (max_positions > 0) {
    rc = append_impl(key, value, batch_indices, positions, positions_dtype, k_cache, v_cache, num_pages, page_size,
                     stride_page, stride_entry, stride_head, kv_indices, num_indices, kv_indptr, batch_size,
                     num_tokens, num_kv_heads, head_size, k_stride_token, k_stride_head, v_stride_token,
                     v_stride_head, max_positions, status);
    if (rc != 0) return rc;
  }
  if (beta == 0.0f) return 0;
  if (original_max <= 0) return -1;
  /* the query scale on the rotated q (k untouched: a second rope pass is not wanted) */
  const float inv_orig = 1.0f / (float)original_max;
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t pos = positions_dtype == ORC_INT64 ? ((const int64_t*)positions)[t]
                                                     : (int64_t)((const int32_t*)positions)[t];
    if (pos < 0 || pos >= max_positions) continue;
    const float sc = llama4_q_scale(pos, beta, inv_orig, dtype);
    for (int64_t h = 0; h < num_q_heads; ++h) {
      uint16_t* p = (uint16_t*)query + t * q_stride_token + h * q_stride_head;
      for (int64_t i = 0; i < head_size; ++i) p[i] = to_act(ld_act(&p[i], dtype) * sc, dtype);
    }
  }
  return 0;
}

/* ---------------------------------------------------------------------------------------------
 * Token-embedding gather: out[t] = table[ids[t]], a byte copy (torch.nn.functional.embedding).
 * Out-of-range ids give a zero row and set bit 1 of *status.
 * --------------------------------------------------------------------------------------------- */
int orc_embedding_gather(void* out, const void* table, const void* ids, int ids_dtype,
                         int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                         int64_t out_stride, int64_t table_stride, int elem_size, int32_t* status) {
  if (num_tokens < 0 || hidden_size <= 0 || elem_size <= 0) return -1;
  const size_t rb = (size_t)hidden_size * (size_t)elem_size;
  int32_t flags = 0;
#pragma omp parallel for schedule(static) reduction(| : flags)
  for (int64_t t = 0; t < num_tokens; ++t) {
    const int64_t id = ids_dtype == ORC_INT64 ? ((const int64_t*)ids)[t]
                                              : (int64_t)((const int32_t*)ids)[t];
    unsigned char* dst = (unsigned char*)out + (size_t)t * (size_t)out_stride * (size_t)elem_size;
    if (id < 0 || id >= vocab_size) { memset(dst, 0, rb); flags |= 1; continue; }
    memcpy(dst, (const unsigned char*)table + (size_t)id * (size_t)table_stride * (size_t)elem_size, rb);
  }
  if (status) *status |= flags;
  return 0;
}

/* ModelRunner.fill_placeholders (miniagentserve/engine/model_runner.py:149-154) then the gather: an id
 * -1-r (r >= 0) is replaced, in `ids`, by last[r]; r >= n_last is an out-of-range id. */
int orc_embedding_gather_fill_placeholders(void* out, const void* table, void* ids, int ids_dtype,
                                           const void* last, int last_dtype, int64_t n_last,
                                           int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                                           int64_t out_stride, int64_t table_stride, int elem_size,
                                           int32_t* status) {
  for (int64_t t = 0; t < num_tokens; ++t) {
    int64_t id = ids_dtype == ORC_INT64 ? ((int64_t*)ids)[t] : (int64_t)((int32_t*)ids)[t];
    if (id >= 0) continue;
    const int64_t r = -1 - id;
    if (r >= n_last) continue; /* stays negative: gathered as out of range */
    id = last_dtype == ORC_INT64 ? ((const int64_t*)last)[r] : (int64_t)((const int32_t*)last)[r];
    if (ids_dtype == ORC_INT64) ((int64_t*)ids)[t] = id; else ((int32_t*)ids)[t] = (int32_t)id;
  }
  return orc_embedding_gather(out, table, ids, ids_dtype, num_tokens, hidden_size, vocab_size, out_stride,
                              table_stride, elem_size, status);
}
