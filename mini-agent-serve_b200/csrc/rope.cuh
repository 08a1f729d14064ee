// rope.cuh -- rotary embedding applied in place to q and k from an fp32 cos|sin cache (sm_100a).
//
// Semantics follow flashinfer 0.6.11.post2, the kernels behind apply_rope_with_cos_sin_cache_inplace
// (FI/data/include/flashinfer/pos_enc.cuh:129-147 neox, :218-234 interleaved, :361-420 token loop):
// cos = cache[pos, i], sin = cache[pos, rotary_dim/2 + i]; fp32 math, rounded once per element.
// Neox pairs element i with i + rotary_dim/2; the interleaved form pairs 2i with 2i + 1.
//
// Three paths. The default, when q heads and k heads are each contiguous within a token (as for
// q/k views of one fused qkv row), is the token-staged TMA ring further below (rope_ring_kernel),
// which can also append k and v to the paged KV cache in the same pass. Padded heads take the vector
// kernel described next, and odd rotary_dim or alignment the generic one.
//
// Vector kernel: work unit = one (token, head). A unit is handled by rotary_dim/16 threads; thread j of a unit
// owns the 8 pairs whose cos/sin are cache[pos, 8j .. 8j+8), so each thread does exactly two
// 16-byte loads and two 16-byte stores of q/k (both halves of its pairs) plus four 16-byte cos/sin
// loads that hit L1 for all heads of a token after the first. Units run token-major, heads of one
// token adjacent, so q and k of a token stream through together, and each thread group takes two
// adjacent units per iteration with all four q/k loads in flight before any position is examined.
// q and k may be strided views of one fused qkv row (Devstral2Attention.forward,
// miniagentserve/models/devstral2/devstral2.py:158).
#pragma once

#include "common.cuh"
#include "paged_kv.cuh"

namespace mas {

struct RopeArgs {
  const void* pos;
  void* q;
  void* k;
  const float* cache;
  int64_t T;
  int64_t P;     // cache rows
  int64_t qsn, qsh, ksn, ksh;  // element strides
  int32_t Hq, Hkv;
  int32_t rd;    // rotary dim
  int32_t tpu;   // threads per unit, rd / 16 (vector path)
  int32_t* status;
  float q_beta;      // llama-4 query scale (0: off), see llama4_q_scale
  float q_inv_orig;  // fp32 reciprocal of original_max_position_embeddings
};

constexpr int kRopeThreads = 256;

__device__ __forceinline__ void load_f8(const float* p, float (&f)[8]) {
  const Vec16 a = ld_ro(p);
  const Vec16 b = ld_ro(p + 4);
  f[0] = __uint_as_float(a.a); f[1] = __uint_as_float(a.b);
  f[2] = __uint_as_float(a.c); f[3] = __uint_as_float(a.d);
  f[4] = __uint_as_float(b.a); f[5] = __uint_as_float(b.b);
  f[6] = __uint_as_float(b.c); f[7] = __uint_as_float(b.d);
}

// The rotation of one pair, evaluated as flashinfer's compiled kernel does (pos_enc.cuh:129-147
// and :218-234 contract to one fused multiply-add with a separately rounded second product):
//   a' = fma(a, c, -(b*s)),  b' = fma(b, c, a*s).
// Written with explicit intrinsics so the result does not depend on the compiler's contraction.
__device__ __forceinline__ void rotate(float a, float b, float c, float s, float& ra, float& rb) {
  ra = __fmaf_rn(a, c, -__fmul_rn(b, s));
  rb = __fmaf_rn(b, c, __fmul_rn(a, s));
}

// `rotate` on the 8 neox pairs (x0[e], x1[e]) of one group, two pairs per packed instruction:
// b*(-s) is exactly -(b*s), so with nsn = -sn the packed form rounds every lane as `rotate` does.
__device__ __forceinline__ void rotate8_neox(const float (&x0)[8], const float (&x1)[8], const float (&cs)[8],
                                             const float (&sn)[8], const float (&nsn)[8], float (&o0)[8],
                                             float (&o1)[8]) {
#pragma unroll
  for (int e = 0; e < 8; e += 2) {
    const float2 a = make_float2(x0[e], x0[e + 1]), b = make_float2(x1[e], x1[e + 1]);
    const float2 c = make_float2(cs[e], cs[e + 1]);
    const float2 ra = fma2_f32(a, c, mul2_f32(b, make_float2(nsn[e], nsn[e + 1])));
    const float2 rb = fma2_f32(b, c, mul2_f32(a, make_float2(sn[e], sn[e + 1])));
    o0[e] = ra.x; o0[e + 1] = ra.y;
    o1[e] = rb.x; o1[e + 1] = rb.y;
  }
}

// llama-4 query scale of a token (Devstral2Attention.forward, devstral2.py:175-179), evaluated the
// way eager torch evaluates `1 + beta * log1p(floor(pos.float() / original_max))` on CUDA: the
// division by the host scalar is a multiplication by its fp32 reciprocal, every operation is rounded
// separately (no contraction into an fma), and the result is rounded to the activation type before
// it multiplies q.
template <typename T>
__device__ __forceinline__ float llama4_q_scale(int64_t pos, float beta, float inv_orig) {
  const float k = floorf(__fmul_rn((float)pos, inv_orig));
  return Elem<T>::to_f(Elem<T>::from_f(__fadd_rn(1.0f, __fmul_rn(beta, log1pf(k)))));
}

// The rotated q value as the reference holds it (rounded to T), times the token's scale.
template <typename T>
__device__ __forceinline__ float scaled_q(float rotated, float scale) {
  return __fmul_rn(Elem<T>::to_f(Elem<T>::from_f(rotated)), scale);
}

// The same scale applied to eight rotated q values already packed as T, two per packed multiply.
// The product of two bf16 (8-bit significands) or two fp16 (11-bit) values is exact in fp32, so the
// packed multiply's single rounding to T equals scaled_q's fp32 product rounded to T.
template <typename T>
__device__ __forceinline__ uint32_t mul2_rn(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t mul2_rn<__nv_bfloat16>(uint32_t a, uint32_t b) {
  const __nv_bfloat162 r = __hmul2_rn(*reinterpret_cast<const __nv_bfloat162*>(&a),
                                      *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
template <>
__device__ __forceinline__ uint32_t mul2_rn<__half>(uint32_t a, uint32_t b) {
  const __half2 r = __hmul2_rn(*reinterpret_cast<const __half2*>(&a), *reinterpret_cast<const __half2*>(&b));
  return *reinterpret_cast<const uint32_t*>(&r);
}
template <typename T>
__device__ __forceinline__ Vec16 scaled_q8(const Vec16& v, uint32_t scale2) {
  Vec16 r;
  r.a = mul2_rn<T>(v.a, scale2);
  r.b = mul2_rn<T>(v.b, scale2);
  r.c = mul2_rn<T>(v.c, scale2);
  r.d = mul2_rn<T>(v.d, scale2);
  return r;
}

// Each thread group handles kRopeUnits adjacent units per iteration (usually heads of one token,
// so the position and the cos/sin row are shared). All q/k loads of the iteration are issued before
// the position is checked: a load never waits on another load's latency, and a position out of
// range only suppresses the stores.
constexpr int kRopeUnits = 2;

template <typename T, typename PosT, bool NEOX>
__global__ void __launch_bounds__(kRopeThreads) rope_vec_kernel(const RopeArgs a) {
  pdl_wait();
  const int tpu = a.tpu;
  const int g = threadIdx.x / tpu;
  const int j = threadIdx.x - g * tpu;
  const int upb = kRopeThreads / tpu;
  if (g < upb) {
    const uint32_t NH = (uint32_t)(a.Hq + a.Hkv);
    const uint32_t units = (uint32_t)a.T * NH;  // host guarantees < 2^31
    const int half = a.rd >> 1;
    const PosT* pos_p = static_cast<const PosT*>(a.pos);
    // element offsets of this thread's two 16-byte vectors within a head
    const int off0 = NEOX ? j * 8 : j * 16;
    const int off1 = NEOX ? half + j * 8 : j * 16 + 8;
    const uint32_t stride = gridDim.x * (uint32_t)upb * kRopeUnits;
    for (uint32_t u0 = (blockIdx.x * (uint32_t)upb + (uint32_t)g) * kRopeUnits; u0 < units; u0 += stride) {
      T* ptr[kRopeUnits];
      uint32_t tok[kRopeUnits], head[kRopeUnits];
      Vec16 v0[kRopeUnits], v1[kRopeUnits];
#pragma unroll
      for (int i = 0; i < kRopeUnits; ++i) {
        const uint32_t u = u0 + i;
        ptr[i] = nullptr;
        if (u < units) {
          const uint32_t t = u / NH;
          const uint32_t h = u - t * NH;
          tok[i] = t;
          head[i] = h;
          ptr[i] = (h < (uint32_t)a.Hq)
                       ? static_cast<T*>(a.q) + (int64_t)t * a.qsn + (int64_t)h * a.qsh
                       : static_cast<T*>(a.k) + (int64_t)t * a.ksn + (int64_t)(h - a.Hq) * a.ksh;
          v0[i] = ld_plain(ptr[i] + off0);
          v1[i] = ld_plain(ptr[i] + off1);
        }
      }
#pragma unroll
      for (int i = 0; i < kRopeUnits; ++i) {
        if (ptr[i] == nullptr) continue;
        const int64_t pos = (int64_t)pos_p[tok[i]];
        if (pos < 0 || pos >= a.P) {
          if (j == 0) flag_status(a.status, MAS_STATUS_ROPE_POS_OUT_OF_RANGE);
          continue;
        }
        const float* c = a.cache + pos * a.rd;
        float cs[8], sn[8], x0[8], x1[8], o0[8], o1[8];
        load_f8(c + j * 8, cs);
        load_f8(c + half + j * 8, sn);
        unpack8<T>(v0[i], x0);
        unpack8<T>(v1[i], x1);
        if constexpr (NEOX) {
#pragma unroll
          for (int e = 0; e < 8; ++e) rotate(x0[e], x1[e], cs[e], sn[e], o0[e], o1[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            rotate(x0[2 * e], x0[2 * e + 1], cs[e], sn[e], o0[2 * e], o0[2 * e + 1]);
            rotate(x1[2 * e], x1[2 * e + 1], cs[4 + e], sn[4 + e], o1[2 * e], o1[2 * e + 1]);
          }
        }
        if (a.q_beta != 0.f && head[i] < (uint32_t)a.Hq) {
          const float qs = llama4_q_scale<T>(pos, a.q_beta, a.q_inv_orig);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            o0[e] = scaled_q<T>(o0[e], qs);
            o1[e] = scaled_q<T>(o1[e], qs);
          }
        }
        st_plain(ptr[i] + off0, pack8<T>(o0));
        st_plain(ptr[i] + off1, pack8<T>(o1));
      }
    }
  }
  pdl_launch_dependents();
}

// Token-staged ring (q heads and k heads each contiguous within a token, 16-byte aligned rows): a
// persistent, warp-specialised TMA ring. Each CTA owns a contiguous block of tokens; their positions
// are staged in shared memory up front (one coalesced read, validated there). Warp 0's first lane
// streams, per token, the q row, the k row and the token's cos|sin cache row into an S-stage ring
// with three bulk copies (cp.async.bulk, `full` mbarrier). The consumer warps rotate every pair of
// the token from shared memory (cos/sin included), store the results to q/k with 16-byte stores,
// and release the stage on its `empty` mbarrier. A token whose position is out of range gets no
// copies and no stores. Every wait is bounded.
//
// APPEND fuses the paged KV append that follows rope in the attention layer (paged_kv.cuh): the
// token's v row is staged too and its cache slot is computed in the position pre-pass, the rotated
// k vectors go to the k cache as well as back to k, and the consumers copy the k tail past
// rotary_dim and the v heads from shared memory into the cache. k and v are read from HBM once.
struct RopeRingArgs {
  const void* pos;
  void* q;
  void* k;
  const float* cache;
  int64_t T;
  int64_t P;
  int64_t qsn, ksn;          // token strides (elements); heads are contiguous (stride = head_size)
  int32_t Hq, Hkv, D, rd;
  int32_t stages;
  int32_t tokens_per_cta;
  int32_t* status;
  int32_t* fault;
  float q_beta;      // llama-4 query scale (0: off), see llama4_q_scale
  float q_inv_orig;
  const void* v;     // APPEND: v rows (heads contiguous), token stride vsn
  int64_t vsn;
  PagedKVArgs kv;
  int32_t early_dependents;  // signal programmatic dependents after the prologue instead of at the end
  int32_t prefetch_qk;       // start the first stages' q/k copies before the positions are staged
};

constexpr int kRopeConsumerWarps = 8;        // default consumer warps per CTA
constexpr int kRopeMaxConsumerWarps = 16;
constexpr int kRopeRingMaxThreads = 32 * (1 + kRopeMaxConsumerWarps);
constexpr int kRopeMaxTokensPerCta = 2048;

__host__ __device__ inline uint32_t rope_stage_bytes(int Hq, int Hkv, int D, int rd, int elem_bytes, bool append) {
  return (uint32_t)((Hq + Hkv + (append ? Hkv : 0)) * D * elem_bytes + rd * 4);
}
// Per token: its position (and, with APPEND, its cache slot) as int64.
__host__ __device__ inline size_t rope_ring_smem_bytes(uint32_t stage, int stages, int tokens_per_cta, bool append) {
  return (size_t)stages * stage + (size_t)stages * 16 + (size_t)tokens_per_cta * (append ? 16 : 8);
}

template <typename T, typename PosT, bool NEOX, bool APPEND>
__global__ void __launch_bounds__(kRopeRingMaxThreads) rope_ring_kernel(const RopeRingArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int S = a.stages;
  const int NH = a.Hq + a.Hkv;
  const uint32_t q_bytes = (uint32_t)(a.Hq * a.D) * (uint32_t)sizeof(T);
  const uint32_t k_bytes = (uint32_t)(a.Hkv * a.D) * (uint32_t)sizeof(T);
  const uint32_t v_bytes = APPEND ? k_bytes : 0u;
  const uint32_t c_bytes = (uint32_t)a.rd * 4u;
  const uint32_t stage_bytes = q_bytes + k_bytes + v_bytes + c_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  uint64_t* empty = full + S;
  int64_t* spos = reinterpret_cast<int64_t*>(empty + S);
  int64_t* sslot = spos + a.tokens_per_cta;  // APPEND only
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int64_t tok0 = (int64_t)blockIdx.x * a.tokens_per_cta;
  const int n = (int)min((int64_t)a.tokens_per_cta, a.T - tok0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], (blockDim.x >> 5) - 1);  // one arrival per consumer warp
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  T* const qb = static_cast<T*>(a.q);
  T* const kb = static_cast<T*>(a.k);
  // A token's q and k rows do not depend on its position: the producer lane starts the first
  // stages' q/k copies (expected bytes raised, no arrival yet) before the positions are read and
  // staged; the cos|sin row (and v) and the stage's one arrival follow in the loop below.
  const int pre = a.prefetch_qk ? min(n, S) : 0;
  if (tid == 0) {
    for (int i = 0; i < pre; ++i) {
      unsigned char* st = smem + (size_t)i * stage_bytes;
      const int64_t t = tok0 + i;
      mbar_expect_tx(&full[i], q_bytes + k_bytes);
      if (q_bytes) bulk_load(st, qb + t * a.qsn, q_bytes, &full[i]);
      if (k_bytes) bulk_load(st + q_bytes, kb + t * a.ksn, k_bytes, &full[i]);
    }
  }
  const PosT* pos_p = static_cast<const PosT*>(a.pos) + tok0;
  for (int i = tid; i < n; i += blockDim.x) {
    const int64_t pos = (int64_t)pos_p[i];
    const bool valid = pos >= 0 && pos < a.P;
    if (!valid) flag_status(a.status, MAS_STATUS_ROPE_POS_OUT_OF_RANGE);
    spos[i] = valid ? pos : -1;
    if constexpr (APPEND) {
      int64_t slot = -1;
      if (valid) {
        slot = kv_slot(a.kv, tok0 + i, pos);
        if (slot < 0) flag_status(a.status, MAS_STATUS_KV_SLOT_OUT_OF_RANGE);
      }
      sslot[i] = slot;
    }
  }
  __syncthreads();
  // The grid is resident (at most the SMs' capacity), so letting the next kernel's CTAs launch now
  // only lets them take the SM space this kernel leaves free; their griddepcontrol.wait still waits
  // for this whole grid to finish.
  if (a.early_dependents) pdl_launch_dependents();

  int issued = 0;     // producer lane: tokens whose stage has been filled (or marked empty)
  bool gave_up = false;  // this thread's bounded wait ran out
  if (warp == 0) {
    if (lane == 0) {
      for (int i = 0; i < n; ++i) {
        const int s = i % S;
        if (i >= S && !mbar_wait_bounded(&empty[s], (uint32_t)((i / S) - 1) & 1u)) {
          atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
          gave_up = true;
          break;
        }
        issued = i + 1;
        const int64_t pos = spos[i];
        if (pos < 0) {  // (prefetched q/k still land before the phase completes)
          mbar_arrive(&full[s]);
          continue;
        }
        unsigned char* st = smem + (size_t)s * stage_bytes;
        const int64_t t = tok0 + i;
        const bool with_v = APPEND && v_bytes != 0u && sslot[i] >= 0;
        const bool qk_in_flight = i < pre;
        mbar_arrive_expect_tx(&full[s], c_bytes + (with_v ? v_bytes : 0u) + (qk_in_flight ? 0u : q_bytes + k_bytes));
        if (!qk_in_flight) {
          if (q_bytes) bulk_load(st, qb + t * a.qsn, q_bytes, &full[s]);
          if (k_bytes) bulk_load(st + q_bytes, kb + t * a.ksn, k_bytes, &full[s]);
        }
        if (with_v) bulk_load(st + q_bytes + k_bytes, static_cast<const T*>(a.v) + t * a.vsn, v_bytes, &full[s]);
        bulk_load(st + q_bytes + k_bytes + v_bytes, a.cache + pos * a.rd, c_bytes, &full[s]);
      }
    }
  } else {
    const int ct = tid - 32;
    const int ncons = blockDim.x - 32;
    const int tpu = a.rd >> 4;  // threads' worth of 8-pair groups per head
    const int half = a.rd >> 1;
    const int groups = NH * tpu;
    // When the consumer count is a multiple of tpu, every thread keeps one pair group j for all heads
    // and tokens: its cos/sin values are read once per token and the heads follow by a fixed step.
    const bool fixed_j = ncons % tpu == 0;
    const int jf = ct % tpu, h0 = ct / tpu, hstep = ncons / tpu;
    for (int i = 0; i < n; ++i) {
      const int s = i % S;
      // every lane waits (each needs the barrier's acquire); the warp gives up as one
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (uint32_t)(i / S) & 1u))) {
        if (lane == 0) atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
        gave_up = true;
        break;
      }
      if (spos[i] >= 0) {
        const unsigned char* st = smem + (size_t)s * stage_bytes;
        const float* c = reinterpret_cast<const float*>(st + q_bytes + k_bytes + v_bytes);
        const int64_t t = tok0 + i;
        const int64_t slot = APPEND ? sslot[i] : -1;
        const float qs = a.q_beta != 0.f ? llama4_q_scale<T>(spos[i], a.q_beta, a.q_inv_orig) : 0.f;
        const uint32_t qs2 = Elem<T>::from_f2(qs, qs);  // exact: qs is already a T value
        // One group: the 8 rotation pairs of staged head h held in the 16-byte vectors at off0, off1.
        const auto group = [&](int h, int j, const float (&cs)[8], const float (&sn)[8], const float (&nsn)[8]) {
          const T* sh = reinterpret_cast<const T*>(st) + (size_t)h * a.D;  // staged head (q then k)
          T* gh = h < a.Hq ? qb + t * a.qsn + (int64_t)h * a.D : kb + t * a.ksn + (int64_t)(h - a.Hq) * a.D;
          const int off0 = NEOX ? j * 8 : j * 16;
          const int off1 = NEOX ? half + j * 8 : j * 16 + 8;
          float x0[8], x1[8], o0[8], o1[8];
          unpack8<T>(*reinterpret_cast<const Vec16*>(sh + off0), x0);
          unpack8<T>(*reinterpret_cast<const Vec16*>(sh + off1), x1);
          if constexpr (NEOX) {
            rotate8_neox(x0, x1, cs, sn, nsn, o0, o1);
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              rotate(x0[2 * e], x0[2 * e + 1], cs[e], sn[e], o0[2 * e], o0[2 * e + 1]);
              rotate(x1[2 * e], x1[2 * e + 1], cs[4 + e], sn[4 + e], o1[2 * e], o1[2 * e + 1]);
            }
          }
          const Vec16 p0 = pack8<T>(o0), p1 = pack8<T>(o1);
          if (a.q_beta != 0.f && h < a.Hq) {
            st_plain(gh + off0, scaled_q8<T>(p0, qs2));
            st_plain(gh + off1, scaled_q8<T>(p1, qs2));
          } else {
            st_plain(gh + off0, p0);
            st_plain(gh + off1, p1);
          }
          if (APPEND && h >= a.Hq && slot >= 0) {
            T* ch = static_cast<T*>(a.kv.k_cache) + slot + (int64_t)(h - a.Hq) * a.kv.stride_head;
            st_plain(ch + off0, p0);
            st_plain(ch + off1, p1);
          }
        };
        // cos/sin of pair group j (cos in c[0, half), sin in c[half, rd)).
        // (nsn = -sn feeds the packed neox rotation.)
        const auto load_cs = [&](int j, float (&cs)[8], float (&sn)[8], float (&nsn)[8]) {
          const float4 c0 = *reinterpret_cast<const float4*>(c + j * 8);
          const float4 c1 = *reinterpret_cast<const float4*>(c + j * 8 + 4);
          const float4 s0 = *reinterpret_cast<const float4*>(c + half + j * 8);
          const float4 s1 = *reinterpret_cast<const float4*>(c + half + j * 8 + 4);
          cs[0] = c0.x; cs[1] = c0.y; cs[2] = c0.z; cs[3] = c0.w;
          cs[4] = c1.x; cs[5] = c1.y; cs[6] = c1.z; cs[7] = c1.w;
          sn[0] = s0.x; sn[1] = s0.y; sn[2] = s0.z; sn[3] = s0.w;
          sn[4] = s1.x; sn[5] = s1.y; sn[6] = s1.z; sn[7] = s1.w;
#pragma unroll
          for (int e = 0; e < 8; ++e) nsn[e] = NEOX ? -sn[e] : 0.f;
        };
        if (fixed_j) {
          float cs[8], sn[8], nsn[8];
          load_cs(jf, cs, sn, nsn);
          for (int h = h0; h < NH; h += hstep) group(h, jf, cs, sn, nsn);
        } else {
          for (int gi = ct; gi < groups; gi += ncons) {
            const int h = gi / tpu;
            const int j = gi - h * tpu;
            float cs[8], sn[8], nsn[8];
            load_cs(j, cs, sn, nsn);
            group(h, j, cs, sn, nsn);
          }
        }
        if constexpr (APPEND) {
          // the k tail past rotary_dim (unrotated) and every v head: staged rows -> cache
          if (slot >= 0) {
            const int tail_v = (a.D - a.rd) >> 3;  // 16-byte vectors per k head tail
            const int d_v = a.D >> 3;               // 16-byte vectors per v head
            const int n_tail = a.Hkv * tail_v;
            const int n_copy = n_tail + a.Hkv * d_v;
            const T* sk = reinterpret_cast<const T*>(st + q_bytes);
            const T* sv = reinterpret_cast<const T*>(st + q_bytes + k_bytes);
            // Copies go to the highest-numbered consumers first: with fixed pair groups the lowest-
            // numbered ones take the extra heads, so this evens out the work per thread and token.
            for (int u = ncons - 1 - ct; u < n_copy; u += ncons) {
              if (u < n_tail) {
                const int h = u / tail_v, j = u - h * tail_v;
                const int off = a.rd + j * 8;
                st_plain(static_cast<T*>(a.kv.k_cache) + slot + (int64_t)h * a.kv.stride_head + off,
                         *reinterpret_cast<const Vec16*>(sk + (size_t)h * a.D + off));
              } else {
                const int r = u - n_tail;
                const int h = r / d_v, j = r - h * d_v;
                st_plain(static_cast<T*>(a.kv.v_cache) + slot + (int64_t)h * a.kv.stride_head + j * 8,
                         *reinterpret_cast<const Vec16*>(sv + (size_t)h * a.D + j * 8));
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
  }
  // After a wait gave up anywhere in the CTA, the producer lane waits for the copies it issued
  // before the CTA's shared memory is released.
  if (__syncthreads_or(gave_up) && tid == 0) drain_ring(full, S, issued);
  pdl_launch_dependents();
}

// Generic path: one thread per rotation pair, scalar elements, any rotary_dim and alignment.
template <typename T, typename PosT, bool NEOX>
__global__ void __launch_bounds__(kRopeThreads) rope_generic_kernel(const RopeArgs a) {
  pdl_wait();
  const int64_t NH = a.Hq + a.Hkv;
  const int64_t half = a.rd >> 1;
  const int64_t total = a.T * NH * half;
  const PosT* pos_p = static_cast<const PosT*>(a.pos);
  for (int64_t idx = (int64_t)blockIdx.x * kRopeThreads + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * kRopeThreads) {
    const int64_t i = idx % half;
    const int64_t uh = idx / half;
    const int64_t h = uh % NH;
    const int64_t t = uh / NH;
    const int64_t pos = (int64_t)pos_p[t];
    if (pos < 0 || pos >= a.P) {
      if (i == 0 && h == 0) flag_status(a.status, MAS_STATUS_ROPE_POS_OUT_OF_RANGE);
      continue;
    }
    const float c = a.cache[pos * a.rd + i];
    const float s = a.cache[pos * a.rd + half + i];
    uint16_t* p = (h < a.Hq)
                      ? static_cast<uint16_t*>(a.q) + t * a.qsn + h * a.qsh
                      : static_cast<uint16_t*>(a.k) + t * a.ksn + (h - a.Hq) * a.ksh;
    const int64_t i0 = NEOX ? i : 2 * i;
    const int64_t i1 = NEOX ? i + half : 2 * i + 1;
    float r0, r1;
    rotate(Elem<T>::to_f(p[i0]), Elem<T>::to_f(p[i1]), c, s, r0, r1);
    if (a.q_beta != 0.f && h < a.Hq) {
      const float qs = llama4_q_scale<T>(pos, a.q_beta, a.q_inv_orig);
      r0 = scaled_q<T>(r0, qs);
      r1 = scaled_q<T>(r1, qs);
    }
    p[i0] = Elem<T>::from_f(r0);
    p[i1] = Elem<T>::from_f(r1);
  }
  pdl_launch_dependents();
}

// The llama-4 query scale of the elements past rotary_dim (partial rotary only): q[t, h, i] for
// rotary_dim <= i < head_size, one element per thread. Tokens with an out-of-range position are
// left as is, like the rotation.
template <typename T, typename PosT>
__global__ void __launch_bounds__(kRopeThreads) rope_q_tail_scale_kernel(const RopeArgs a, int32_t head_size) {
  pdl_wait();
  const int64_t tail = head_size - a.rd;
  const int64_t total = a.T * a.Hq * tail;
  const PosT* pos_p = static_cast<const PosT*>(a.pos);
  for (int64_t idx = (int64_t)blockIdx.x * kRopeThreads + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * kRopeThreads) {
    const int64_t i = a.rd + idx % tail;
    const int64_t th = idx / tail;
    const int64_t h = th % a.Hq;
    const int64_t t = th / a.Hq;
    const int64_t pos = (int64_t)pos_p[t];
    if (pos < 0 || pos >= a.P) continue;
    uint16_t* p = static_cast<uint16_t*>(a.q) + t * a.qsn + h * a.qsh + i;
    *p = Elem<T>::from_f(__fmul_rn(Elem<T>::to_f(*p), llama4_q_scale<T>(pos, a.q_beta, a.q_inv_orig)));
  }
  pdl_launch_dependents();
}

}  // namespace mas
