// rope.cuh -- rotary embedding applied in place to q and k from an fp32 cos|sin cache (sm_100a).
//
// Semantics follow flashinfer 0.6.11.post2, the kernels behind apply_rope_with_cos_sin_cache_inplace
// (FI/data/include/flashinfer/pos_enc.cuh:129-147 neox, :218-234 interleaved, :361-420 token loop):
// cos = cache[pos, i], sin = cache[pos, rotary_dim/2 + i]; fp32 math, rounded once per element.
// Neox pairs element i with i + rotary_dim/2; the interleaved form pairs 2i with 2i + 1.
//
// Work unit = one (token, head). A unit is handled by rotary_dim/16 threads; thread j of a unit
// owns the 8 pairs whose cos/sin are cache[pos, 8j .. 8j+8), so each thread does exactly two
// 16-byte loads and two 16-byte stores of q/k (both halves of its pairs) plus four 16-byte cos/sin
// loads that hit L1 for all heads of a token after the first. Units run token-major, heads of one
// token adjacent, so q and k of a token stream through together, and each thread group takes two
// adjacent units per iteration with all four q/k loads in flight before any position is examined.
// q and k may be strided views of one fused qkv row (Devstral2Attention.forward,
// miniagentserve/models/devstral2/devstral2.py:158).
#pragma once

#include "common.cuh"

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
};

constexpr int kRopeThreads = 256;

__device__ __forceinline__ void load_f8(const float* p, float (&f)[8]) {
  const Vec16 a = ld_cached(p);
  const Vec16 b = ld_cached(p + 4);
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
      uint32_t tok[kRopeUnits];
      Vec16 v0[kRopeUnits], v1[kRopeUnits];
#pragma unroll
      for (int i = 0; i < kRopeUnits; ++i) {
        const uint32_t u = u0 + i;
        ptr[i] = nullptr;
        if (u < units) {
          const uint32_t t = u / NH;
          const uint32_t h = u - t * NH;
          tok[i] = t;
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
        st_plain(ptr[i] + off0, pack8<T>(o0));
        st_plain(ptr[i] + off1, pack8<T>(o1));
      }
    }
  }
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
    p[i0] = Elem<T>::from_f(r0);
    p[i1] = Elem<T>::from_f(r1);
  }
  pdl_launch_dependents();
}

}  // namespace mas
