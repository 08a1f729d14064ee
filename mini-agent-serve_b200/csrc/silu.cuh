// silu.cuh -- SiLU-and-mul gating for sm_100a: out[t, i] = round(silu(gate) * up), i < d,
// gate = in[t, i], up = in[t, d + i], silu(v) = v / (1 + exp(-v)) in fp32.
//
// Semantics follow flashinfer 0.6.11.post2 (FI/data/include/flashinfer/activation.cuh:29-65 with
// the activation of FI/jit/activation.py:77-80, which uses the __expf intrinsic): fp32 math and
// one rounding of the product. The quotient here is the IEEE-rounded one.
//
// Pure streaming (3 x 2 bytes per output element, nothing reused), so the design is about bytes in
// flight: a 2-D grid of (column tiles, rows), each thread issuing U pairs of 16-byte streaming loads
// before its first use, with no per-element index division. A scalar path covers d % 8 != 0 and
// unaligned rows.
#pragma once

#include "common.cuh"

namespace mas {

struct SiluArgs {
  void* out;
  const void* in;
  int64_t rows;
  int64_t in_stride;   // elements
  int64_t out_stride;  // elements
  int32_t d;
};

__device__ __forceinline__ float silu_f32(float v) { return v / (1.0f + __expf(-v)); }

constexpr int kSiluThreads = 256;

template <typename T, int U>
__global__ void __launch_bounds__(kSiluThreads) silu_mul_vec_kernel(const SiluArgs a) {
  pdl_wait();
  const int nvec = a.d >> 3;
  const int tile = kSiluThreads * U;
  for (int64_t row = blockIdx.y; row < a.rows; row += gridDim.y) {
    const T* g = static_cast<const T*>(a.in) + row * a.in_stride;
    const T* u = g + a.d;
    T* o = static_cast<T*>(a.out) + row * a.out_stride;
    for (int v0 = blockIdx.x * tile + threadIdx.x; v0 < nvec; v0 += gridDim.x * tile) {
      Vec16 gv[U], uv[U];
#pragma unroll
      for (int i = 0; i < U; ++i) {
        const int v = v0 + i * kSiluThreads;
        if (v < nvec) {
          gv[i] = ld_stream(g + (size_t)v * 8);
          uv[i] = ld_stream(u + (size_t)v * 8);
        }
      }
#pragma unroll
      for (int i = 0; i < U; ++i) {
        const int v = v0 + i * kSiluThreads;
        if (v < nvec) {
          float gf[8], uf[8], y[8];
          unpack8<T>(gv[i], gf);
          unpack8<T>(uv[i], uf);
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = silu_f32(gf[e]) * uf[e];
          st_plain(o + (size_t)v * 8, pack8<T>(y));
        }
      }
    }
  }
  pdl_launch_dependents();
}

template <typename T>
__global__ void __launch_bounds__(kSiluThreads) silu_mul_generic_kernel(const SiluArgs a) {
  pdl_wait();
  for (int64_t row = blockIdx.y; row < a.rows; row += gridDim.y) {
    const uint16_t* g = static_cast<const uint16_t*>(a.in) + row * a.in_stride;
    const uint16_t* u = g + a.d;
    uint16_t* o = static_cast<uint16_t*>(a.out) + row * a.out_stride;
    for (int i = blockIdx.x * kSiluThreads + threadIdx.x; i < a.d; i += gridDim.x * kSiluThreads) {
      o[i] = Elem<T>::from_f(silu_f32(Elem<T>::to_f(g[i])) * Elem<T>::to_f(u[i]));
    }
  }
  pdl_launch_dependents();
}

}  // namespace mas
