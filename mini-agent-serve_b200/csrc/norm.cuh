// norm.cuh -- fused residual add + RMSNorm (bf16/fp16 in place, or e4m3 out) for sm_100a.
//
// Semantics follow flashinfer 0.6.11.post2, the kernels the reference calls
// (FI/norm/kernels/fused_add_rmsnorm.py:380-406 and :700-728; FI/data/include/flashinfer/norm.cuh:
// 387-480 and :517-600): h = f32(x) + f32(r) is kept in fp32, the residual is stored as round(h),
// and the norm is taken over the UNROUNDED h: y = h * rsqrt(sum(h^2)/H + eps) * w, rounded once.
// The e4m3 variant multiplies by 1/scale, clamps to +-448 and rounds to nearest even.
//
// Fast path (rows of H % 8 == 0 elements, 16-byte aligned rows): a persistent grid. Each CTA owns
// a contiguous block of rows and runs an S-stage ring in shared memory; thread 0 streams whole rows
// of x and r into the ring with TMA bulk copies (cp.async.bulk, mbarrier transaction counts), so
// several rows per SM are always in flight. Each thread owns the same VPT 16-byte column slots of
// every row and holds its slice of the weight in registers for the whole kernel. h is recomputed
// from the staged row for the output pass (bit-identical, and it keeps registers low enough for
// several CTAs per SM); a stage is refilled once every thread is past the next row's barrier.
//
// Generic path (any H, stride or alignment): one CTA per row, two passes over global memory; the
// second pass recomputes h from the still-unmodified inputs, so no scratch space is needed.
#pragma once

#include "common.cuh"

namespace mas {

struct NormArgs {
  void* x;              // [rows, x_stride] input; overwritten by y unless `out` is set
  void* r;              // [rows, r_stride] residual, overwritten by round(h)
  const void* w;        // [H] weight
  uint8_t* out;         // [rows, out_stride] e4m3 output (quant variant) or nullptr
  const float* scale;   // quant scale (device, one float)
  int64_t rows;
  int64_t x_stride;     // elements
  int64_t r_stride;
  int64_t out_stride;
  int32_t H;
  int32_t stages;       // ring depth (fast path)
  int32_t rows_per_cta; // fast path
  float eps;
  int32_t* fault;       // library fault word (bulk-copy timeouts)
};

constexpr int kNormMaxWarps = 32;

// Shared-memory bytes of the fast path for one CTA.
__host__ __device__ inline size_t norm_tma_smem_bytes(int H, int stages, int elem_bytes) {
  const size_t stage = 2ull * (size_t)H * (size_t)elem_bytes;
  return (size_t)stages * stage + (size_t)stages * 8 + 2 * kNormMaxWarps * sizeof(float);
}

template <typename T, int VPT, bool QUANT>
__global__ void __launch_bounds__(512) norm_tma_kernel(const NormArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;  // 16-byte vectors per row
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  const int S = a.stages;
  unsigned char* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * 2 * row_bytes);
  float* red = reinterpret_cast<float*>(bars + S);  // [2][kNormMaxWarps]

  const int tid = threadIdx.x;
  const int nt = blockDim.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int nwarps = nt >> 5;

  const int64_t row0 = (int64_t)blockIdx.x * a.rows_per_cta;
  const int n = (int)min((int64_t)a.rows_per_cta, a.rows - row0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();

  // This thread's slice of the weight, for every row.
  Vec16 wv[VPT];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int v = tid + j * nt;
    if (v < NV) wv[j] = ld_cached(static_cast<const T*>(a.w) + (size_t)v * 8);
  }
  float inv_scale = 1.0f;
  if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);

  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);
  auto issue = [&](int k) {
    const int s = k % S;
    unsigned char* st = ring + (size_t)s * 2 * row_bytes;
    mbar_arrive_expect_tx(&bars[s], 2 * row_bytes);
    bulk_load(st, xb + (row0 + k) * a.x_stride, row_bytes, &bars[s]);
    bulk_load(st + row_bytes, rb + (row0 + k) * a.r_stride, row_bytes, &bars[s]);
  };
  if (tid == 0) {
    const int pre = n < S ? n : S;
    for (int k = 0; k < pre; ++k) issue(k);
  }

  const float inv_h = 1.0f / (float)H;
  int k = 0;
  for (; k < n; ++k) {
    const int s = k % S;
    const bool ok = mbar_wait_bounded(&bars[s], (uint32_t)(k / S) & 1u);
    const unsigned char* sx = ring + (size_t)s * 2 * row_bytes;
    const unsigned char* sr = sx + row_bytes;
    const int64_t row = row0 + k;

    // Pass 1: h = x + r, residual <- round(h), sum of h^2.
    float ss = 0.f;
    if (ok) {
#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = tid + j * nt;
        if (v < NV) {
          float xf[8], rf[8];
          unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), xf);
          unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            xf[e] += rf[e];
            ss += xf[e] * xf[e];
          }
          st_plain(rb + row * a.r_stride + (size_t)v * 8, pack8<T>(xf));
        }
      }
    }
    ss = warp_sum(ss);
    float* red_k = red + (k & 1) * kNormMaxWarps;
    if (lane == 0) red_k[warp] = ss;
    // Past this barrier every thread has finished row k-1 entirely, so its stage is free.
    if (__syncthreads_or(!ok)) break;
    if (tid == 0 && k >= 1 && k - 1 + S < n) issue(k - 1 + S);

    float tot = 0.f;
    for (int w = 0; w < nwarps; ++w) tot += red_k[w];
    const float rstd = rsqrtf(tot * inv_h + a.eps);

    // Pass 2: y = h * rstd * w from the same staged row.
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = tid + j * nt;
      if (v < NV) {
        float xf[8], rf[8], wf[8];
        unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), xf);
        unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
        unpack8<T>(wv[j], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) xf[e] = (xf[e] + rf[e]) * rstd * wf[e];
        if constexpr (QUANT) {
          uint2 q;
          q.x = (uint32_t)f2_to_e4m3x2(xf[0] * inv_scale, xf[1] * inv_scale) |
                ((uint32_t)f2_to_e4m3x2(xf[2] * inv_scale, xf[3] * inv_scale) << 16);
          q.y = (uint32_t)f2_to_e4m3x2(xf[4] * inv_scale, xf[5] * inv_scale) |
                ((uint32_t)f2_to_e4m3x2(xf[6] * inv_scale, xf[7] * inv_scale) << 16);
          *reinterpret_cast<uint2*>(a.out + row * a.out_stride + (size_t)v * 8) = q;
        } else {
          st_plain(xb + row * a.x_stride + (size_t)v * 8, pack8<T>(xf));
        }
      }
    }
  }

  if (k < n && tid == 0) {
    // A bulk copy never completed: record it, then wait (bounded) for the copies still in flight
    // into this CTA's ring before the CTA exits and its shared memory is released. Rows issued so
    // far: [0, min(n, S)) from the prologue and row kk-1+S at every completed iteration kk >= 1.
    atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
    const int issued_end = min(n, (k >= 1 ? k - 1 : 0) + S);
    for (int kk = k; kk < issued_end; ++kk)
      (void)mbar_wait_bounded(&bars[kk % S], (uint32_t)(kk / S) & 1u);
  }
  pdl_launch_dependents();
}

// Generic path: one CTA per row, scalar elements, any alignment.
template <typename T, bool QUANT>
__global__ void __launch_bounds__(256) norm_generic_kernel(const NormArgs a) {
  __shared__ float red[kNormMaxWarps];
  const int tid = threadIdx.x, nt = blockDim.x;
  const int H = a.H;
  pdl_wait();
  const float inv_scale = QUANT ? 1.0f / __ldg(a.scale) : 1.0f;
  const uint16_t* wp = static_cast<const uint16_t*>(a.w);
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    uint16_t* xp = static_cast<uint16_t*>(a.x) + row * a.x_stride;
    uint16_t* rp = static_cast<uint16_t*>(a.r) + row * a.r_stride;
    float ss = 0.f;
    for (int i = tid; i < H; i += nt) {
      const float h = Elem<T>::to_f(xp[i]) + Elem<T>::to_f(rp[i]);
      ss += h * h;
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < (nt >> 5); ++w) tot += red[w];
    const float rstd = rsqrtf(tot * (1.0f / (float)H) + a.eps);
    for (int i = tid; i < H; i += nt) {
      const float h = Elem<T>::to_f(xp[i]) + Elem<T>::to_f(rp[i]);
      const float y = h * rstd * Elem<T>::to_f(wp[i]);
      rp[i] = Elem<T>::from_f(h);
      if constexpr (QUANT) {
        a.out[row * a.out_stride + i] = (uint8_t)(f2_to_e4m3x2(y * inv_scale, 0.f) & 0xffu);
      } else {
        xp[i] = Elem<T>::from_f(y);
      }
    }
    __syncthreads();  // red[] is rewritten by the next row
  }
  pdl_launch_dependents();
}

}  // namespace mas
