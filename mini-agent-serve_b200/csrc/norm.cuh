// norm.cuh -- fused residual add + RMSNorm (bf16/fp16 in place, or e4m3 out) for sm_100a.
//
// Semantics follow flashinfer 0.6.11.post2, the kernels the reference calls
// (FI/norm/kernels/fused_add_rmsnorm.py:380-406 and :700-728; FI/data/include/flashinfer/norm.cuh:
// 387-480 and :517-600): h = f32(x) + f32(r) is kept in fp32, the residual is stored as round(h),
// and the norm is taken over the UNROUNDED h: y = h * rsqrt(sum(h^2)/H + eps) * w, rounded once.
// The e4m3 variant multiplies by 1/scale, clamps to +-448 and rounds to nearest even.
//
// Fast paths (rows of H % 8 == 0 elements, 16-byte aligned rows), all staging whole rows of x and r
// in shared memory with bulk copies (cp.async.bulk) and keeping the thread's weight slice in
// registers:
//   - norm_loop_kernel (the default up to H = 3072): a persistent grid; each CTA loops over row
//     groups with the next group's copies in flight in a small ring, every thread a consumer;
//   - norm_loop_keep_kernel (the default for 3072 < H <= 6144): the same loop with one row per CTA
//     and iteration and h kept in registers, each stage refilled as soon as its first pass is done;
//   - norm_row_keep_kernel (the default for 6144 < H <= 12288): one short-lived CTA per row, h kept
//     in registers between the passes;
//   - norm_row_kernel (the default above): one short-lived CTA per group of rows, one mbarrier;
//   - norm_tma_kernel (selectable, and the path for rows too wide for the others): a persistent,
//     warp-specialised ring. Warp 0's first lane streams rows into an S-stage ring (`full`
//     mbarriers); the consumer warps form `groups` groups, group g taking rows g, g + groups, ...,
//     so that several rows are in their reduction phase at once, and release stages on `empty`
//     mbarriers. S must be a multiple of `groups` (see the kernel).
// Every wait is bounded.
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
  int32_t groups;       // fast path: consumer groups per CTA (rows k = g, g + groups, ... per group)
  float eps;
  int32_t* fault;       // library fault word (bulk-copy timeouts)
};

constexpr int kNormMaxWarps = 32;

// Shared-memory bytes of the fast path for one CTA.
constexpr int kNormMaxGroups = 4;

__host__ __device__ inline size_t norm_tma_smem_bytes(int H, int stages, int elem_bytes) {
  const size_t stage = 2ull * (size_t)H * (size_t)elem_bytes;
  return (size_t)stages * stage + (size_t)stages * 16 + kNormMaxGroups * 2 * kNormMaxWarps * sizeof(float);
}

// Named barrier `id` (1 + consumer group) over one group's warps, OR-reducing a predicate (the
// producer warp and the other groups never join it).
__device__ __forceinline__ bool group_sync_or(int id, bool pred, int nthreads) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return out != 0;
}

constexpr int kNormMaxConsumers = 512;

template <typename T, int VPT, bool QUANT>
__global__ void __launch_bounds__(32 + kNormMaxConsumers) norm_tma_kernel(const NormArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;  // 16-byte vectors per row
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  const int S = a.stages;
  unsigned char* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * 2 * row_bytes);
  uint64_t* empty = full + S;
  float* red = reinterpret_cast<float*>(empty + S);  // [2][kNormMaxWarps]

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int G = a.groups;
  const int gsize = (blockDim.x - 32) / G;  // threads per consumer group (a multiple of 32)
  const int gw = gsize >> 5;                // warps per group

  const int64_t row0 = (int64_t)blockIdx.x * a.rows_per_cta;
  const int n = (int)min((int64_t)a.rows_per_cta, a.rows - row0);
  // Stage s serves rows s, s + S, ...; group g consumes rows g, g + G, .... The parity waits below
  // are exact only if a stage's previous row belonged to the same group, i.e. S % G == 0 (a group
  // could otherwise reach a stage two phases early). The host guarantees it; refuse otherwise.
  if (S % G != 0) {
    if (tid == 0) atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
    return;
  }

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], gw);  // each row is consumed by exactly one group
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();

  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);

  int issued = 0;        // producer lane: rows whose copies were issued
  bool gave_up = false;  // this thread's (or its group's) bounded wait ran out
  if (warp == 0) {
    if (lane == 0) {
      for (int k = 0; k < n; ++k) {
        const int s = k % S;
        if (k >= S && !mbar_wait_bounded(&empty[s], (uint32_t)((k / S) - 1) & 1u)) {
          atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
          gave_up = true;
          break;
        }
        issued = k + 1;
        unsigned char* st = ring + (size_t)s * 2 * row_bytes;
        mbar_arrive_expect_tx(&full[s], 2 * row_bytes);
        bulk_load(st, xb + (row0 + k) * a.x_stride, row_bytes, &full[s]);
        bulk_load(st + row_bytes, rb + (row0 + k) * a.r_stride, row_bytes, &full[s]);
      }
    }
  } else {
    const int g = (tid - 32) / gsize;   // consumer group
    const int ct = tid - 32 - g * gsize;  // thread index within the group
    const int cw = ct >> 5;
    // This thread's slice of the weight, for every row.
    Vec16 wv[VPT];
#pragma unroll
    for (int j = 0; j < VPT; ++j) {
      const int v = ct + j * gsize;
      if (v < NV) wv[j] = ld_ro(static_cast<const T*>(a.w) + (size_t)v * 8);
    }
    float inv_scale = 1.0f;
    if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);
    const float inv_h = 1.0f / (float)H;
    float* gred = red + g * 2 * kNormMaxWarps;

    for (int k = g; k < n; k += G) {
      const int s = k % S;
      const bool ok = mbar_wait_bounded(&full[s], (uint32_t)(k / S) & 1u);
      const unsigned char* sx = ring + (size_t)s * 2 * row_bytes;
      const unsigned char* sr = sx + row_bytes;
      const int64_t row = row0 + k;

      // h = x + r, residual <- round(h), sum of h^2. With few columns per thread h stays in
      // registers and the stage is released at once; otherwise h is re-read from the stage in the
      // second pass and the stage is released after it.
      constexpr bool kKeepH = VPT <= 4;
      float h[kKeepH ? VPT : 1][8];
      float ss = 0.f;
      if (ok) {
#pragma unroll
        for (int j = 0; j < VPT; ++j) {
          const int v = ct + j * gsize;
          if (v < NV) {
            float xf[8], rf[8];
            unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), xf);
            unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              xf[e] += rf[e];
              ss += xf[e] * xf[e];
              if constexpr (kKeepH) h[j][e] = xf[e];
            }
            st_plain(rb + row * a.r_stride + (size_t)v * 8, pack8<T>(xf));
          }
        }
      }
      if constexpr (kKeepH) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }

      ss = warp_sum(ss);
      float* red_k = gred + ((k / G) & 1) * kNormMaxWarps;
      if (lane == 0) red_k[cw] = ss;
      if (group_sync_or(1 + g, !ok, gsize)) {
        if (ct == 0) atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
        gave_up = true;
        break;
      }
      float tot = 0.f;
      for (int w = 0; w < gw; ++w) tot += red_k[w];
      const float rstd = rsqrtf(tot * inv_h + a.eps);

#pragma unroll
      for (int j = 0; j < VPT; ++j) {
        const int v = ct + j * gsize;
        if (v < NV) {
          float y[8], wf[8];
          if constexpr (kKeepH) {
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] = h[j][e];
          } else {
            float rf[8];
            unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), y);
            unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
#pragma unroll
            for (int e = 0; e < 8; ++e) y[e] += rf[e];
          }
          unpack8<T>(wv[j], wf);
#pragma unroll
          for (int e = 0; e < 8; ++e) y[e] = y[e] * rstd * wf[e];
          if constexpr (QUANT) {
            uint2 q;
            q.x = (uint32_t)f2_to_e4m3x2(y[0] * inv_scale, y[1] * inv_scale) |
                  ((uint32_t)f2_to_e4m3x2(y[2] * inv_scale, y[3] * inv_scale) << 16);
            q.y = (uint32_t)f2_to_e4m3x2(y[4] * inv_scale, y[5] * inv_scale) |
                  ((uint32_t)f2_to_e4m3x2(y[6] * inv_scale, y[7] * inv_scale) << 16);
            *reinterpret_cast<uint2*>(a.out + row * a.out_stride + (size_t)v * 8) = q;
          } else {
            st_plain(xb + row * a.x_stride + (size_t)v * 8, pack8<T>(y));
          }
        }
      }
      if constexpr (!kKeepH) {
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
  }
  // After a wait gave up anywhere in the CTA, the producer lane waits for the copies it issued
  // before the CTA's shared memory is released.
  if (__syncthreads_or(gave_up) && tid == 0) drain_ring(full, S, issued);
  pdl_launch_dependents();
}

// Row-block variant of the fast path: a non-persistent grid of small CTAs, each owning `rpc` rows
// handled by `tpr` threads apiece. Thread 0 stages all of the CTA's x and r rows with bulk copies
// on one mbarrier; each row's threads then form h from shared memory, reduce it (warp shuffles, a
// shared partial sum per warp, one CTA barrier) and write both outputs, re-reading h from shared
// memory for the second pass. Several such CTAs per SM keep several rows in their reduction phase
// at once. The wait is bounded.
constexpr int kNormRowMaxThreads = 512;

__host__ __device__ inline size_t norm_row_smem_bytes(int H, int rpc, int elem_bytes) {
  return (size_t)rpc * 2 * (size_t)H * (size_t)elem_bytes + 16 + (size_t)(kNormRowMaxThreads / 32) * sizeof(float);
}

// MAXV bounds the 16-byte vectors a thread handles per row (ceil(H/8 / tpr)); the thread's weight
// slice is loaded into registers before the row arrives, so its latency overlaps the bulk copies.
template <typename T, bool QUANT, int MAXV>
__global__ void __launch_bounds__(kNormRowMaxThreads) norm_row_kernel(const NormArgs a, int tpr, int rpc) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + (size_t)rpc * 2 * row_bytes);
  float* red = reinterpret_cast<float*>(bar + 2);
  const int tid = threadIdx.x;
  const int rr = tid / tpr;   // row slot of this thread within the CTA
  const int rt = tid - rr * tpr;
  const int64_t row0 = (int64_t)blockIdx.x * rpc;
  const int nrows = (int)min((int64_t)rpc, a.rows - row0);

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, (uint32_t)nrows * 2 * row_bytes);
    for (int i = 0; i < nrows; ++i) {
      unsigned char* st = smem + (size_t)i * 2 * row_bytes;
      bulk_load(st, xb + (row0 + i) * a.x_stride, row_bytes, bar);
      bulk_load(st + row_bytes, rb + (row0 + i) * a.r_stride, row_bytes, bar);
    }
  }
  float inv_scale = 1.0f;
  if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);
  Vec16 wv[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = rt + j * tpr;
    if (v < NV) wv[j] = ld_ro(static_cast<const T*>(a.w) + (size_t)v * 8);
  }
  const bool ok = mbar_wait_bounded(bar, 0);
  const bool active = rr < nrows;
  const int64_t row = row0 + rr;
  const unsigned char* sx = smem + (size_t)rr * 2 * row_bytes;
  const unsigned char* sr = sx + row_bytes;

  float ss = 0.f;
  if (ok && active) {
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int v = rt + j * tpr;
      if (v >= NV) break;
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
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
      (void)mbar_wait_bounded(bar, 0);  // the copies may still be landing in this CTA's shared memory
    }
    pdl_launch_dependents();
    return;
  }
  if (active) {
    float tot = 0.f;
    const int w0 = (rr * tpr) >> 5, nw = tpr >> 5;
    for (int w = 0; w < nw; ++w) tot += red[w0 + w];
    const float rstd = rsqrtf(tot * (1.0f / (float)H) + a.eps);
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int v = rt + j * tpr;
      if (v >= NV) break;
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
  pdl_launch_dependents();
}

// Row-block variant that keeps h = x + r in registers between the two passes (one row of NT threads
// per CTA, at most MAXV vectors per thread): the second pass needs no shared-memory re-read and no
// re-unpacking, at the price of about 160 registers a thread at MAXV = 12 (3 CTAs of 128 threads per
// SM instead of 4; the launch bounds hold the compiler to that, without them it took 178 registers
// and fit only 2). Steps with few rows use wider rows (NT = 256, 512) to spread each row's latency.
template <typename T, bool QUANT, int MAXV, int NT = 128>
__global__ void __launch_bounds__(NT, NT > 128 ? 1 : (MAXV <= 8 ? 4 : 3)) norm_row_keep_kernel(const NormArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 2 * (size_t)row_bytes);
  float* red = reinterpret_cast<float*>(bar + 2);
  const int tid = threadIdx.x;
  const int64_t row = blockIdx.x;

  if (tid == 0) {
    mbar_init(bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);
  if (tid == 0) {
    mbar_arrive_expect_tx(bar, 2 * row_bytes);
    bulk_load(smem, xb + row * a.x_stride, row_bytes, bar);
    bulk_load(smem + row_bytes, rb + row * a.r_stride, row_bytes, bar);
  }
  float inv_scale = 1.0f;
  if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);
  Vec16 wv[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = tid + j * NT;
    if (v < NV) wv[j] = ld_ro(static_cast<const T*>(a.w) + (size_t)v * 8);
  }
  const bool ok = mbar_wait_bounded(bar, 0);
  const unsigned char* sx = smem;
  const unsigned char* sr = smem + row_bytes;
  float h[MAXV][8];
  float ss = 0.f;
  if (ok) {
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int v = tid + j * NT;
      if (v < NV) {
        float rf[8];
        unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), h[j]);
        unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          h[j][e] += rf[e];
          ss += h[j][e] * h[j][e];
        }
        st_plain(rb + row * a.r_stride + (size_t)v * 8, pack8<T>(h[j]));
      }
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  if (__syncthreads_or(!ok)) {
    if (tid == 0) {
      atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
      (void)mbar_wait_bounded(bar, 0);  // the copies may still be landing in this CTA's shared memory
    }
    pdl_launch_dependents();
    return;
  }
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) tot += red[w];
  const float rstd = rsqrtf(tot * (1.0f / (float)H) + a.eps);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = tid + j * NT;
    if (v < NV) {
      float y[8], wf[8];
      unpack8<T>(wv[j], wf);
#pragma unroll
      for (int e = 0; e < 8; ++e) y[e] = h[j][e] * rstd * wf[e];
      if constexpr (QUANT) {
        uint2 q;
        q.x = (uint32_t)f2_to_e4m3x2(y[0] * inv_scale, y[1] * inv_scale) |
              ((uint32_t)f2_to_e4m3x2(y[2] * inv_scale, y[3] * inv_scale) << 16);
        q.y = (uint32_t)f2_to_e4m3x2(y[4] * inv_scale, y[5] * inv_scale) |
              ((uint32_t)f2_to_e4m3x2(y[6] * inv_scale, y[7] * inv_scale) << 16);
        *reinterpret_cast<uint2*>(a.out + row * a.out_stride + (size_t)v * 8) = q;
      } else {
        st_plain(xb + row * a.x_stride + (size_t)v * 8, pack8<T>(y));
      }
    }
  }
  pdl_launch_dependents();
}

// Persistent variant of the row-block kernel: grid = SMs x resident CTAs, CTA c handling row groups
// c, c + grid, ... (rpc rows each, tpr threads per row). Thread 0 keeps S - 1 groups' bulk copies in
// flight ahead of the one being computed, in an S-stage shared-memory ring (one mbarrier per stage);
// the weight slice stays in registers for the CTA's lifetime. Each iteration ends with a CTA
// barrier, after which the stage just consumed is refilled. No producer warp: every thread computes.
__host__ __device__ inline size_t norm_loop_smem_bytes(int H, int rpc, int stages, int elem_bytes) {
  return (size_t)stages * rpc * 2 * (size_t)H * (size_t)elem_bytes + (size_t)stages * 8 +
         (size_t)(kNormRowMaxThreads / 32) * sizeof(float);
}

template <typename T, bool QUANT, int MAXV>
__global__ void __launch_bounds__(kNormRowMaxThreads) norm_loop_kernel(const NormArgs a, int tpr, int rpc) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;
  const int S = a.stages;
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  const size_t stage_bytes = (size_t)rpc * 2 * row_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  float* red = reinterpret_cast<float*>(bar + S);
  const int tid = threadIdx.x;
  const int rr = tid / tpr;
  const int rt = tid - rr * tpr;
  const int64_t ngroups = (a.rows + rpc - 1) / rpc;
  const int64_t g0 = blockIdx.x, gstep = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);
  auto issue = [&](int64_t g, int s) {
    const int64_t row0 = g * rpc;
    const int n = (int)min((int64_t)rpc, a.rows - row0);
    unsigned char* st = smem + (size_t)s * stage_bytes;
    mbar_arrive_expect_tx(&bar[s], (uint32_t)n * 2 * row_bytes);
    for (int i = 0; i < n; ++i) {
      bulk_load(st + (size_t)i * 2 * row_bytes, xb + (row0 + i) * a.x_stride, row_bytes, &bar[s]);
      bulk_load(st + (size_t)i * 2 * row_bytes + row_bytes, rb + (row0 + i) * a.r_stride, row_bytes, &bar[s]);
    }
  };
  if (tid == 0) {
    for (int k = 0; k < S - 1; ++k) {
      const int64_t g = g0 + (int64_t)k * gstep;
      if (g < ngroups) issue(g, k);
    }
  }
  float inv_scale = 1.0f;
  if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);
  Vec16 wv[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = rt + j * tpr;
    if (v < NV) wv[j] = ld_ro(static_cast<const T*>(a.w) + (size_t)v * 8);
  }

  int k = 0;
  bool timed_out = false;
  for (int64_t g = g0; g < ngroups; g += gstep, ++k) {
    const int s = k % S;
    if (tid == 0) {
      const int64_t gn = g + (int64_t)(S - 1) * gstep;  // refill the stage consumed last iteration
      if (gn < ngroups) {
        fence_proxy_async_smem();
        issue(gn, (k + S - 1) % S);
      }
    }
    const bool ok = mbar_wait_bounded(&bar[s], (uint32_t)(k / S) & 1u);
    const int64_t row0 = g * rpc;
    const bool active = rr < (int)min((int64_t)rpc, a.rows - row0);
    const int64_t row = row0 + rr;
    const unsigned char* sx = smem + (size_t)s * stage_bytes + (size_t)rr * 2 * row_bytes;
    const unsigned char* sr = sx + row_bytes;
    float ss = 0.f;
    if (ok && active) {
#pragma unroll
      for (int j = 0; j < MAXV; ++j) {
        const int v = rt + j * tpr;
        if (v >= NV) break;
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
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    if (__syncthreads_or(!ok)) {
      timed_out = true;
      break;
    }
    if (active) {
      float tot = 0.f;
      const int w0 = (rr * tpr) >> 5, nw = tpr >> 5;
      for (int w = 0; w < nw; ++w) tot += red[w0 + w];
      const float rstd = rsqrtf(tot * (1.0f / (float)H) + a.eps);
#pragma unroll
      for (int j = 0; j < MAXV; ++j) {
        const int v = rt + j * tpr;
        if (v >= NV) break;
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
    __syncthreads();  // stage s and red[] are free again
  }
  if (timed_out && tid == 0) {
    // Iteration k's wait gave up: the fills of iterations k .. k + S - 1 may still be landing in this
    // CTA's shared memory. Wait for each (bounded) before the CTA exits.
    atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
    for (int m = 0; m < S; ++m) {
      const int64_t gm = g0 + (int64_t)(k + m) * gstep;
      if (gm < ngroups) (void)mbar_wait_bounded(&bar[(k + m) % S], (uint32_t)((k + m) / S) & 1u);
    }
  }
  pdl_launch_dependents();
}

// Persistent loop that keeps h = x + r in registers (one row of NT threads per CTA and iteration, at
// most MAXV vectors per thread). Once the first pass has read a stage, that stage is no longer needed:
// thread 0 refills it right after the reduction barrier, so the next copy is in flight while the
// second pass runs from registers, and no barrier closes the iteration (the reduction slots are
// double-buffered by iteration parity instead).
__host__ __device__ inline size_t norm_loop_keep_smem_bytes(int H, int stages, int nt, int elem_bytes) {
  return (size_t)stages * 2 * (size_t)H * (size_t)elem_bytes + (size_t)stages * 8 +
         2 * (size_t)(nt / 32) * sizeof(float);
}

template <typename T, bool QUANT, int MAXV, int NT>
__global__ void __launch_bounds__(NT, 4) norm_loop_keep_kernel(const NormArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int H = a.H;
  const int NV = H >> 3;
  const int S = a.stages;
  const uint32_t row_bytes = (uint32_t)H * (uint32_t)sizeof(T);
  const size_t stage_bytes = 2 * (size_t)row_bytes;
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + (size_t)S * stage_bytes);
  float* red = reinterpret_cast<float*>(bar + S);
  const int tid = threadIdx.x;
  const int64_t g0 = blockIdx.x, gstep = gridDim.x;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bar[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();
  T* const xb = static_cast<T*>(a.x);
  T* const rb = static_cast<T*>(a.r);
  auto issue = [&](int64_t row, int s) {
    unsigned char* st = smem + (size_t)s * stage_bytes;
    mbar_arrive_expect_tx(&bar[s], 2 * row_bytes);
    bulk_load(st, xb + row * a.x_stride, row_bytes, &bar[s]);
    bulk_load(st + row_bytes, rb + row * a.r_stride, row_bytes, &bar[s]);
  };
  if (tid == 0) {
    for (int k = 0; k < S; ++k) {
      const int64_t row = g0 + (int64_t)k * gstep;
      if (row < a.rows) issue(row, k);
    }
  }
  float inv_scale = 1.0f;
  if constexpr (QUANT) inv_scale = 1.0f / __ldg(a.scale);
  Vec16 wv[MAXV];
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = tid + j * NT;
    if (v < NV) wv[j] = ld_ro(static_cast<const T*>(a.w) + (size_t)v * 8);
  }

  int k = 0;
  bool timed_out = false;
  for (int64_t row = g0; row < a.rows; row += gstep, ++k) {
    const int s = k % S;
    const bool ok = mbar_wait_bounded(&bar[s], (uint32_t)(k / S) & 1u);
    const unsigned char* sx = smem + (size_t)s * stage_bytes;
    const unsigned char* sr = sx + row_bytes;
    float h[MAXV][8];
    float ss = 0.f;
    if (ok) {
#pragma unroll
      for (int j = 0; j < MAXV; ++j) {
        const int v = tid + j * NT;
        if (v < NV) {
          float rf[8];
          unpack8<T>(*reinterpret_cast<const Vec16*>(sx + (size_t)v * 16), h[j]);
          unpack8<T>(*reinterpret_cast<const Vec16*>(sr + (size_t)v * 16), rf);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            h[j][e] += rf[e];
            ss += h[j][e] * h[j][e];
          }
          st_plain(rb + row * a.r_stride + (size_t)v * 8, pack8<T>(h[j]));
        }
      }
    }
    ss = warp_sum(ss);
    float* rk = red + (k & 1) * (NT / 32);
    if ((tid & 31) == 0) rk[tid >> 5] = ss;
    if (__syncthreads_or(!ok)) {
      timed_out = true;
      break;
    }
    if (tid == 0) {  // every thread has read stage s: refill it with the row S iterations ahead
      const int64_t rn = row + (int64_t)S * gstep;
      if (rn < a.rows) {
        fence_proxy_async_smem();
        issue(rn, s);
      }
    }
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) tot += rk[w];
    const float rstd = rsqrtf(tot * (1.0f / (float)H) + a.eps);
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
      const int v = tid + j * NT;
      if (v < NV) {
        float y[8], wf[8];
        unpack8<T>(wv[j], wf);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = h[j][e] * rstd * wf[e];
        if constexpr (QUANT) {
          uint2 q;
          q.x = (uint32_t)f2_to_e4m3x2(y[0] * inv_scale, y[1] * inv_scale) |
                ((uint32_t)f2_to_e4m3x2(y[2] * inv_scale, y[3] * inv_scale) << 16);
          q.y = (uint32_t)f2_to_e4m3x2(y[4] * inv_scale, y[5] * inv_scale) |
                ((uint32_t)f2_to_e4m3x2(y[6] * inv_scale, y[7] * inv_scale) << 16);
          *reinterpret_cast<uint2*>(a.out + row * a.out_stride + (size_t)v * 8) = q;
        } else {
          st_plain(xb + row * a.x_stride + (size_t)v * 8, pack8<T>(y));
        }
      }
    }
  }
  if (timed_out && tid == 0) {
    // Iteration k's wait gave up: the fills of iterations k .. k + S - 1 may still be landing in this
    // CTA's shared memory. Wait for each (bounded) before the CTA exits.
    atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
    for (int m = 0; m < S; ++m) {
      const int64_t rm = g0 + (int64_t)(k + m) * gstep;
      if (rm < a.rows) (void)mbar_wait_bounded(&bar[(k + m) % S], (uint32_t)((k + m) / S) & 1u);
    }
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
