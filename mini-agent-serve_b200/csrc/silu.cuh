// silu.cuh -- SiLU-and-mul gating for sm_100a: out[t, i] = round(silu(gate) * up), i < d,
// gate = in[t, i], up = in[t, d + i], silu(v) = v / (1 + exp(-v)) in fp32.
//
// Semantics follow flashinfer 0.6.11.post2 (FI/data/include/flashinfer/activation.cuh:29-65 with
// the activation of FI/jit/activation.py:77-80, compiled with fast math: the __expf intrinsic and
// the approximate divide): fp32 math and one rounding of the product.
//
// Pure streaming (6 bytes per output element, nothing reused), so the design is about bytes in
// flight per SM. The default fast path is the register variant below (full occupancy at 32
// registers). The alternative fast path (MAS_SILU_IMPL=ring) is a persistent, warp-specialised TMA
// ring. The work is cut into tiles of (token, kSiluChunk columns); each CTA owns a contiguous range
// of tiles. Warp 0 is the producer: one lane streams the gate and up halves of each tile into an
// S-stage shared-memory ring with two bulk copies (cp.async.bulk, completion on the stage's `full`
// mbarrier). The other warps consume: wait on `full`, read 16-byte vectors from shared memory,
// compute, store 16-byte vectors to the output, and release the stage on its `empty` mbarrier
// (one arrival per consumer warp), which the producer waits on before refilling it. Every wait is
// bounded. A scalar path covers d % 8 != 0 and unaligned rows.
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
  int32_t stages;          // TMA ring
  int64_t tiles_per_cta;   // TMA ring
  int32_t* fault;
  const float* scale;      // quant variant: activation scale (device scalar)
};

// flashinfer compiles `val / (1.0f + __expf(-val))` with fast math, which makes the quotient the
// approximate divide: the numerator times the reciprocal of the divisor, where a divisor of 2^126 or
// more (gate below about -87.3) has a zero reciprocal. __fdividef is that divide, and it reproduces
// the reference's outputs there (-0), not the tiny values an IEEE quotient would give.
__device__ __forceinline__ float silu_f32(float v) { return __fdividef(v, 1.0f + __expf(-v)); }

constexpr int kSiluThreads = 256;            // scalar path
constexpr int kSiluConsumerWarps = 16;
constexpr int kSiluRingThreads = 32 * (1 + kSiluConsumerWarps);
constexpr int kSiluChunk = 4096;             // columns per tile: 8 KB of gate + 8 KB of up (bf16)

__host__ __device__ inline size_t silu_ring_smem_bytes(int stages, int elem_bytes) {
  return (size_t)stages * 2 * kSiluChunk * elem_bytes + (size_t)stages * 16;
}

template <typename T>
__global__ void __launch_bounds__(kSiluRingThreads) silu_mul_ring_kernel(const SiluArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int S = a.stages;
  constexpr int kStageBytes = 2 * kSiluChunk * (int)sizeof(T);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * kStageBytes);
  uint64_t* empty = full + S;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const int64_t cpr = (a.d + kSiluChunk - 1) / kSiluChunk;  // tiles per row
  const int64_t total = a.rows * cpr;
  const int64_t t0 = (int64_t)blockIdx.x * a.tiles_per_cta;
  const int n = (int)min(a.tiles_per_cta, total - t0);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kSiluConsumerWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  pdl_wait();

  int issued = 0;        // producer lane: tiles whose loads were issued
  bool gave_up = false;  // this thread's bounded wait ran out
  if (warp == 0) {
    // Producer. A failed wait (which means a copy or a consumer never finished) ends the stream.
    if (lane == 0) {
      const T* in = static_cast<const T*>(a.in);
      for (int k = 0; k < n; ++k) {
        const int s = k % S;
        if (k >= S && !mbar_wait_bounded(&empty[s], (uint32_t)((k / S) - 1) & 1u)) {
          atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
          gave_up = true;
          break;
        }
        issued = k + 1;
        const int64_t tile = t0 + k;
        const int64_t row = tile / cpr;
        const int c0 = (int)(tile - row * cpr) * kSiluChunk;
        const uint32_t bytes = (uint32_t)min(kSiluChunk, a.d - c0) * (uint32_t)sizeof(T);
        unsigned char* st = smem + (size_t)s * kStageBytes;
        const T* g = in + row * a.in_stride + c0;
        mbar_arrive_expect_tx(&full[s], 2 * bytes);
        bulk_load(st, g, bytes, &full[s]);
        bulk_load(st + kStageBytes / 2, g + a.d, bytes, &full[s]);
      }
    }
  } else {
    const int ct = tid - 32;  // consumer thread index
    T* out = static_cast<T*>(a.out);
    for (int k = 0; k < n; ++k) {
      const int s = k % S;
      // every lane waits (each needs the barrier's acquire); the warp gives up as one
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[s], (uint32_t)(k / S) & 1u))) {
        if (lane == 0) atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
        gave_up = true;
        break;
      }
      const int64_t tile = t0 + k;
      const int64_t row = tile / cpr;
      const int c0 = (int)(tile - row * cpr) * kSiluChunk;
      const int nv = min(kSiluChunk, a.d - c0) >> 3;
      const unsigned char* sg = smem + (size_t)s * kStageBytes;
      const unsigned char* su = sg + kStageBytes / 2;
      T* o = out + row * a.out_stride + c0;
      for (int v = ct; v < nv; v += 32 * kSiluConsumerWarps) {
        float gf[8], uf[8], y[8];
        unpack8<T>(*reinterpret_cast<const Vec16*>(sg + (size_t)v * 16), gf);
        unpack8<T>(*reinterpret_cast<const Vec16*>(su + (size_t)v * 16), uf);
#pragma unroll
        for (int e = 0; e < 8; ++e) y[e] = silu_f32(gf[e]) * uf[e];
        st_plain(o + (size_t)v * 8, pack8<T>(y));
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

// The fp32 quotient act / scale of FP8Linear's activation quantisation, without a divide
// instruction: q0 = act * r with r = 1/scale (rounded once per thread), then one remainder step of
// Markstein's FMA division (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): rem = fma(-scale, q0, act) is exact and
// fma(r, rem, q0) is the correctly rounded quotient. The step is applied where it can change the
// e4m3 result, |q0| in [2^-12, 512): below, e4m3 rounds to a zero of the right sign; above, it
// saturates. With this restriction the quotient equals the IEEE one on every bf16 and every fp16
// activation, checked exhaustively on the CPU for 20,000 scales. `fast` is false when scale or r is
// not a normal number; the IEEE divide is used then.
struct QuantDiv {
  float scale, r;
  float r_lo, r_hi;  // RN(r * (1 -+ 2^-20)): brackets for quant2_e4m3
  bool fast;
  __device__ __forceinline__ float operator()(float x) const {
    if (!fast) return __fdiv_rn(x, scale);
    const float q0 = __fmul_rn(x, r);
    const float q1 = __fmaf_rn(r, __fmaf_rn(-scale, q0, x), q0);
    const float a = fabsf(q0);
    return (a >= 0x1p-12f && a < 512.0f) ? q1 : q0;
  }
};

__device__ __forceinline__ QuantDiv make_quant_div(float s) {
  QuantDiv d;
  d.scale = s;
  d.r = __frcp_rn(s);
  d.r_lo = __fmul_rn(d.r, 1.0f - 0x1p-20f);
  d.r_hi = __fmul_rn(d.r, 1.0f + 0x1p-20f);
  d.fast = fabsf(s) >= 0x1p-126f && fabsf(s) <= 0x1.fffffep127f && fabsf(d.r) >= 0x1p-126f &&
           fabsf(d.r) <= 0x1.fffffep127f;
  return d;
}

// FP8Linear's activation quantisation of four silu outputs (already rounded to the activation type):
// (act / scale) in fp32, clamped to +-448 and rounded to nearest even e4m3 (satfinite does the
// clamp; NaN stays NaN, as with a clamp that propagates it).
//
// Two activations at a time, usually without forming the quotient: x * r_lo and x * r_hi bracket
// RN_f32(x / scale) (each carries at most three roundings of 2^-24 against the 2^-20 margin), and
// rounding to e4m3 is monotonic, so when both brackets round to the same code that code is the
// quotient's. Otherwise (a bracket straddles an e4m3 rounding boundary: about 1e-5 of inputs for a
// general scale, up to 0.3 % for a power-of-two scale, whose quotients can land on exact ties) the
// pair takes the remainder-corrected quotient. Checked on the CPU over every bf16 and fp16 input.
__device__ __forceinline__ uint16_t quant2_e4m3(float x0, float x1, const QuantDiv& div) {
  if (div.fast) {
    const float2 x = make_float2(x0, x1);
    const float2 lo2 = mul2_f32(x, make_float2(div.r_lo, div.r_lo));
    const float2 hi2 = mul2_f32(x, make_float2(div.r_hi, div.r_hi));
    const uint16_t lo = f2_to_e4m3x2(lo2.x, lo2.y);
    const uint16_t hi = f2_to_e4m3x2(hi2.x, hi2.y);
    if (lo == hi) return lo;
  }
  return f2_to_e4m3x2(div(x0), div(x1));
}

__device__ __forceinline__ uint32_t quant4_e4m3(const float* act, const QuantDiv& div) {
  return (uint32_t)quant2_e4m3(act[0], act[1], div) | ((uint32_t)quant2_e4m3(act[2], act[3], div) << 16);
}

// quant4_e4m3 for a scale whose reciprocal is a normal number (div.fast): the four codes of both
// brackets are compared at once; only when they differ does each pair take quant2_e4m3's path.
__device__ __forceinline__ uint32_t quant4_e4m3_fast(const float* act, const QuantDiv& div) {
  const float2 rl = make_float2(div.r_lo, div.r_lo), rh = make_float2(div.r_hi, div.r_hi);
  const float2 l01 = mul2_f32(make_float2(act[0], act[1]), rl), l23 = mul2_f32(make_float2(act[2], act[3]), rl);
  const float2 h01 = mul2_f32(make_float2(act[0], act[1]), rh), h23 = mul2_f32(make_float2(act[2], act[3]), rh);
  const uint32_t lo = (uint32_t)f2_to_e4m3x2(l01.x, l01.y) | ((uint32_t)f2_to_e4m3x2(l23.x, l23.y) << 16);
  const uint32_t hi = (uint32_t)f2_to_e4m3x2(h01.x, h01.y) | ((uint32_t)f2_to_e4m3x2(h23.x, h23.y) << 16);
  if (lo == hi) return lo;
  return quant4_e4m3(act, div);
}

// Register variant (the default fast path): one 16-byte gate/up pair per thread and row, 32
// registers, so 2048 threads per SM keep 64 KB of loads in flight; a 2-D grid of (256-vector column
// blocks, row groups), each thread walking the rows of its group. QUANT writes 8 e4m3 bytes per
// thread instead of 8 activations. NOALLOC loads gate/up with L1::no_allocate (the host picks it for
// launches whose data fit in about two L2s, plain read-only loads for those that stream from HBM).
template <typename T, bool QUANT, bool NOALLOC = false>
__global__ void __launch_bounds__(kSiluThreads, 8) silu_mul_vec_kernel(const SiluArgs a) {
  pdl_wait();
  const int nvec = a.d >> 3;
  const int v = blockIdx.x * kSiluThreads + threadIdx.x;
  QuantDiv div = {1.0f, 1.0f, 1.0f, 1.0f, true};
  if constexpr (QUANT) {
    // one reciprocal per CTA (the IEEE reciprocal is a multi-instruction sequence)
    __shared__ QuantDiv sdiv;
    if (threadIdx.x == 0) sdiv = make_quant_div(*a.scale);
    __syncthreads();
    div = sdiv;
  }
  if (v < nvec) {
    for (int64_t row = blockIdx.y; row < a.rows; row += gridDim.y) {
      const T* g = static_cast<const T*>(a.in) + row * a.in_stride + (size_t)v * 8;
      const Vec16 gv = NOALLOC ? ld_ro_noalloc(g) : ld_ro(g);
      const Vec16 uv = NOALLOC ? ld_ro_noalloc(g + a.d) : ld_ro(g + a.d);
      float gf[8], uf[8], y[8];
      unpack8<T>(gv, gf);
      unpack8<T>(uv, uf);
#pragma unroll
      for (int e = 0; e < 8; e += 2) {
        const float2 p = mul2_f32(make_float2(silu_f32(gf[e]), silu_f32(gf[e + 1])), make_float2(uf[e], uf[e + 1]));
        y[e] = p.x;
        y[e + 1] = p.y;
      }
      if constexpr (QUANT) {
        unpack8<T>(pack8<T>(y), y);  // the activation as the unfused op would have stored it
        uint2 q;
        if (div.fast) {
          q.x = quant4_e4m3_fast(y, div);
          q.y = quant4_e4m3_fast(y + 4, div);
        } else {
          q.x = quant4_e4m3(y, div);
          q.y = quant4_e4m3(y + 4, div);
        }
        *reinterpret_cast<uint2*>(static_cast<uint8_t*>(a.out) + row * a.out_stride + (size_t)v * 8) = q;
      } else {
        st_plain(static_cast<T*>(a.out) + row * a.out_stride + (size_t)v * 8, pack8<T>(y));
      }
    }
  }
  pdl_launch_dependents();
}

template <typename T, bool QUANT>
__global__ void __launch_bounds__(kSiluThreads) silu_mul_generic_kernel(const SiluArgs a) {
  pdl_wait();
  const QuantDiv div = make_quant_div(QUANT ? *a.scale : 1.0f);
  for (int64_t row = blockIdx.y; row < a.rows; row += gridDim.y) {
    const uint16_t* g = static_cast<const uint16_t*>(a.in) + row * a.in_stride;
    const uint16_t* u = g + a.d;
    for (int i = blockIdx.x * kSiluThreads + threadIdx.x; i < a.d; i += gridDim.x * kSiluThreads) {
      const uint16_t act = Elem<T>::from_f(silu_f32(Elem<T>::to_f(g[i])) * Elem<T>::to_f(u[i]));
      if constexpr (QUANT) {
        static_cast<uint8_t*>(a.out)[row * a.out_stride + i] =
            (uint8_t)(f2_to_e4m3x2(div(Elem<T>::to_f(act)), 0.f) & 0xffu);
      } else {
        static_cast<uint16_t*>(a.out)[row * a.out_stride + i] = act;
      }
    }
  }
  pdl_launch_dependents();
}

}  // namespace mas
