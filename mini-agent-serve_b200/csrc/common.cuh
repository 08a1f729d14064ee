// common.cuh -- device helpers shared by the per-token layer-op kernels (sm_100a).
//
// Bulk copies are the TMA engine's non-tensor form (cp.async.bulk): a contiguous run of bytes
// between global and shared memory, completion tracked by an mbarrier transaction count (loads) or
// a bulk async-group (stores). Every copy has exactly one destination CTA: this GPU's own.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/mas_b200.h"

namespace mas {

constexpr int kWarp = 32;
// A bounded wait gives up after this many nanoseconds of %globaltimer and reports
// MAS_STATUS_COPY_TIMEOUT. A bulk copy of a few tens of KB normally lands in a few microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
constexpr uint32_t kWaitMaxPolls = 1u << 28;      // hard cap on polls, independent of the timer

struct alignas(16) Vec16 {
  uint32_t a, b, c, d;
};

// ---------------------------------------------------------------------------------------------
// Element conversions. Activations are bf16 or fp16; the math is fp32 with one rounding (RNE).
// ---------------------------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float2 to_f2(uint32_t u) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
  }
  static __device__ __forceinline__ uint32_t from_f2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float to_f(uint16_t u) {
    return __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(&u));
  }
  static __device__ __forceinline__ uint16_t from_f(float f) {
    __nv_bfloat16 v = __float2bfloat16_rn(f);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};

template <>
struct Elem<__half> {
  static __device__ __forceinline__ float2 to_f2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2*>(&u));
  }
  static __device__ __forceinline__ uint32_t from_f2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static __device__ __forceinline__ float to_f(uint16_t u) {
    return __half2float(*reinterpret_cast<const __half*>(&u));
  }
  static __device__ __forceinline__ uint16_t from_f(float f) {
    __half v = __float2half_rn(f);
    return *reinterpret_cast<uint16_t*>(&v);
  }
};

// 8 packed 16-bit elements <-> 8 floats.
template <typename T>
__device__ __forceinline__ void unpack8(const Vec16& v, float (&f)[8]) {
  float2 p;
  p = Elem<T>::to_f2(v.a); f[0] = p.x; f[1] = p.y;
  p = Elem<T>::to_f2(v.b); f[2] = p.x; f[3] = p.y;
  p = Elem<T>::to_f2(v.c); f[4] = p.x; f[5] = p.y;
  p = Elem<T>::to_f2(v.d); f[6] = p.x; f[7] = p.y;
}

template <typename T>
__device__ __forceinline__ Vec16 pack8(const float (&f)[8]) {
  Vec16 v;
  v.a = Elem<T>::from_f2(f[0], f[1]);
  v.b = Elem<T>::from_f2(f[2], f[3]);
  v.c = Elem<T>::from_f2(f[4], f[5]);
  v.d = Elem<T>::from_f2(f[6], f[7]);
  return v;
}

// Two floats -> two e4m3 bytes (round to nearest even, saturating to +-448), PTX cvt on sm_89+.
// The first operand of the PTX instruction lands in the upper byte.
__device__ __forceinline__ uint16_t f2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two fp32 values in one instruction (sm_100's packed f32x2 arithmetic): each lane is an ordinary
// IEEE multiply rounded to nearest even, so the results equal two scalar multiplies bit for bit;
// the pair costs one issue slot instead of two.
__device__ __forceinline__ float2 mul2_f32(float2 a, float2 b) {
  float2 c;
  asm("{\n\t.reg .b64 ra, rb, rc;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rc, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rc;\n\t}"
      : "=f"(c.x), "=f"(c.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return c;
}

// a * b + c on two fp32 pairs, one rounding per lane (two scalar fmas, one issue slot).
__device__ __forceinline__ float2 fma2_f32(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\t"
      "mov.b64 rb, {%4, %5};\n\t"
      "mov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

// ---------------------------------------------------------------------------------------------
// Global memory access.
// ---------------------------------------------------------------------------------------------
// Read-only 16-byte load through the non-coherent path, for data no kernel writes while this one
// runs (inputs read once, weights, cos/sin rows). Without an L1 hint: L1::no_allocate on the streaming
// reads of SiLU-mul measured 3 % slower (233.6 against 226.6 us for an [8192, 65536] input).
__device__ __forceinline__ Vec16 ld_ro(const void* p) {
  Vec16 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.a), "=r"(v.b), "=r"(v.c), "=r"(v.d)
               : "l"(p));
  return v;
}
// Read-only 16-byte load that allocates no L1 line (SiLU-mul's loads when its data may partly come
// from L2: a 512-token step of an 88-layer chain 3.27 ms against 3.73 with ld_ro).
__device__ __forceinline__ Vec16 ld_ro_noalloc(const void* p) {
  Vec16 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.a), "=r"(v.b), "=r"(v.c), "=r"(v.d)
               : "l"(p));
  return v;
}
// Plain coherent 16-byte load (data this kernel also writes).
__device__ __forceinline__ Vec16 ld_plain(const void* p) {
  Vec16 v;
  asm volatile("ld.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.a), "=r"(v.b), "=r"(v.c), "=r"(v.d)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_plain(void* p, const Vec16& v) {
  asm volatile("st.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.a), "r"(v.b), "r"(v.c),
               "r"(v.d)
               : "memory");
}

// ---------------------------------------------------------------------------------------------
// Programmatic dependent launch. Both are no-ops when the grid was not launched with the
// programmatic-serialization attribute.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" :::);
}

// ---------------------------------------------------------------------------------------------
// Shared memory, mbarriers and bulk copies.
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
// Makes the initialised barriers visible to the async proxy (the TMA engine).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
// Raises the expected transaction bytes of the barrier's current phase without arriving on it.
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Waits for the phase with the given parity to complete; false if the time limit ran out first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  for (uint32_t polls = 1; polls < kWaitMaxPolls; ++polls) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((polls & 255u) == 0u && global_timer_ns() - t0 > limit_ns) return false;
  }
  return false;
}

// Before a ring kernel's CTA exits after a wait gave up: waits (bounded) for the latest phase of
// every stage whose loads were issued, so no bulk copy is still writing into this CTA's shared
// memory when it is released. `issued` loads went to stages k % stages in order, and a barrier's
// phases complete in order, so the latest phase of each stage covers the earlier ones.
__device__ __forceinline__ void drain_ring(uint64_t* full, int stages, int issued) {
  for (int s = 0; s < stages && s < issued; ++s) {
    const int k = s + ((issued - 1 - s) / stages) * stages;  // the last load into stage s
    (void)mbar_wait_bounded(&full[s], (uint32_t)(k / stages) & 1u);
  }
}

// Global -> shared bulk copy, completion counted on `bar` (bytes: multiple of 16, both addresses
// 16-byte aligned). The destination is this CTA's own shared memory.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
// Shared -> global bulk copy, tracked by the issuing thread's bulk async-groups.
__device__ __forceinline__ void bulk_store(void* gmem_dst, const void* smem_src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gmem_dst),
               "r"(smem_u32(smem_src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Blocks until at most N of this thread's bulk groups still have to READ their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Blocks until every bulk group of this thread has completed (its writes are performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory accesses before later async-proxy accesses.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void flag_status(int32_t* status, int32_t bit) {
  if (status != nullptr) atomicOr(status, bit);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = kWarp / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

}  // namespace mas
