// mas_b200.cu -- the C ABI (include/mas_b200.h): argument checks, path choice, launch shapes.
//
// One translation unit holds every kernel, so the library is a single fatbin for sm_100a and needs
// no relocatable device code. Entry points never allocate or synchronise; the only per-process
// state is the per-device set-up of mas_prepare_device (shared-memory opt-in, SM count, the address
// of the fault word), done once per device under a lock.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.cuh"
#include "embed.cuh"
#include "norm.cuh"
#include "rope.cuh"
#include "silu.cuh"

namespace mas {

// Library fault word: bulk-copy wait timeouts land here.
__device__ int32_t g_fault_word;
// Library status word: the data-error bits (MAS_STATUS_*) of calls made without a status word of
// their own. One per device (each device's copy of the module has its own).
__device__ int32_t g_status_word;

namespace {

constexpr int kMaxDevices = 64;
constexpr size_t kMaxSmemPerCta = 227 * 1024;
// Shared memory the TMA rings may use per SM: the SM has 228 KB, less 1 KB reserved per resident CTA.
constexpr size_t kRingBytesPerSm = 216 * 1024;

struct DeviceState {
  std::once_flag once;
  cudaError_t err = cudaSuccess;
  int sm_count = 0;
  int l2_bytes = 0;
  int32_t* fault = nullptr;
  int32_t* status = nullptr;  // this device's g_status_word
};
DeviceState g_dev[kMaxDevices];

// Optional integer override from the environment (tuning knobs, read once per process).
int env_int(const char* name, int fallback) {
  const char* v = std::getenv(name);
  if (v == nullptr || *v == '\0') return fallback;
  return std::atoi(v);
}

// Optional choice between two fast-path designs of a kernel ("ring" or another name), read once.
bool env_is(const char* name, const char* value) {
  const char* v = std::getenv(name);
  return v != nullptr && std::strcmp(v, value) == 0;
}

template <typename K>
cudaError_t opt_in_smem(K kernel) {
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)kMaxSmemPerCta);
}

template <typename T, bool Q>
cudaError_t opt_in_norm() {
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 1, Q>);
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 2, Q>);
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 3, Q>);
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 4, Q>);
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 5, Q>);
  if (e == cudaSuccess) e = opt_in_smem(norm_tma_kernel<T, 6, Q>);
  return e;
}

template <typename T, bool Q>
cudaError_t opt_in_norm_row() {
  cudaError_t e = opt_in_smem(norm_row_kernel<T, Q, 4>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_kernel<T, Q, 8>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_kernel<T, Q, 12>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_kernel<T, Q, 16>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_kernel<T, Q, 4>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_kernel<T, Q, 8>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_kernel<T, Q, 12>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_kernel<T, Q, 16>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 4>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 6>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 8>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 12>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 6, 256>);
  if (e == cudaSuccess) e = opt_in_smem(norm_row_keep_kernel<T, Q, 3, 512>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_keep_kernel<T, Q, 4, 128>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_keep_kernel<T, Q, 4, 160>);
  if (e == cudaSuccess) e = opt_in_smem(norm_loop_keep_kernel<T, Q, 4, 192>);
  return e;
}

template <typename T>
cudaError_t opt_in_rope_ring() {
  cudaError_t e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int32_t, true, false>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int32_t, false, false>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int64_t, true, false>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int64_t, false, false>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int32_t, true, true>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int32_t, false, true>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(rope_ring_kernel<T, int64_t, true, true>)) != cudaSuccess) return e;
  return opt_in_smem(rope_ring_kernel<T, int64_t, false, true>);
}

cudaError_t prepare_current(DeviceState& st, int device) {
  cudaError_t e = cudaDeviceGetAttribute(&st.sm_count, cudaDevAttrMultiProcessorCount, device);
  if (e != cudaSuccess) return e;
  if ((e = cudaDeviceGetAttribute(&st.l2_bytes, cudaDevAttrL2CacheSize, device)) != cudaSuccess) return e;
  if ((e = opt_in_norm<__nv_bfloat16, false>()) != cudaSuccess) return e;
  if ((e = opt_in_norm<__nv_bfloat16, true>()) != cudaSuccess) return e;
  if ((e = opt_in_norm<__half, false>()) != cudaSuccess) return e;
  if ((e = opt_in_norm<__half, true>()) != cudaSuccess) return e;
  if ((e = opt_in_norm_row<__nv_bfloat16, false>()) != cudaSuccess) return e;
  if ((e = opt_in_norm_row<__nv_bfloat16, true>()) != cudaSuccess) return e;
  if ((e = opt_in_norm_row<__half, false>()) != cudaSuccess) return e;
  if ((e = opt_in_norm_row<__half, true>()) != cudaSuccess) return e;
  if ((e = opt_in_smem(silu_mul_ring_kernel<__nv_bfloat16>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(silu_mul_ring_kernel<__half>)) != cudaSuccess) return e;
  if ((e = opt_in_rope_ring<__nv_bfloat16>()) != cudaSuccess) return e;
  if ((e = opt_in_rope_ring<__half>()) != cudaSuccess) return e;
  if ((e = opt_in_smem(embed_tma_kernel<int32_t>)) != cudaSuccess) return e;
  if ((e = opt_in_smem(embed_tma_kernel<int64_t>)) != cudaSuccess) return e;
  void* fault = nullptr;
  if ((e = cudaGetSymbolAddress(&fault, g_fault_word)) != cudaSuccess) return e;
  st.fault = static_cast<int32_t*>(fault);
  void* status = nullptr;
  if ((e = cudaGetSymbolAddress(&status, g_status_word)) != cudaSuccess) return e;
  st.status = static_cast<int32_t*>(status);
  return cudaSuccess;
}

// Runs the one-time set-up of `device` with that device current, restoring the caller's device.
int prepare(int device) {
  if (device < 0 || device >= kMaxDevices) return MAS_ERR_INVALID_ARGUMENT;
  DeviceState& st = g_dev[device];
  std::call_once(st.once, [&] {
    int prev = -1;
    cudaError_t e = cudaGetDevice(&prev);
    if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
    if (e == cudaSuccess) e = prepare_current(st, device);
    if (prev >= 0 && prev != device) (void)cudaSetDevice(prev);
    st.err = e;
  });
  return st.err == cudaSuccess ? MAS_OK : (int)st.err;
}

// Current device, prepared. Returns a status code; on success *out points at its state.
int current_device(DeviceState** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) {
    (void)cudaGetLastError();
    return MAS_ERR_NO_DEVICE;
  }
  const int rc = prepare(dev);
  if (rc != MAS_OK) return rc;
  *out = &g_dev[dev];
  return MAS_OK;
}

template <typename... KArgs, typename... Args>
int launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, int pdl,
           Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
  return e == cudaSuccess ? MAS_OK : (int)e;
}

// Resident CTAs per SM of `kernel` at this block size and dynamic shared memory, cached per
// (device, kernel, block, smem) because the occupancy query is not free.
struct OccKey {
  int dev;
  const void* fn;
  int nt;
  size_t smem;
};
std::mutex g_occ_mu;
OccKey g_occ_key[256];
int g_occ_val[256];
int g_occ_n = 0;

int resident_ctas(const void* fn, int nt, size_t smem) {
  int dev = 0;
  (void)cudaGetDevice(&dev);
  {
    std::lock_guard<std::mutex> lk(g_occ_mu);
    for (int i = 0; i < g_occ_n; ++i)
      if (g_occ_key[i].dev == dev && g_occ_key[i].fn == fn && g_occ_key[i].nt == nt &&
          g_occ_key[i].smem == smem)
        return g_occ_val[i];
  }
  int blocks = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, nt, smem) != cudaSuccess) {
    (void)cudaGetLastError();
    blocks = 1;
  }
  if (blocks < 1) blocks = 1;
  std::lock_guard<std::mutex> lk(g_occ_mu);
  if (g_occ_n < 256) {
    g_occ_key[g_occ_n] = OccKey{dev, fn, nt, smem};
    g_occ_val[g_occ_n] = blocks;
    ++g_occ_n;
  }
  return blocks;
}

template <typename T, bool Q>
const void* norm_tma_fn(int vpt) {
  switch (vpt) {
    case 1: return (const void*)norm_tma_kernel<T, 1, Q>;
    case 2: return (const void*)norm_tma_kernel<T, 2, Q>;
    case 3: return (const void*)norm_tma_kernel<T, 3, Q>;
    case 4: return (const void*)norm_tma_kernel<T, 4, Q>;
    case 5: return (const void*)norm_tma_kernel<T, 5, Q>;
    case 6: return (const void*)norm_tma_kernel<T, 6, Q>;
    default: return nullptr;
  }
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ------------------------------------------------------------------------------------------
// Fused add RMSNorm (both variants).
// ------------------------------------------------------------------------------------------
template <typename T, bool Q>
int launch_norm_tma(NormArgs a, int vpt, int nt, size_t smem, int grid, void* stream, int pdl) {
  switch (vpt) {
    case 1: return launch(norm_tma_kernel<T, 1, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    case 2: return launch(norm_tma_kernel<T, 2, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    case 3: return launch(norm_tma_kernel<T, 3, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    case 4: return launch(norm_tma_kernel<T, 4, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    case 5: return launch(norm_tma_kernel<T, 5, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    case 6: return launch(norm_tma_kernel<T, 6, Q>, dim3(grid), dim3(nt), smem, stream, pdl, a);
    default: return MAS_ERR_UNSUPPORTED_SHAPE;
  }
}

template <typename T, bool Q>
int run_norm(NormArgs a, const DeviceState& st, bool fast_ok, void* stream, int pdl) {
  const int H = a.H;
  static const bool use_ring = env_is("MAS_NORM_IMPL", "ring");
  static const bool use_row = env_is("MAS_NORM_IMPL", "row");
  static const bool use_loop = env_is("MAS_NORM_IMPL", "loop");
  static const bool use_rowreg = env_is("MAS_NORM_IMPL", "rowreg");
  static const bool use_loopreg = env_is("MAS_NORM_IMPL", "loopreg");
  const bool loopreg_default = !use_ring && !use_row && !use_loop && !use_rowreg;
  if (fast_ok && H % 8 == 0 && (use_loopreg || loopreg_default) && H / 8 > 3 * 128 && H / 8 <= 4 * 192) {
    // Default for 3072 < H <= 6144: the register-resident persistent loop (norm_loop_keep_kernel),
    // one row of nt = H/32 threads (rounded up to a warp: 128, 160 or 192) per CTA and iteration, two
    // stages. Configuration 1 (H = 5120, 4096 rows), against norm_loop_kernel's 26.8-27.0 us (bf16)
    // and 25.8 us (e4m3 out): bf16 26.4-26.6 us at four CTAs per SM (within 1 % of every other
    // stage / CTA count); e4m3 out 23.1-23.4 us at three CTAs per SM, against 25.0 at four and 27-28
    // at two (three stages: 23.7-23.8).
    static const int env_stages = env_int("MAS_NORM_STAGES", 0);
    static const int env_ctas = env_int("MAS_NORM_CTAS_PER_SM", 0);
    const int nt = (int)ceil_div(ceil_div(H / 8, 4), 32) * 32;
    const int stages = std::max(2, std::min(8, env_stages > 0 ? env_stages : 2));
    const size_t smem = norm_loop_keep_smem_bytes(H, stages, nt, (int)sizeof(T));
    if (smem <= kMaxSmemPerCta) {
      const void* fn = nt == 128 ? (const void*)norm_loop_keep_kernel<T, Q, 4, 128>
                     : nt == 160 ? (const void*)norm_loop_keep_kernel<T, Q, 4, 160>
                                 : (const void*)norm_loop_keep_kernel<T, Q, 4, 192>;
      int ctas = resident_ctas(fn, nt, smem);
      if (env_ctas > 0) ctas = std::min(ctas, env_ctas);
      else if (Q) ctas = std::min(ctas, 3);
      const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(a.rows, (int64_t)st.sm_count * std::max(1, ctas)));
      a.stages = stages;
      const dim3 g((unsigned)grid), b(nt);
      if (nt == 128) return launch(norm_loop_keep_kernel<T, Q, 4, 128>, g, b, smem, stream, pdl, a);
      if (nt == 160) return launch(norm_loop_keep_kernel<T, Q, 4, 160>, g, b, smem, stream, pdl, a);
      return launch(norm_loop_keep_kernel<T, Q, 4, 192>, g, b, smem, stream, pdl, a);
    }
  }
  // Default up to H = 3072 (and for any H up to 6144 that the loop above does not take): the
  // persistent loop (at H = 5120 it measured 26.3 us against 29.5 for the row-block grid); the
  // register-resident row kernel above H = 6144 (below).
  if (fast_ok && H % 8 == 0 &&
      (use_loop || (!use_ring && !use_row && !use_rowreg && H <= 6144))) {
    // Persistent row-group loop (norm_loop_kernel): S-stage ring, every thread a consumer. By
    // default at most 4 vectors per thread (threads per row = H/32, rounded up to a warp), CTAs of at
    // least 128 threads (one row each from 128 threads per row up) and two stages: at H = 5120, four
    // CTAs of one row per SM (e4m3 out: 25.8 us against 26.5 for two CTAs of two rows).
    static const int env_tpr = env_int("MAS_NORM_TPR", 0);
    static const int env_cta = env_int("MAS_NORM_CTA_THREADS", 0);
    static const int env_stages = env_int("MAS_NORM_STAGES", 0);
    static const int env_ctas = env_int("MAS_NORM_CTAS_PER_SM", 0);
    int tpr = (int)ceil_div(ceil_div(H / 8, 4), 32) * 32;
    if (env_tpr > 0) tpr = env_tpr;
    tpr = std::max(32, std::min(tpr, kNormRowMaxThreads)) / 32 * 32;
    int cta = env_cta > 0 ? env_cta : std::max(tpr, 128 / tpr * tpr);
    cta = std::max(tpr, std::min(cta, kNormRowMaxThreads)) / tpr * tpr;
    const int rpc = cta / tpr;
    const int vpt = (int)ceil_div(H / 8, tpr);
    const int stages = std::max(2, std::min(8, env_stages > 0 ? env_stages : 2));
    const size_t smem = norm_loop_smem_bytes(H, rpc, stages, (int)sizeof(T));
    if (smem <= kMaxSmemPerCta && vpt <= 16) {
      const void* fn = vpt <= 4 ? (const void*)norm_loop_kernel<T, Q, 4>
                     : vpt <= 8 ? (const void*)norm_loop_kernel<T, Q, 8>
                     : vpt <= 12 ? (const void*)norm_loop_kernel<T, Q, 12>
                                 : (const void*)norm_loop_kernel<T, Q, 16>;
      int ctas = resident_ctas(fn, cta, smem);
      if (env_ctas > 0) ctas = std::min(ctas, env_ctas);
      const int64_t ngroups = ceil_div(a.rows, rpc);
      const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(ngroups, (int64_t)st.sm_count * std::max(1, ctas)));
      a.stages = stages;
      const dim3 g((unsigned)grid), b(cta);
      if (vpt <= 4) return launch(norm_loop_kernel<T, Q, 4>, g, b, smem, stream, pdl, a, tpr, rpc);
      if (vpt <= 8) return launch(norm_loop_kernel<T, Q, 8>, g, b, smem, stream, pdl, a, tpr, rpc);
      if (vpt <= 12) return launch(norm_loop_kernel<T, Q, 12>, g, b, smem, stream, pdl, a, tpr, rpc);
      return launch(norm_loop_kernel<T, Q, 16>, g, b, smem, stream, pdl, a, tpr, rpc);
    }
  }
  // Above H = 6144 (up to 12288) the register-resident row kernel: one row of 128 threads per CTA,
  // of 256 threads when a step has at most eight rows per SM, of 512 at most one. At H = 12288 in
  // isolation: 4352 rows 65.6-65.7 us (the row kernel below 66.6-67.2, flashinfer 65.9-66.0), e4m3
  // out 57.5-57.6 us (60.0-60.3, flashinfer 70.1-70.8). In a CUDA graph (row kernel / flashinfer in
  // brackets): 64 rows 2.43 us (2.89 / 2.70), 256 rows 3.56 (4.5 / 4.55), 512 rows 6.3 (7.6 / 7.6),
  // 1024 rows 11.1 (11.9 / 12.8); from about 2048 rows 128 threads are as fast or faster.
  const bool rowreg_default = !use_ring && !use_row && !use_loop && H > 6144;
  if (fast_ok && H % 8 == 0 && (use_rowreg || rowreg_default) && H / 8 <= 12 * 128 && a.rows <= INT32_MAX) {
    const int nv = H / 8;
    static const int env_nt = env_int("MAS_NORM_KEEP_THREADS", 0);
    int nt = a.rows <= (int64_t)st.sm_count ? 512 : a.rows <= 8 * (int64_t)st.sm_count ? 256 : 128;
    if (env_nt == 128 || env_nt == 256 || env_nt == 512) nt = env_nt;
    const size_t smem = 2 * (size_t)H * sizeof(T) + 16 + (size_t)(nt / 32) * sizeof(float);
    const dim3 g((unsigned)a.rows), b(nt);
    if (nt == 512 && nv <= 3 * 512) return launch(norm_row_keep_kernel<T, Q, 3, 512>, g, b, smem, stream, pdl, a);
    if (nt == 256 && nv <= 6 * 256) return launch(norm_row_keep_kernel<T, Q, 6, 256>, g, b, smem, stream, pdl, a);
    if (nv <= 4 * 128) return launch(norm_row_keep_kernel<T, Q, 4>, dim3((unsigned)a.rows), dim3(128), smem, stream, pdl, a);
    if (nv <= 6 * 128) return launch(norm_row_keep_kernel<T, Q, 6>, dim3((unsigned)a.rows), dim3(128), smem, stream, pdl, a);
    if (nv <= 8 * 128) return launch(norm_row_keep_kernel<T, Q, 8>, dim3((unsigned)a.rows), dim3(128), smem, stream, pdl, a);
    return launch(norm_row_keep_kernel<T, Q, 12>, dim3((unsigned)a.rows), dim3(128), smem, stream, pdl, a);
  }
  if (fast_ok && H % 8 == 0 && !use_ring) {
    // Row-block CTAs (H above 12288, or MAS_NORM_IMPL=row): threads per row grow with H (32 ... 256),
    // 128 or 256 threads per CTA. A step with few rows (at most about one or three per SM) has too
    // few CTAs to hide a row's latency, so its rows get four or two times the threads (at H = 12288
    // in a CUDA graph: 64 rows 3.7 -> 2.8 us, 256 rows 4.8 -> 4.3 us).
    static const int env_tpr = env_int("MAS_NORM_TPR", 0);
    static const int env_cta = env_int("MAS_NORM_CTA_THREADS", 0);
    int tpr = H <= 3072 ? 32 : H <= 6144 ? 64 : H <= 16384 ? 128 : 256;
    if (a.rows <= (int64_t)st.sm_count) tpr *= 4;
    else if (a.rows <= 3 * (int64_t)st.sm_count) tpr *= 2;
    if (env_tpr > 0) tpr = env_tpr;
    int cta = env_cta > 0 ? env_cta : std::max(128, tpr);
    tpr = std::max(32, std::min(tpr, kNormRowMaxThreads)) / 32 * 32;
    cta = std::max(tpr, std::min(cta, kNormRowMaxThreads)) / tpr * tpr;
    const int rpc = cta / tpr;
    const size_t smem = norm_row_smem_bytes(H, rpc, (int)sizeof(T));
    const int vpt = (int)ceil_div(H / 8, tpr);
    if (smem <= kMaxSmemPerCta && vpt <= 16) {
      const int64_t grid = ceil_div(a.rows, rpc);
      const dim3 g((unsigned)grid), b(cta);
      if (grid <= INT32_MAX) {
        if (vpt <= 4) return launch(norm_row_kernel<T, Q, 4>, g, b, smem, stream, pdl, a, tpr, rpc);
        if (vpt <= 8) return launch(norm_row_kernel<T, Q, 8>, g, b, smem, stream, pdl, a, tpr, rpc);
        if (vpt <= 12) return launch(norm_row_kernel<T, Q, 12>, g, b, smem, stream, pdl, a, tpr, rpc);
        return launch(norm_row_kernel<T, Q, 16>, g, b, smem, stream, pdl, a, tpr, rpc);
      }
    }
  }
  if (fast_ok && H % 8 == 0) {
    const int nv = H / 8;
    static const int env_groups = env_int("MAS_NORM_GROUPS", 0);
    const int groups = std::max(1, std::min(kNormMaxGroups, env_groups > 0 ? env_groups : 2));
    const int vpt = (int)ceil_div(nv, kNormMaxConsumers / groups);
    const int gsize = (int)ceil_div(ceil_div(nv, vpt), 32) * 32;
    const int nt = 32 + groups * gsize;  // producer warp + consumer groups
    a.groups = groups;
    const size_t stage = 2ull * (size_t)H * sizeof(T);
    static const int env_ctas = env_int("MAS_NORM_CTAS_PER_SM", 0);
    static const int env_stages = env_int("MAS_NORM_STAGES", 0);
    // Ring depth first (4 stages), then as many CTAs per SM as the ring budget, the thread limit and
    // the occupancy (registers) allow; budget left over deepens the ring (up to 8 stages).
    // Consumer group g takes rows g, g + G, ... and stage s serves rows s, s + S, ...; with S a
    // multiple of G the previous user of a stage is the same group, which keeps every parity wait
    // on the stage's barriers within one phase (norm_tma_kernel relies on it). So S is rounded down
    // to a multiple of G (G <= 4 <= 8 leaves at least G stages).
    const auto multiple_of_groups = [groups](int st_) { return std::max(groups, st_ / groups * groups); };
    const void* fn = norm_tma_fn<T, Q>(vpt);
    int stages = env_stages > 0 ? env_stages : 4;
    if ((size_t)stages * stage > kRingBytesPerSm) stages = (int)std::max<size_t>(2, kRingBytesPerSm / stage);
    stages = multiple_of_groups(std::max(2, std::min(8, stages)));
    size_t smem = norm_tma_smem_bytes(H, stages, (int)sizeof(T));
    if (fn != nullptr && smem <= kMaxSmemPerCta) {
      int ctas = env_ctas > 0 ? env_ctas : (int)std::max<size_t>(1, kRingBytesPerSm / ((size_t)stages * stage));
      ctas = std::max(1, std::min({ctas, 2048 / nt, resident_ctas(fn, nt, smem)}));
      if (env_stages <= 0) {
        const int deeper = multiple_of_groups((int)std::min<size_t>(8, kRingBytesPerSm / ((size_t)ctas * stage)));
        if (deeper > stages && norm_tma_smem_bytes(H, deeper, (int)sizeof(T)) <= kMaxSmemPerCta) {
          stages = deeper;
          smem = norm_tma_smem_bytes(H, stages, (int)sizeof(T));
          ctas = std::max(1, std::min(ctas, resident_ctas(fn, nt, smem)));  // the grid must stay resident
        }
      }
      int64_t grid = std::min<int64_t>(a.rows, (int64_t)st.sm_count * ctas);
      a.rows_per_cta = (int32_t)ceil_div(a.rows, grid);
      grid = ceil_div(a.rows, a.rows_per_cta);
      a.stages = stages;
      return launch_norm_tma<T, Q>(a, vpt, nt, smem, (int)grid, stream, pdl);
    }
  }
  const int64_t grid = std::min<int64_t>(a.rows, 1 << 20);
  return launch(norm_generic_kernel<T, Q>, dim3((unsigned)grid), dim3(256), 0, stream, pdl, a);
}

int check_act_dtype(int dtype) {
  return (dtype == MAS_DTYPE_BF16 || dtype == MAS_DTYPE_FP16) ? MAS_OK : MAS_ERR_UNSUPPORTED_DTYPE;
}

// Launches the token-staged rope ring (APPEND: fused with the paged KV append) when its shared
// memory fits; returns kNotLaunched otherwise.
constexpr int kNotLaunched = -1000;  // neither a MAS_ERR_* code nor a cudaError_t

template <bool APPEND>
int launch_rope_ring_t(RopeRingArgs r, bool bf, bool i64, bool neox, DeviceState* st, void* stream,
                       int enable_pdl) {
  const uint32_t stage = rope_stage_bytes(r.Hq, r.Hkv, r.D, r.rd, 2, APPEND);
  static const int env_stages = env_int("MAS_ROPE_STAGES", 0);
  static const int env_warps = env_int("MAS_ROPE_CONSUMER_WARPS", 0);
  static const int env_ctas = env_int("MAS_ROPE_CTAS_PER_SM", 0);
  // Two stages for small per-token stages (configuration 3: 10.75 KB), three for large ones (the chain
  // shape: 27 KB); measured best of 2-4 stages x 8-16 consumer warps at both shapes.
  const int stages = std::max(2, std::min(16, env_stages > 0 ? env_stages : (stage <= 16384 ? 2 : 3)));
  const int threads = 32 * (1 + std::max(1, std::min(kRopeMaxConsumerWarps, env_warps > 0 ? env_warps : kRopeConsumerWarps)));
  // The grid has at least one CTA per SM, so a CTA holds the positions of at most ceil(T / SMs)
  // tokens; with that bound the shared memory per CTA is known before the CTA count is chosen.
  // (rounded up to 64 tokens, which keeps the occupancy cache small across batch sizes).
  const int tok_cap = (int)std::min<int64_t>(kRopeMaxTokensPerCta, ceil_div(ceil_div(r.T, (int64_t)st->sm_count), 64) * 64);
  const size_t per_cta = rope_ring_smem_bytes(stage, stages, tok_cap, APPEND);
  if (per_cta > kMaxSmemPerCta) return kNotLaunched;
  const void* fn = bf ? (i64 ? (neox ? (const void*)rope_ring_kernel<__nv_bfloat16, int64_t, true, APPEND>
                                     : (const void*)rope_ring_kernel<__nv_bfloat16, int64_t, false, APPEND>)
                             : (neox ? (const void*)rope_ring_kernel<__nv_bfloat16, int32_t, true, APPEND>
                                     : (const void*)rope_ring_kernel<__nv_bfloat16, int32_t, false, APPEND>))
                      : (i64 ? (neox ? (const void*)rope_ring_kernel<__half, int64_t, true, APPEND>
                                     : (const void*)rope_ring_kernel<__half, int64_t, false, APPEND>)
                             : (neox ? (const void*)rope_ring_kernel<__half, int32_t, true, APPEND>
                                     : (const void*)rope_ring_kernel<__half, int32_t, false, APPEND>));
  // As many CTAs per SM as shared memory, registers and threads allow: the consumer side, not the
  // depth of one ring, limits a CTA (measured at the chain shape: 2-3 CTAs of 3 stages beat one of 4-8).
  int ctas = std::max(1, resident_ctas(fn, threads, per_cta));
  if (env_ctas > 0) ctas = std::min(ctas, env_ctas);
  int64_t grid = std::max<int64_t>((int64_t)st->sm_count * ctas, ceil_div(r.T, kRopeMaxTokensPerCta));
  grid = std::min<int64_t>(grid, r.T);
  r.tokens_per_cta = (int32_t)ceil_div(r.T, grid);
  grid = ceil_div(r.T, r.tokens_per_cta);
  r.stages = stages;
  static const int env_early = env_int("MAS_ROPE_EARLY_DEPENDENTS", 0);
  r.early_dependents = env_early > 0 ? 1 : 0;
  static const int env_prefetch = env_int("MAS_ROPE_PREFETCH_QK", 1);
  r.prefetch_qk = env_prefetch > 0 ? 1 : 0;
  const size_t smem = rope_ring_smem_bytes(stage, stages, r.tokens_per_cta, APPEND);
  const dim3 g((unsigned)grid), b(threads);
  if (bf) {
    if (i64) return neox ? launch(rope_ring_kernel<__nv_bfloat16, int64_t, true, APPEND>, g, b, smem, stream, enable_pdl, r)
                         : launch(rope_ring_kernel<__nv_bfloat16, int64_t, false, APPEND>, g, b, smem, stream, enable_pdl, r);
    return neox ? launch(rope_ring_kernel<__nv_bfloat16, int32_t, true, APPEND>, g, b, smem, stream, enable_pdl, r)
                : launch(rope_ring_kernel<__nv_bfloat16, int32_t, false, APPEND>, g, b, smem, stream, enable_pdl, r);
  }
  if (i64) return neox ? launch(rope_ring_kernel<__half, int64_t, true, APPEND>, g, b, smem, stream, enable_pdl, r)
                       : launch(rope_ring_kernel<__half, int64_t, false, APPEND>, g, b, smem, stream, enable_pdl, r);
  return neox ? launch(rope_ring_kernel<__half, int32_t, true, APPEND>, g, b, smem, stream, enable_pdl, r)
              : launch(rope_ring_kernel<__half, int32_t, false, APPEND>, g, b, smem, stream, enable_pdl, r);
}

int launch_rope_ring(const RopeRingArgs& r, bool append, bool bf, bool i64, bool neox, DeviceState* st,
                     void* stream, int enable_pdl) {
  return append ? launch_rope_ring_t<true>(r, bf, i64, neox, st, stream, enable_pdl)
                : launch_rope_ring_t<false>(r, bf, i64, neox, st, stream, enable_pdl);
}

// Whether the fused ring can also append: v heads contiguous within a token, 16-byte aligned v rows
// and cache rows.
bool append_ring_ok(const AppendArgs& a, int64_t head_size) {
  return (a.Hkv == 0 || (a.vsh == head_size && aligned(a.v, 16) && a.vsn % 8 == 0)) &&
         aligned(a.kv.k_cache, 16) && aligned(a.kv.v_cache, 16) && a.kv.stride_page % 8 == 0 &&
         a.kv.stride_entry % 8 == 0 && a.kv.stride_head % 8 == 0;
}

int launch_append(const AppendArgs& args, bool bf, bool i64, DeviceState* st, void* stream, int enable_pdl) {
  AppendArgs a = args;
  if (a.status == nullptr) a.status = st->status;
  if (a.T == 0 || a.Hkv == 0) return MAS_OK;
  const bool vec = a.D % 8 == 0 && aligned(a.k, 16) && aligned(a.v, 16) && a.ksn % 8 == 0 && a.ksh % 8 == 0 &&
                   a.vsn % 8 == 0 && a.vsh % 8 == 0 && aligned(a.kv.k_cache, 16) && aligned(a.kv.v_cache, 16) &&
                   a.kv.stride_page % 8 == 0 && a.kv.stride_entry % 8 == 0 && a.kv.stride_head % 8 == 0;
  const dim3 blk(kAppendThreads);
  if (vec) {
    // a warp per token, grid-strided over at most 8 CTAs of 8 warps per SM
    const int64_t warps_per_cta = kAppendThreads / 32;
    const dim3 grid((unsigned)std::min<int64_t>(ceil_div(a.T, warps_per_cta), (int64_t)st->sm_count * 8));
    if (bf) return i64 ? launch(append_kv_vec_kernel<__nv_bfloat16, int64_t>, grid, blk, 0, stream, enable_pdl, a)
                       : launch(append_kv_vec_kernel<__nv_bfloat16, int32_t>, grid, blk, 0, stream, enable_pdl, a);
    return i64 ? launch(append_kv_vec_kernel<__half, int64_t>, grid, blk, 0, stream, enable_pdl, a)
               : launch(append_kv_vec_kernel<__half, int32_t>, grid, blk, 0, stream, enable_pdl, a);
  }
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(a.T * a.Hkv * a.D, kAppendThreads), 1 << 22));
  if (bf) return i64 ? launch(append_kv_generic_kernel<__nv_bfloat16, int64_t>, grid, blk, 0, stream, enable_pdl, a)
                     : launch(append_kv_generic_kernel<__nv_bfloat16, int32_t>, grid, blk, 0, stream, enable_pdl, a);
  return i64 ? launch(append_kv_generic_kernel<__half, int64_t>, grid, blk, 0, stream, enable_pdl, a)
             : launch(append_kv_generic_kernel<__half, int32_t>, grid, blk, 0, stream, enable_pdl, a);
}

// Checks a MasPagedKVCache and the k/v layout, and fills AppendArgs (all but k, v and positions).
int make_append_args(AppendArgs* out, const MasPagedKVCache* c, const int32_t* batch_indices,
                     int64_t num_tokens, int64_t num_kv_heads, int64_t head_size, int64_t k_stride_token,
                     int64_t k_stride_head, int64_t v_stride_token, int64_t v_stride_head, int32_t* status) {
  if (!c || num_tokens < 0 || num_kv_heads < 0 || head_size <= 0 || num_kv_heads > INT32_MAX ||
      head_size > INT32_MAX)
    return MAS_ERR_INVALID_ARGUMENT;
  if (num_tokens > 0 && num_kv_heads > 0) {
    if (!c->k_cache || !c->v_cache || !c->kv_indices || !c->kv_indptr || !batch_indices)
      return MAS_ERR_INVALID_ARGUMENT;
    if (c->page_size <= 0 || c->num_pages < 0 || c->num_indices < 0 || c->batch_size < 0 ||
        c->stride_page < 0 || c->stride_entry < 0 || c->stride_head < 0)
      return MAS_ERR_INVALID_ARGUMENT;
  }
  AppendArgs a = {};
  a.T = num_tokens; a.ksn = k_stride_token; a.ksh = k_stride_head; a.vsn = v_stride_token; a.vsh = v_stride_head;
  a.Hkv = (int32_t)num_kv_heads; a.D = (int32_t)head_size; a.status = status;
  a.kv.k_cache = c->k_cache; a.kv.v_cache = c->v_cache; a.kv.num_pages = c->num_pages;
  a.kv.page_size = c->page_size; a.kv.stride_page = c->stride_page; a.kv.stride_entry = c->stride_entry;
  a.kv.stride_head = c->stride_head; a.kv.kv_indices = c->kv_indices; a.kv.num_indices = c->num_indices;
  a.kv.kv_indptr = c->kv_indptr; a.kv.batch_size = c->batch_size; a.kv.batch_indices = batch_indices;
  *out = a;
  return MAS_OK;
}

// Self-test of the bounded wait every bulk-copy consumer uses: one thread waits on an mbarrier that
// nothing will ever complete, with the caller's time limit, then reports the timeout exactly as the
// kernels do (MAS_STATUS_COPY_TIMEOUT in the fault word) and returns. No copy is in flight, so the
// CTA can leave with the barrier pending.
__global__ void selftest_wait_kernel(uint64_t limit_ns, int32_t* fault) {
  __shared__ uint64_t bar;
  mbar_init(&bar, 1);
  fence_barrier_init();
  if (!mbar_wait_bounded(&bar, 0, limit_ns)) atomicOr(fault, MAS_STATUS_COPY_TIMEOUT);
}

// Reads (and optionally zeroes) one of the library's per-device words with `device` current,
// restoring the caller's device. Synchronises the host with the device.
int read_word(int device, int32_t& word, int32_t* value, int clear) {
  if (value == nullptr) return MAS_ERR_INVALID_ARGUMENT;
  int rc = prepare(device);
  if (rc != MAS_OK) return rc;
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e == cudaSuccess && prev != device) e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(value, word, sizeof(int32_t));
  if (e == cudaSuccess && clear) {
    const int32_t zero = 0;
    e = cudaMemcpyToSymbol(word, &zero, sizeof(int32_t));
  }
  if (prev >= 0 && prev != device) (void)cudaSetDevice(prev);
  return e == cudaSuccess ? MAS_OK : (int)e;
}

}  // namespace
}  // namespace mas

using namespace mas;

extern "C" {

int mas_version(void) { return (0 << 16) | 1; }

const char* mas_status_string(int code) {
  switch (code) {
    case MAS_OK: return "ok";
    case MAS_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer, negative size or stride shorter than a row)";
    case MAS_ERR_UNSUPPORTED_DTYPE: return "unsupported dtype";
    case MAS_ERR_UNSUPPORTED_SHAPE: return "unsupported shape";
    case MAS_ERR_NO_DEVICE: return "no current CUDA device";
    default:
      if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
      return "unknown mas_b200 status code";
  }
}

int mas_prepare_device(int device) { return prepare(device); }

int mas_read_fault_word(int device, int32_t* value, int clear) {
  return read_word(device, g_fault_word, value, clear);
}

int mas_read_status_word(int device, int32_t* value, int clear) {
  return read_word(device, g_status_word, value, clear);
}

int mas_selftest_bounded_wait(int64_t limit_ns, void* stream) {
  if (limit_ns <= 0 || limit_ns > (int64_t)kWaitLimitNs) return MAS_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  return launch(selftest_wait_kernel, dim3(1), dim3(1), 0, stream, 0, (uint64_t)limit_ns, st->fault);
}

int mas_fused_add_rmsnorm(void* input, void* residual, const void* weight, int64_t num_tokens,
                          int64_t hidden_size, int64_t input_stride, int64_t residual_stride,
                          float eps, int dtype, int enable_pdl, void* stream) {
  if (num_tokens < 0 || hidden_size <= 0 || hidden_size > INT32_MAX) return MAS_ERR_INVALID_ARGUMENT;
  if (check_act_dtype(dtype) != MAS_OK) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens == 0) return MAS_OK;
  if (!input || !residual || !weight) return MAS_ERR_INVALID_ARGUMENT;
  if (input_stride < hidden_size || residual_stride < hidden_size) return MAS_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  NormArgs a = {};
  a.x = input; a.r = residual; a.w = weight; a.out = nullptr; a.scale = nullptr;
  a.rows = num_tokens; a.x_stride = input_stride; a.r_stride = residual_stride; a.out_stride = 0;
  a.H = (int32_t)hidden_size; a.eps = eps; a.fault = st->fault;
  const bool fast_ok = aligned(input, 16) && aligned(residual, 16) && aligned(weight, 16) &&
                       input_stride % 8 == 0 && residual_stride % 8 == 0;
  if (dtype == MAS_DTYPE_BF16) return run_norm<__nv_bfloat16, false>(a, *st, fast_ok, stream, enable_pdl);
  return run_norm<__half, false>(a, *st, fast_ok, stream, enable_pdl);
}

int mas_fused_add_rmsnorm_quant(void* out, const void* input, void* residual, const void* weight,
                                const float* scale, int64_t num_tokens, int64_t hidden_size,
                                int64_t out_stride, int64_t input_stride, int64_t residual_stride,
                                float eps, int dtype, int out_dtype, int enable_pdl, void* stream) {
  if (num_tokens < 0 || hidden_size <= 0 || hidden_size > INT32_MAX) return MAS_ERR_INVALID_ARGUMENT;
  if (check_act_dtype(dtype) != MAS_OK || out_dtype != MAS_DTYPE_FP8_E4M3) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens == 0) return MAS_OK;
  if (!out || !input || !residual || !weight || !scale) return MAS_ERR_INVALID_ARGUMENT;
  if (input_stride < hidden_size || residual_stride < hidden_size || out_stride < hidden_size)
    return MAS_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  NormArgs a = {};
  a.x = const_cast<void*>(input); a.r = residual; a.w = weight;
  a.out = static_cast<uint8_t*>(out); a.scale = scale;
  a.rows = num_tokens; a.x_stride = input_stride; a.r_stride = residual_stride;
  a.out_stride = out_stride; a.H = (int32_t)hidden_size; a.eps = eps; a.fault = st->fault;
  const bool fast_ok = aligned(input, 16) && aligned(residual, 16) && aligned(weight, 16) &&
                       aligned(out, 8) && input_stride % 8 == 0 && residual_stride % 8 == 0 &&
                       out_stride % 8 == 0;
  if (dtype == MAS_DTYPE_BF16) return run_norm<__nv_bfloat16, true>(a, *st, fast_ok, stream, enable_pdl);
  return run_norm<__half, true>(a, *st, fast_ok, stream, enable_pdl);
}

// One launch of SiLU-and-mul; `scale` != nullptr selects the e4m3 output (quant) form.
static int silu_impl(void* out, const void* input, const float* scale, int64_t num_tokens, int64_t d,
                     int64_t out_stride, int64_t input_stride, int dtype, int enable_pdl,
                     void* stream) {
  if (num_tokens < 0 || d < 0 || d > (INT32_MAX / 2)) return MAS_ERR_INVALID_ARGUMENT;
  if (check_act_dtype(dtype) != MAS_OK) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens == 0 || d == 0) return MAS_OK;
  if (!out || !input) return MAS_ERR_INVALID_ARGUMENT;
  if (input_stride < 2 * d || out_stride < d) return MAS_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  const bool quant = scale != nullptr;
  SiluArgs a = {};
  a.out = out; a.in = input; a.rows = num_tokens; a.in_stride = input_stride;
  a.out_stride = out_stride; a.d = (int32_t)d; a.fault = st->fault; a.scale = scale;
  const int out_align = quant ? 8 : 16;
  const bool vec = d % 8 == 0 && aligned(out, out_align) && aligned(input, 16) && input_stride % 8 == 0 &&
                   out_stride % 8 == 0;
  static const bool use_ring = env_is("MAS_SILU_IMPL", "ring");
  const bool bf16 = dtype == MAS_DTYPE_BF16;
  if (vec && (quant || !use_ring)) {
    static const int env_rows = env_int("MAS_SILU_GRID_ROWS", 0);
    // About 20 row groups per SM: each thread walks a few rows, so CTA start-up is amortised (16-28
    // per SM measured within 1 %). The e4m3 form is issue-bound and gains from longer-lived threads:
    // 4 per SM (chain shape: 109 us against 119 at 16 per SM). The group count is then evened out so
    // that every group walks the same number of rows (4352 rows: 2176 groups of 2, not 2368 of 1-2).
    const int64_t groups = env_rows > 0 ? env_rows : (quant ? 4 : 20) * (int64_t)st->sm_count;
    const int64_t target = std::min<int64_t>({num_tokens, groups, 65535});
    const int64_t per = ceil_div(num_tokens, target);
    const dim3 grid((unsigned)ceil_div(d / 8, kSiluThreads), (unsigned)ceil_div(num_tokens, per));
    const dim3 block(kSiluThreads);
    // Loads without an L1 line (L1::no_allocate) when the launch's input and output fit in about two
    // L2s, so that part of them may be served by L2 (decode-sized steps); plain read-only loads for
    // steps that stream from HBM. Measured at the chain width (I = 28672): a 512-token step of the
    // 88-layer chain 3.28 ms against 3.73; [4352, 57344] 108.9 against 110.3 us and [8192, 65536]
    // 225.7 against 233.6 us with the plain loads.
    static const int env_noalloc = env_int("MAS_SILU_NOALLOC", -1);
    const double footprint = (double)num_tokens * (double)d * (quant ? 5.0 : 6.0);  // bf16/fp16 in, out
    const bool noalloc = env_noalloc >= 0 ? env_noalloc > 0 : footprint <= 2.0 * (double)st->l2_bytes;
    if (quant) {
      if (noalloc)
        return bf16 ? launch(silu_mul_vec_kernel<__nv_bfloat16, true, true>, grid, block, 0, stream, enable_pdl, a)
                    : launch(silu_mul_vec_kernel<__half, true, true>, grid, block, 0, stream, enable_pdl, a);
      return bf16 ? launch(silu_mul_vec_kernel<__nv_bfloat16, true>, grid, block, 0, stream, enable_pdl, a)
                  : launch(silu_mul_vec_kernel<__half, true>, grid, block, 0, stream, enable_pdl, a);
    }
    if (noalloc)
      return bf16 ? launch(silu_mul_vec_kernel<__nv_bfloat16, false, true>, grid, block, 0, stream, enable_pdl, a)
                  : launch(silu_mul_vec_kernel<__half, false, true>, grid, block, 0, stream, enable_pdl, a);
    return bf16 ? launch(silu_mul_vec_kernel<__nv_bfloat16, false>, grid, block, 0, stream, enable_pdl, a)
                : launch(silu_mul_vec_kernel<__half, false>, grid, block, 0, stream, enable_pdl, a);
  }
  if (vec) {
    static const int env_stages = env_int("MAS_SILU_STAGES", 0);
    static const int env_ctas = env_int("MAS_SILU_CTAS_PER_SM", 0);
    const int stages = std::max(2, std::min(16, env_stages > 0 ? env_stages : 6));
    const size_t smem = silu_ring_smem_bytes(stages, 2);
    int ctas = env_ctas > 0 ? env_ctas : (int)std::max<size_t>(1, kRingBytesPerSm / smem);
    const void* fn = bf16 ? (const void*)silu_mul_ring_kernel<__nv_bfloat16>
                          : (const void*)silu_mul_ring_kernel<__half>;
    ctas = std::min(ctas, resident_ctas(fn, kSiluRingThreads, smem));
    const int64_t tiles = num_tokens * ceil_div(d, kSiluChunk);
    int64_t grid = std::min<int64_t>(tiles, (int64_t)st->sm_count * ctas);
    a.tiles_per_cta = ceil_div(tiles, grid);
    grid = ceil_div(tiles, a.tiles_per_cta);
    a.stages = stages;
    if (smem <= kMaxSmemPerCta) {
      return bf16 ? launch(silu_mul_ring_kernel<__nv_bfloat16>, dim3((unsigned)grid), dim3(kSiluRingThreads), smem,
                           stream, enable_pdl, a)
                  : launch(silu_mul_ring_kernel<__half>, dim3((unsigned)grid), dim3(kSiluRingThreads), smem, stream,
                           enable_pdl, a);
    }
  }
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(d, kSiluThreads), 1 << 16),
                  (unsigned)std::min<int64_t>(num_tokens, 65535));
  const dim3 block(kSiluThreads);
  if (quant) {
    return bf16 ? launch(silu_mul_generic_kernel<__nv_bfloat16, true>, grid, block, 0, stream, enable_pdl, a)
                : launch(silu_mul_generic_kernel<__half, true>, grid, block, 0, stream, enable_pdl, a);
  }
  return bf16 ? launch(silu_mul_generic_kernel<__nv_bfloat16, false>, grid, block, 0, stream, enable_pdl, a)
              : launch(silu_mul_generic_kernel<__half, false>, grid, block, 0, stream, enable_pdl, a);
}

int mas_silu_and_mul(void* out, const void* input, int64_t num_tokens, int64_t d,
                     int64_t out_stride, int64_t input_stride, int dtype, int enable_pdl,
                     void* stream) {
  return silu_impl(out, input, nullptr, num_tokens, d, out_stride, input_stride, dtype, enable_pdl, stream);
}

int mas_silu_and_mul_quant(void* out, const void* input, const float* scale, int64_t num_tokens,
                           int64_t d, int64_t out_stride, int64_t input_stride, int dtype,
                           int out_dtype, int enable_pdl, void* stream) {
  if (out_dtype != MAS_DTYPE_FP8_E4M3) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (!scale) return MAS_ERR_INVALID_ARGUMENT;
  return silu_impl(out, input, scale, num_tokens, d, out_stride, input_stride, dtype, enable_pdl, stream);
}

// Rotation (and, when q_beta != 0, the llama-4 query scale) of every rotary pair: one launch.
static int rope_main(const void* positions, int positions_dtype, void* query, void* key,
                     const float* cos_sin_cache, int64_t num_tokens, int64_t num_q_heads,
                     int64_t num_kv_heads, int64_t head_size, int64_t rotary_dim,
                     int64_t max_positions, int64_t q_stride_token, int64_t q_stride_head,
                     int64_t k_stride_token, int64_t k_stride_head, int is_neox, int dtype,
                     int32_t* status, int enable_pdl, void* stream, float q_beta, float q_inv_orig,
                     const AppendArgs* app = nullptr) {
  if (num_tokens < 0 || num_q_heads < 0 || num_kv_heads < 0 || head_size <= 0 ||
      max_positions < 0 || num_q_heads + num_kv_heads > INT32_MAX)
    return MAS_ERR_INVALID_ARGUMENT;
  if (check_act_dtype(dtype) != MAS_OK) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (positions_dtype != MAS_DTYPE_INT32 && positions_dtype != MAS_DTYPE_INT64)
    return MAS_ERR_UNSUPPORTED_DTYPE;
  if (rotary_dim <= 0 || rotary_dim % 2 != 0 || rotary_dim > head_size) return MAS_ERR_UNSUPPORTED_SHAPE;
  const int64_t NH = num_q_heads + num_kv_heads;
  if (num_tokens == 0 || NH == 0) return MAS_OK;
  if (!positions || !cos_sin_cache) return MAS_ERR_INVALID_ARGUMENT;
  if ((num_q_heads > 0 && !query) || (num_kv_heads > 0 && !key)) return MAS_ERR_INVALID_ARGUMENT;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  if (status == nullptr) status = st->status;
  RopeArgs a = {};
  a.pos = positions; a.q = query; a.k = key; a.cache = cos_sin_cache;
  a.T = num_tokens; a.P = max_positions;
  a.qsn = q_stride_token; a.qsh = q_stride_head; a.ksn = k_stride_token; a.ksh = k_stride_head;
  a.Hq = (int32_t)num_q_heads; a.Hkv = (int32_t)num_kv_heads; a.rd = (int32_t)rotary_dim;
  a.status = status; a.q_beta = q_beta; a.q_inv_orig = q_inv_orig;
  const bool q_al = num_q_heads == 0 || (aligned(query, 16) && q_stride_token % 8 == 0 && q_stride_head % 8 == 0);
  const bool k_al = num_kv_heads == 0 || (aligned(key, 16) && k_stride_token % 8 == 0 && k_stride_head % 8 == 0);
  const bool vec = rotary_dim % 16 == 0 && rotary_dim / 16 <= 32 && q_al && k_al &&
                   aligned(cos_sin_cache, 16) && num_tokens * NH < (int64_t)INT32_MAX;
  const bool i64 = positions_dtype == MAS_DTYPE_INT64;
  const bool bf = dtype == MAS_DTYPE_BF16;
  const bool neox = is_neox != 0;
  const dim3 blk(kRopeThreads);
#define MAS_ROPE_LAUNCH(KERNEL, GRID)                                                              \
  do {                                                                                             \
    if (bf) {                                                                                      \
      if (i64) return neox ? launch(KERNEL<__nv_bfloat16, int64_t, true>, GRID, blk, 0, stream, enable_pdl, a) \
                           : launch(KERNEL<__nv_bfloat16, int64_t, false>, GRID, blk, 0, stream, enable_pdl, a); \
      return neox ? launch(KERNEL<__nv_bfloat16, int32_t, true>, GRID, blk, 0, stream, enable_pdl, a)  \
                  : launch(KERNEL<__nv_bfloat16, int32_t, false>, GRID, blk, 0, stream, enable_pdl, a); \
    }                                                                                              \
    if (i64) return neox ? launch(KERNEL<__half, int64_t, true>, GRID, blk, 0, stream, enable_pdl, a) \
                         : launch(KERNEL<__half, int64_t, false>, GRID, blk, 0, stream, enable_pdl, a); \
    return neox ? launch(KERNEL<__half, int32_t, true>, GRID, blk, 0, stream, enable_pdl, a)        \
                : launch(KERNEL<__half, int32_t, false>, GRID, blk, 0, stream, enable_pdl, a);      \
  } while (0)
  // Token-staged TMA ring: q heads and k heads contiguous within each token, 16-byte aligned rows,
  // and enough tokens for the ring's prologue to pay off; a step with only a few tokens per SM goes to
  // the vector kernel, which issues all its loads at once (in a CUDA graph at the chain's shape: 64
  // tokens 2.8 -> 2.2 us, 256 tokens 3.6 -> 3.2 us; from 512 tokens the ring is faster: 5.1 against
  // 5.7 us, and 40 against 44 us at 4352). The fused paged append always takes the ring.
  static const bool force_vec = env_is("MAS_ROPE_IMPL", "vec");
  static const bool force_ring = env_is("MAS_ROPE_IMPL", "ring");
  static const int env_ring_min = env_int("MAS_ROPE_RING_MIN_TOKENS", 0);
  const int64_t ring_min = env_ring_min > 0 ? env_ring_min : 2 * (int64_t)st->sm_count;
  const bool few_tokens = app == nullptr && !force_ring && num_tokens < ring_min;
  const bool ring = vec && !force_vec && !few_tokens && head_size % 8 == 0 &&
                    (num_q_heads == 0 || q_stride_head == head_size) &&
                    (num_kv_heads == 0 || k_stride_head == head_size);
  if (ring && (!app || append_ring_ok(*app, head_size))) {
    RopeRingArgs r = {};
    r.pos = positions; r.q = query; r.k = key; r.cache = cos_sin_cache; r.T = num_tokens; r.P = max_positions;
    r.qsn = q_stride_token; r.ksn = k_stride_token; r.Hq = (int32_t)num_q_heads; r.Hkv = (int32_t)num_kv_heads;
    r.D = (int32_t)head_size; r.rd = (int32_t)rotary_dim; r.status = status; r.fault = st->fault;
    r.q_beta = q_beta; r.q_inv_orig = q_inv_orig;
    if (app) {
      r.v = app->v; r.vsn = app->vsn; r.kv = app->kv;
    }
    const int rc_ring = launch_rope_ring(r, app != nullptr, bf, i64, neox, st, stream, enable_pdl);
    if (rc_ring != kNotLaunched) return rc_ring;
  }
  if (app) {
    // Unfused: the rope launch, then the append launch (tokens that rope skipped stay unappended).
    const int rc2 = rope_main(positions, positions_dtype, query, key, cos_sin_cache, num_tokens, num_q_heads,
                              num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token, q_stride_head,
                              k_stride_token, k_stride_head, is_neox, dtype, status, enable_pdl, stream, q_beta,
                              q_inv_orig, nullptr);
    if (rc2 != MAS_OK || max_positions == 0) return rc2;
    AppendArgs ap = *app;
    ap.pos_limit = max_positions;
    return launch_append(ap, bf, i64, st, stream, enable_pdl);
  }
  if (vec) {
    a.tpu = (int32_t)(rotary_dim / 16);
    const int64_t upb = kRopeThreads / a.tpu;
    const dim3 grid((unsigned)std::min<int64_t>(ceil_div(num_tokens * NH, upb * kRopeUnits), INT32_MAX));
    MAS_ROPE_LAUNCH(rope_vec_kernel, grid);
  }
  const int64_t pairs = num_tokens * NH * (rotary_dim / 2);
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(pairs, kRopeThreads), 1 << 22));
  MAS_ROPE_LAUNCH(rope_generic_kernel, grid);
#undef MAS_ROPE_LAUNCH
}

int mas_rope_cos_sin_cache_inplace(const void* positions, int positions_dtype, void* query,
                                   void* key, const float* cos_sin_cache, int64_t num_tokens,
                                   int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                   int64_t rotary_dim, int64_t max_positions,
                                   int64_t q_stride_token, int64_t q_stride_head,
                                   int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                   int dtype, int32_t* status, int enable_pdl, void* stream) {
  return rope_main(positions, positions_dtype, query, key, cos_sin_cache, num_tokens, num_q_heads,
                   num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token, q_stride_head,
                   k_stride_token, k_stride_head, is_neox, dtype, status, enable_pdl, stream, 0.f, 0.f);
}

// Rope with the llama-4 query scale (optionally fused with the paged append), plus the element-wise
// scale of the q elements past rotary_dim when the rotary part is partial.
static int rope_q_scale_impl(const void* positions, int positions_dtype, void* query, void* key,
                             const float* cos_sin_cache, int64_t num_tokens, int64_t num_q_heads,
                             int64_t num_kv_heads, int64_t head_size, int64_t rotary_dim, int64_t max_positions,
                             int64_t q_stride_token, int64_t q_stride_head, int64_t k_stride_token,
                             int64_t k_stride_head, int is_neox, float q_scale_beta, int64_t q_scale_original_max,
                             int dtype, int32_t* status, int enable_pdl, void* stream, const AppendArgs* app) {
  float inv_orig = 0.f;
  if (q_scale_beta != 0.f) {
    if (q_scale_original_max <= 0) return MAS_ERR_INVALID_ARGUMENT;
    // torch divides a CUDA tensor by a host scalar as a multiplication by the fp32 reciprocal.
    inv_orig = 1.0f / (float)q_scale_original_max;
  }
  int rc = rope_main(positions, positions_dtype, query, key, cos_sin_cache, num_tokens, num_q_heads,
                     num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token, q_stride_head,
                     k_stride_token, k_stride_head, is_neox, dtype, status, enable_pdl, stream,
                     q_scale_beta, inv_orig, app);
  if (rc != MAS_OK || q_scale_beta == 0.f || rotary_dim >= head_size || num_q_heads == 0 || num_tokens == 0)
    return rc;
  // Partial rotary: the elements past rotary_dim are scaled by a second, element-wise launch.
  RopeArgs a = {};
  a.pos = positions; a.q = query; a.T = num_tokens; a.P = max_positions; a.qsn = q_stride_token;
  a.qsh = q_stride_head; a.Hq = (int32_t)num_q_heads; a.rd = (int32_t)rotary_dim;
  a.q_beta = q_scale_beta; a.q_inv_orig = inv_orig;
  const int64_t total = num_tokens * num_q_heads * (head_size - rotary_dim);
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(total, kRopeThreads), 1 << 22));
  const bool bf = dtype == MAS_DTYPE_BF16, i64 = positions_dtype == MAS_DTYPE_INT64;
  const int32_t hs = (int32_t)head_size;
  if (bf) return i64 ? launch(rope_q_tail_scale_kernel<__nv_bfloat16, int64_t>, grid, dim3(kRopeThreads), 0, stream, enable_pdl, a, hs)
                     : launch(rope_q_tail_scale_kernel<__nv_bfloat16, int32_t>, grid, dim3(kRopeThreads), 0, stream, enable_pdl, a, hs);
  return i64 ? launch(rope_q_tail_scale_kernel<__half, int64_t>, grid, dim3(kRopeThreads), 0, stream, enable_pdl, a, hs)
             : launch(rope_q_tail_scale_kernel<__half, int32_t>, grid, dim3(kRopeThreads), 0, stream, enable_pdl, a, hs);
}

int mas_rope_cos_sin_cache_q_scale_inplace(const void* positions, int positions_dtype, void* query,
                                           void* key, const float* cos_sin_cache, int64_t num_tokens,
                                           int64_t num_q_heads, int64_t num_kv_heads, int64_t head_size,
                                           int64_t rotary_dim, int64_t max_positions,
                                           int64_t q_stride_token, int64_t q_stride_head,
                                           int64_t k_stride_token, int64_t k_stride_head, int is_neox,
                                           float q_scale_beta, int64_t q_scale_original_max, int dtype,
                                           int32_t* status, int enable_pdl, void* stream) {
  if (q_scale_original_max <= 0) return MAS_ERR_INVALID_ARGUMENT;
  return rope_q_scale_impl(positions, positions_dtype, query, key, cos_sin_cache, num_tokens, num_q_heads,
                           num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token, q_stride_head,
                           k_stride_token, k_stride_head, is_neox, q_scale_beta, q_scale_original_max, dtype,
                           status, enable_pdl, stream, nullptr);
}

int mas_append_paged_kv_cache(const void* key, const void* value, const int32_t* batch_indices,
                              const void* positions, int positions_dtype, const MasPagedKVCache* cache,
                              int64_t num_tokens, int64_t num_kv_heads, int64_t head_size,
                              int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_token,
                              int64_t v_stride_head, int dtype, int32_t* status, int enable_pdl,
                              void* stream) {
  if (check_act_dtype(dtype) != MAS_OK) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (positions_dtype != MAS_DTYPE_INT32 && positions_dtype != MAS_DTYPE_INT64) return MAS_ERR_UNSUPPORTED_DTYPE;
  AppendArgs a;
  int rc = make_append_args(&a, cache, batch_indices, num_tokens, num_kv_heads, head_size, k_stride_token,
                            k_stride_head, v_stride_token, v_stride_head, status);
  if (rc != MAS_OK) return rc;
  if (num_tokens == 0 || num_kv_heads == 0) return MAS_OK;
  if (!key || !value || !positions) return MAS_ERR_INVALID_ARGUMENT;
  a.k = key; a.v = value; a.pos = positions;
  DeviceState* st = nullptr;
  if ((rc = current_device(&st)) != MAS_OK) return rc;
  return launch_append(a, dtype == MAS_DTYPE_BF16, positions_dtype == MAS_DTYPE_INT64, st, stream, enable_pdl);
}

int mas_rope_append_paged_kv_cache(const void* positions, int positions_dtype, void* query, void* key,
                                   const void* value, const float* cos_sin_cache, const int32_t* batch_indices,
                                   const MasPagedKVCache* cache, int64_t num_tokens, int64_t num_q_heads,
                                   int64_t num_kv_heads, int64_t head_size, int64_t rotary_dim,
                                   int64_t max_positions, int64_t q_stride_token, int64_t q_stride_head,
                                   int64_t k_stride_token, int64_t k_stride_head, int64_t v_stride_token,
                                   int64_t v_stride_head, int is_neox, float q_scale_beta,
                                   int64_t q_scale_original_max, int dtype, int32_t* status, int enable_pdl,
                                   void* stream) {
  AppendArgs a;
  int rc = make_append_args(&a, cache, batch_indices, num_tokens, num_kv_heads, head_size, k_stride_token,
                            k_stride_head, v_stride_token, v_stride_head, status);
  if (rc != MAS_OK) return rc;
  if (num_tokens > 0 && num_kv_heads > 0 && !value) return MAS_ERR_INVALID_ARGUMENT;
  a.k = key; a.v = value; a.pos = positions;
  return rope_q_scale_impl(positions, positions_dtype, query, key, cos_sin_cache, num_tokens, num_q_heads,
                           num_kv_heads, head_size, rotary_dim, max_positions, q_stride_token, q_stride_head,
                           k_stride_token, k_stride_head, is_neox, q_scale_beta, q_scale_original_max, dtype,
                           status, enable_pdl, stream, num_kv_heads > 0 ? &a : nullptr);
}

static int gather_impl(void* out, const void* table, const void* ids, int ids_dtype,
                       int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                       int64_t out_stride, int64_t table_stride, int elem_size,
                       int32_t* status, int enable_pdl, void* stream, const void* last,
                       int last_dtype, int64_t num_last) {
  if (num_tokens < 0 || hidden_size <= 0 || vocab_size < 0) return MAS_ERR_INVALID_ARGUMENT;
  if (elem_size != 1 && elem_size != 2 && elem_size != 4 && elem_size != 8) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (ids_dtype != MAS_DTYPE_INT32 && ids_dtype != MAS_DTYPE_INT64) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (num_tokens == 0) return MAS_OK;
  if (!out || !table || !ids) return MAS_ERR_INVALID_ARGUMENT;
  if (out_stride < hidden_size || table_stride < hidden_size) return MAS_ERR_INVALID_ARGUMENT;
  const int64_t row_bytes = hidden_size * elem_size;
  if (row_bytes > INT32_MAX) return MAS_ERR_UNSUPPORTED_SHAPE;
  DeviceState* st = nullptr;
  int rc = current_device(&st);
  if (rc != MAS_OK) return rc;
  EmbedArgs a = {};
  a.out = out; a.table = table; a.ids = ids; a.T = num_tokens; a.V = vocab_size;
  a.out_stride_b = out_stride * elem_size; a.table_stride_b = table_stride * elem_size;
  a.row_bytes = (uint32_t)row_bytes; a.status = status ? status : st->status; a.fault = st->fault;
  a.last = last; a.n_last = num_last; a.last_is_64 = last_dtype == MAS_DTYPE_INT64 ? 1 : 0;
  const bool i64 = ids_dtype == MAS_DTYPE_INT64;
  const bool tma = row_bytes % 16 == 0 && row_bytes <= 64 * 1024 && aligned(out, 16) &&
                   aligned(table, 16) && a.out_stride_b % 16 == 0 && a.table_stride_b % 16 == 0;
  // The register path, one CTA per row and column block of 8 KB, all loads before the stores. In a
  // CUDA graph at H = 12288 it beat the TMA ring at every step size measured: 1.43 against 2.17 us
  // at 64 rows, 5.58 against 6.78 us at 1024, 34.8 against 36.1 us at 4352. The ring stays for
  // placeholder filling (one CTA per row must own the id write-back) and on request.
  static const bool force_tma = env_is("MAS_EMBED_IMPL", "tma");
  if (tma && last == nullptr && !force_tma) {
    const int64_t nvec = row_bytes / 16;
    const int64_t blocks = ceil_div(nvec, (int64_t)kEmbedVecThreads * kEmbedVecPerThread);
    a.chunk_bytes = (uint32_t)(ceil_div(nvec, blocks) * 16);  // equal blocks: 10 KB rows -> 2 x 5 KB
    const dim3 g((unsigned)std::min<int64_t>(num_tokens, INT32_MAX), (unsigned)blocks);
    if (num_tokens <= INT32_MAX) {
      if (i64) return launch(embed_vec_kernel<int64_t>, g, dim3(kEmbedVecThreads), 0, stream, enable_pdl, a);
      return launch(embed_vec_kernel<int32_t>, g, dim3(kEmbedVecThreads), 0, stream, enable_pdl, a);
    }
  }
  if (tma) {
    // Optional column chunks (MAS_EMBED_CHUNKS): a row's copy split over several CTAs. Measured no
    // better than whole rows at 64-1024 rows (the register path above serves small steps); off by
    // default. Never with placeholder filling, whose id write-back one CTA per row must own.
    static const int env_chunks = env_int("MAS_EMBED_CHUNKS", 0);
    int64_t chunks = env_chunks > 0 ? env_chunks : 1;
    chunks = last != nullptr ? 1 : std::max<int64_t>(1, std::min<int64_t>(chunks, row_bytes / 2048));
    a.chunk_bytes = (uint32_t)(ceil_div(ceil_div(row_bytes, chunks), 16) * 16);
    chunks = ceil_div(row_bytes, a.chunk_bytes);
    static const int env_stages = env_int("MAS_EMBED_STAGES", 0);
    int stages = env_stages > 0 ? env_stages : (int)std::max<int64_t>(2, std::min<int64_t>(8, (48 * 1024) / a.chunk_bytes));
    stages = std::max(2, std::min(16, stages));
    const size_t ring = (size_t)stages * (size_t)a.chunk_bytes + 8 * (size_t)kEmbedMaxRowsPerCta;
    const int ctas = (int)std::max<size_t>(1, std::min<size_t>(16, kRingBytesPerSm / ring));
    int64_t grid = std::max<int64_t>((int64_t)st->sm_count * ctas, ceil_div(num_tokens, kEmbedMaxRowsPerCta));
    grid = std::min<int64_t>(grid, num_tokens);
    a.rows_per_cta = (int32_t)ceil_div(num_tokens, grid);
    grid = ceil_div(num_tokens, a.rows_per_cta);
    a.stages = stages;
    const size_t smem = embed_tma_smem_bytes(a.chunk_bytes, stages, a.rows_per_cta);
    if (smem <= kMaxSmemPerCta && grid <= INT32_MAX && chunks <= 65535) {
      const dim3 g((unsigned)grid, (unsigned)chunks);
      if (i64) return launch(embed_tma_kernel<int64_t>, g, dim3(32), smem, stream, enable_pdl, a);
      return launch(embed_tma_kernel<int32_t>, g, dim3(32), smem, stream, enable_pdl, a);
    }
  }
  int unit = 16;
  while (unit > 1 && (row_bytes % unit != 0 || !aligned(out, unit) || !aligned(table, unit) ||
                      a.out_stride_b % unit != 0 || a.table_stride_b % unit != 0))
    unit >>= 1;
  const dim3 grid((unsigned)std::min<int64_t>(ceil_div(num_tokens, 8), 1 << 20));
  if (i64) return launch(embed_generic_kernel<int64_t>, grid, dim3(256), 0, stream, enable_pdl, a, unit);
  return launch(embed_generic_kernel<int32_t>, grid, dim3(256), 0, stream, enable_pdl, a, unit);
}

int mas_embedding_gather(void* out, const void* table, const void* ids, int ids_dtype,
                         int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                         int64_t out_stride, int64_t table_stride, int elem_size,
                         int32_t* status, int enable_pdl, void* stream) {
  return gather_impl(out, table, ids, ids_dtype, num_tokens, hidden_size, vocab_size, out_stride,
                     table_stride, elem_size, status, enable_pdl, stream, nullptr, MAS_DTYPE_INT32, 0);
}

int mas_embedding_gather_fill_placeholders(void* out, const void* table, void* ids, int ids_dtype,
                                           const void* last_tokens, int last_dtype, int64_t num_last,
                                           int64_t num_tokens, int64_t hidden_size, int64_t vocab_size,
                                           int64_t out_stride, int64_t table_stride, int elem_size,
                                           int32_t* status, int enable_pdl, void* stream) {
  if (last_dtype != MAS_DTYPE_INT32 && last_dtype != MAS_DTYPE_INT64) return MAS_ERR_UNSUPPORTED_DTYPE;
  if (num_last < 0 || (num_last > 0 && last_tokens == nullptr)) return MAS_ERR_INVALID_ARGUMENT;
  return gather_impl(out, table, ids, ids_dtype, num_tokens, hidden_size, vocab_size, out_stride,
                     table_stride, elem_size, status, enable_pdl, stream,
                     num_last > 0 ? last_tokens : nullptr, last_dtype, num_last);
}

}  // extern "C"
