// paged_kv.cuh -- appending each token's k and v rows to the paged KV cache, for sm_100a.
//
// Semantics follow flashinfer 0.6.11.post2's append_paged_kv_cache (FI/page.py:280-406 with the
// kernel FI/data/include/flashinfer/page.cuh:259-284 and the element offsets of :161-165), as
// Devstral2Attention.forward calls it (miniagentserve/models/devstral2/devstral2.py:170-173, with
// kv_indices = block_tables.flatten() and kv_indptr = arange(batch + 1) * max_blocks, :289): token t
// of sequence b = batch_indices[t] at position p = positions[t] goes to
//   flat = kv_indptr[b] * page_size + p,  page = kv_indices[flat / page_size],  entry = flat % page_size
//   k_cache[page, entry, h, :] = k[t, h, :]   (NHD; HND swaps entry and head), same for v.
// The copy is byte-exact. Unlike the reference kernel, every index is checked before it is used:
// a batch index outside [0, batch_size), a negative position, a page slot outside kv_indices or a
// page id outside [0, num_pages) skips the token's append and raises MAS_STATUS_KV_SLOT_OUT_OF_RANGE.
//
// This header holds the slot arithmetic (shared with the fused rope + append ring in rope.cuh) and
// the standalone append kernels: a warp per token (one slot computation per warp, its lanes copying
// 16-byte vectors of every k and v head: coalesced 256-byte rows per head) and a scalar fallback
// for unaligned layouts.
#pragma once

#include "common.cuh"

namespace mas {

struct PagedKVArgs {
  void* k_cache;
  void* v_cache;
  int64_t num_pages;
  int64_t page_size;
  int64_t stride_page, stride_entry, stride_head;  // elements; k and v share them
  const int32_t* kv_indices;
  int64_t num_indices;
  const int32_t* kv_indptr;
  int64_t batch_size;
  const int32_t* batch_indices;  // [T]
};

// Element offset of (page, entry, head 0, feature 0) for token t at position pos, or -1 when an
// index is out of range (the caller flags it).
__device__ __forceinline__ int64_t kv_slot(const PagedKVArgs& p, int64_t t, int64_t pos) {
  const int64_t b = p.batch_indices[t];
  if (b < 0 || b >= p.batch_size || pos < 0) return -1;
  const int64_t flat = (int64_t)p.kv_indptr[b] * p.page_size + pos;
  if (flat < 0) return -1;
  const int64_t page_iter = flat / p.page_size;
  const int64_t entry = flat - page_iter * p.page_size;
  if (page_iter >= p.num_indices) return -1;
  const int64_t page = p.kv_indices[page_iter];
  if (page < 0 || page >= p.num_pages) return -1;
  return page * p.stride_page + entry * p.stride_entry;
}

struct AppendArgs {
  const void* k;
  const void* v;
  const void* pos;
  int64_t T;
  int64_t ksn, ksh, vsn, vsh;  // elements
  int32_t Hkv, D;
  int32_t* status;
  int64_t pos_limit;  // > 0: tokens at positions outside [0, pos_limit) are skipped (rope left them as is)
  PagedKVArgs kv;
};

constexpr int kAppendThreads = 256;

template <typename T, typename PosT>
__global__ void __launch_bounds__(kAppendThreads) append_kv_vec_kernel(const AppendArgs a) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * kAppendThreads + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * kAppendThreads) >> 5;
  const int vpr = a.D >> 3;  // 16-byte vectors per head row
  const int per_tensor = a.Hkv * vpr;
  for (int64_t t = warp; t < a.T; t += nwarps) {
    int64_t slot = 0;
    if (lane == 0) {
      const int64_t pos = (int64_t)static_cast<const PosT*>(a.pos)[t];
      if (a.pos_limit > 0 && (pos < 0 || pos >= a.pos_limit)) {
        slot = -1;
      } else {
        slot = kv_slot(a.kv, t, pos);
        if (slot < 0) flag_status(a.status, MAS_STATUS_KV_SLOT_OUT_OF_RANGE);
      }
    }
    slot = __shfl_sync(0xffffffffu, slot, 0);
    if (slot < 0) continue;
    for (int u = lane; u < 2 * per_tensor; u += 32) {
      const bool is_v = u >= per_tensor;
      const int r = is_v ? u - per_tensor : u;
      const int h = r / vpr, j = r - h * vpr;
      const T* src = static_cast<const T*>(is_v ? a.v : a.k) + t * (is_v ? a.vsn : a.ksn) +
                     (int64_t)h * (is_v ? a.vsh : a.ksh) + j * 8;
      T* dst = static_cast<T*>(is_v ? a.kv.v_cache : a.kv.k_cache) + slot + (int64_t)h * a.kv.stride_head + j * 8;
      st_plain(dst, ld_ro(src));
    }
  }
  pdl_launch_dependents();
}

template <typename T, typename PosT>
__global__ void __launch_bounds__(kAppendThreads) append_kv_generic_kernel(const AppendArgs a) {
  pdl_wait();
  const int64_t per_token = (int64_t)a.Hkv * a.D;
  const int64_t total = a.T * per_token;
  for (int64_t idx = (int64_t)blockIdx.x * kAppendThreads + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * kAppendThreads) {
    const int64_t t = idx / per_token;
    const int64_t r = idx - t * per_token;
    const int64_t h = r / a.D, f = r - h * a.D;
    const int64_t pos = (int64_t)static_cast<const PosT*>(a.pos)[t];
    if (a.pos_limit > 0 && (pos < 0 || pos >= a.pos_limit)) continue;
    const int64_t slot = kv_slot(a.kv, t, pos);
    if (slot < 0) {
      if (r == 0) flag_status(a.status, MAS_STATUS_KV_SLOT_OUT_OF_RANGE);
      continue;
    }
    const int64_t dst = slot + h * a.kv.stride_head + f;
    static_cast<uint16_t*>(a.kv.k_cache)[dst] = static_cast<const uint16_t*>(a.k)[t * a.ksn + h * a.ksh + f];
    static_cast<uint16_t*>(a.kv.v_cache)[dst] = static_cast<const uint16_t*>(a.v)[t * a.vsn + h * a.vsh + f];
  }
  pdl_launch_dependents();
}

}  // namespace mas
