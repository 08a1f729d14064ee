// embed.cuh -- token-embedding gather for sm_100a: out[t, :] = table[ids[t], :], a bit copy.
//
// Replaces the aten/inductor embedding behind nn.Embedding (Devstral2Model.embed_tokens,
// miniagentserve/models/devstral2/devstral2.py:260, :282).
//
// TMA path (rows of a multiple of 16 bytes, 16-byte aligned; placeholder filling, or on request):
// the TMA engine does the whole copy.
// Each CTA is one warp that owns a contiguous block of output rows (and, when a step has too few
// rows to occupy every SM, one column chunk of them: blockIdx.y); it stages their ids in shared
// memory (one coalesced read), then lane 0 keeps an S-stage ring busy: a bulk load of the table row
// into a stage (mbarrier transaction count), then a bulk store of that stage into the output row
// (bulk async-group), refilling a stage as soon as its store has finished reading it. Several
// CTAs per SM keep tens of rows in flight per SM with almost no instructions issued.
//
// Generic path (any row size or alignment): one warp per row with the widest unit the alignment
// allows. An id outside [0, V) zeroes its output row in both paths and sets a status bit.
#pragma once

#include "common.cuh"

namespace mas {

struct EmbedArgs {
  void* out;
  const void* table;
  const void* ids;
  int64_t T;
  int64_t V;
  int64_t out_stride_b;    // bytes
  int64_t table_stride_b;  // bytes
  uint32_t row_bytes;
  uint32_t chunk_bytes;    // fast path: bytes of a row one CTA copies (a multiple of 16; blockIdx.y picks
                           // the chunk), the whole row unless few rows must be spread over the SMs
  int32_t stages;
  int32_t rows_per_cta;
  int32_t* status;
  int32_t* fault;
  // Placeholder filling (ModelRunner.fill_placeholders, model_runner.py:149-154): when `last` is set,
  // an id -1-r (r >= 0) stands for last[r], the previous step's sample for row r; the resolved id is
  // written back into ids. r outside [0, n_last) is an out-of-range id.
  const void* last;
  int64_t n_last;
  int32_t last_is_64;
};

// The id of token t, with a placeholder resolved (and written back) when placeholder filling is on.
template <typename IdT>
__device__ __forceinline__ int64_t resolve_id(const EmbedArgs& a, const IdT* ids, int64_t t) {
  int64_t id = (int64_t)ids[t];
  if (a.last != nullptr && id < 0) {
    const int64_t r = -1 - id;
    if (r < a.n_last) {
      id = a.last_is_64 ? static_cast<const int64_t*>(a.last)[r] : (int64_t) static_cast<const int32_t*>(a.last)[r];
      const_cast<IdT*>(ids)[t] = (IdT)id;
    } else {
      id = -1;
    }
  }
  return id;
}

constexpr int kEmbedMaxRowsPerCta = 1024;

__host__ __device__ inline size_t embed_tma_smem_bytes(uint32_t row_bytes, int stages, int rows_per_cta) {
  return (size_t)stages * row_bytes + (size_t)stages * 8 + (size_t)rows_per_cta * 8;
}

template <typename IdT>
__global__ void __launch_bounds__(32) embed_tma_kernel(const EmbedArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  const int S = a.stages;
  const uint32_t col0 = blockIdx.y * a.chunk_bytes;
  const uint32_t rb = min(a.chunk_bytes, a.row_bytes - col0);
  unsigned char* ring = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * a.chunk_bytes);
  int64_t* sid = reinterpret_cast<int64_t*>(bars + S);
  const int lane = threadIdx.x;

  const int64_t row0 = (int64_t)blockIdx.x * a.rows_per_cta;
  const int n = (int)min((int64_t)a.rows_per_cta, a.T - row0);

  if (lane == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  pdl_wait();
  const IdT* ids = static_cast<const IdT*>(a.ids) + row0;
  for (int i = lane; i < n; i += kWarp) {
    const int64_t id = resolve_id<IdT>(a, ids, i);
    const bool valid = id >= 0 && id < a.V;
    if (!valid) flag_status(a.status, MAS_STATUS_EMBED_ID_OUT_OF_RANGE);
    sid[i] = valid ? id : -1;
  }
  __syncwarp();

  const unsigned char* table = static_cast<const unsigned char*>(a.table) + col0;
  unsigned char* out = static_cast<unsigned char*>(a.out) + col0;
  // Rows with an invalid id complete their stage without a copy (plain arrive).
  auto issue = [&](int k) {
    const int s = k % S;
    const int64_t id = sid[k];
    if (id >= 0) {
      mbar_arrive_expect_tx(&bars[s], rb);
      bulk_load(ring + (size_t)s * a.chunk_bytes, table + id * a.table_stride_b, rb, &bars[s]);
    } else {
      mbar_arrive(&bars[s]);
    }
  };
  if (lane == 0) {
    const int pre = n < S ? n : S;
    for (int k = 0; k < pre; ++k) issue(k);
  }

  int k = 0;
  for (; k < n; ++k) {
    const int s = k % S;
    int ok = 1;
    if (lane == 0) ok = mbar_wait_bounded(&bars[s], (uint32_t)(k / S) & 1u) ? 1 : 0;
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) break;
    unsigned char* dst = out + (row0 + k) * a.out_stride_b;
    if (sid[k] >= 0) {
      if (lane == 0) bulk_store(dst, ring + (size_t)s * a.chunk_bytes, rb);
    } else {
      for (uint32_t b = (uint32_t)lane * 16u; b < rb; b += kWarp * 16u)
        st_plain(dst + b, Vec16{0u, 0u, 0u, 0u});
    }
    if (lane == 0) {
      bulk_commit();
      // Refill the previous stage once its store has read it (all groups but the newest done).
      if (k >= 1 && k - 1 + S < n) {
        bulk_wait_read<1>();
        issue(k - 1 + S);
      }
    }
    __syncwarp();
  }
  if (lane == 0) {
    if (k < n) {
      atomicOr(a.fault, MAS_STATUS_COPY_TIMEOUT);
      // Loads issued so far cover rows < min(n, max(k, 1) - 1 + S); wait (bounded) for each.
      const int issued_end = min(n, (k >= 1 ? k - 1 : 0) + S);
      for (int kk = k; kk < issued_end; ++kk)
        (void)mbar_wait_bounded(&bars[kk % S], (uint32_t)(kk / S) & 1u);
    }
    bulk_wait_all();  // the ring must not be released while a store still reads it
  }
  __syncwarp();
  pdl_launch_dependents();
}

// Register path (the default for aligned rows): CTA (row, column block) copies its block of the row
// (blocks of equal size, chunk_bytes each, at most kEmbedVecPerThread 16-byte vectors per thread),
// every load issued before any store, so a row costs about one HBM round trip instead of a bulk load
// followed by a bulk store.
// (Not used with placeholder filling: the CTAs of one row would race on the id write-back.)
constexpr int kEmbedVecThreads = 128;
constexpr int kEmbedVecPerThread = 4;

template <typename IdT>
__global__ void __launch_bounds__(kEmbedVecThreads) embed_vec_kernel(const EmbedArgs a) {
  pdl_wait();
  const int64_t t = blockIdx.x;
  const int64_t id = (int64_t)static_cast<const IdT*>(a.ids)[t];
  const bool valid = id >= 0 && id < a.V;
  if (!valid && blockIdx.y == 0 && threadIdx.x == 0) flag_status(a.status, MAS_STATUS_EMBED_ID_OUT_OF_RANGE);
  // column block blockIdx.y: vectors [b0, b1) of the row, blocks of equal size (chunk_bytes / 16)
  const uint32_t nvec = a.row_bytes >> 4;
  const uint32_t b0 = blockIdx.y * (a.chunk_bytes >> 4);
  const uint32_t b1 = min(nvec, b0 + (a.chunk_bytes >> 4));
  const uint32_t v0 = b0 + threadIdx.x;
  const unsigned char* src = static_cast<const unsigned char*>(a.table) + (valid ? id : 0) * a.table_stride_b;
  unsigned char* dst = static_cast<unsigned char*>(a.out) + t * a.out_stride_b;
  Vec16 v[kEmbedVecPerThread];
#pragma unroll
  for (int j = 0; j < kEmbedVecPerThread; ++j) {
    const uint32_t u = v0 + (uint32_t)j * kEmbedVecThreads;
    if (u < b1) v[j] = valid ? ld_ro(src + (size_t)u * 16) : Vec16{0u, 0u, 0u, 0u};
  }
#pragma unroll
  for (int j = 0; j < kEmbedVecPerThread; ++j) {
    const uint32_t u = v0 + (uint32_t)j * kEmbedVecThreads;
    if (u < b1) st_plain(dst + (size_t)u * 16, v[j]);
  }
  pdl_launch_dependents();
}

// Generic path: one warp per row; `unit` is the widest power-of-two byte count (<= 16) dividing
// the row size, both strides and both base addresses.
template <typename IdT>
__global__ void __launch_bounds__(256) embed_generic_kernel(const EmbedArgs a, int unit) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int64_t wid = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const IdT* ids = static_cast<const IdT*>(a.ids);
  const unsigned char* table = static_cast<const unsigned char*>(a.table);
  unsigned char* out = static_cast<unsigned char*>(a.out);
  for (int64_t t = wid; t < a.T; t += nw) {
    int64_t id = 0;
    if (lane == 0) id = resolve_id<IdT>(a, ids, t);
    id = __shfl_sync(0xffffffffu, id, 0);
    const bool valid = id >= 0 && id < a.V;
    if (!valid && lane == 0) flag_status(a.status, MAS_STATUS_EMBED_ID_OUT_OF_RANGE);
    const unsigned char* src = table + (valid ? id : 0) * a.table_stride_b;
    unsigned char* dst = out + t * a.out_stride_b;
    const uint32_t nu = a.row_bytes / (uint32_t)unit;
    for (uint32_t i = lane; i < nu; i += kWarp) {
      const size_t off = (size_t)i * unit;
      switch (unit) {
        case 16: {
          const Vec16 v = valid ? ld_ro(src + off) : Vec16{0u, 0u, 0u, 0u};
          st_plain(dst + off, v);
          break;
        }
        case 8:
          *reinterpret_cast<uint64_t*>(dst + off) =
              valid ? __ldg(reinterpret_cast<const unsigned long long*>(src + off)) : 0ull;
          break;
        case 4:
          *reinterpret_cast<uint32_t*>(dst + off) =
              valid ? __ldg(reinterpret_cast<const unsigned int*>(src + off)) : 0u;
          break;
        case 2:
          *reinterpret_cast<uint16_t*>(dst + off) =
              valid ? __ldg(reinterpret_cast<const unsigned short*>(src + off)) : (uint16_t)0;
          break;
        default:
          dst[off] = valid ? __ldg(src + off) : (unsigned char)0;
          break;
      }
    }
  }
  pdl_launch_dependents();
}

}  // namespace mas
