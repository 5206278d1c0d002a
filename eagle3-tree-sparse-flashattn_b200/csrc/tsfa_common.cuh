// Shared device helpers of libtsfa: mask decoding, CSR lookups, status words.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tsfa.h"

namespace tsfa {

constexpr int kSmCount = 148;  // B200: 2 dies x 74 SMs
// Limit of the kernels' bounded waits unless a launch asks for a shorter one.
constexpr unsigned long long kDefaultWaitLimitNs = 1000000000ull;

// Layout of the TSFA_SYNC_BYTES region at the start of every workspace (int32 words).
//   [0]     device status (TSFA_OK or TSFA_ERR_DEVICE_TIMEOUT)
//   [1..3]  where a timed-out wait gave up: site, tile, CTA
//   [16]    arrival counter of the metadata builder's last-CTA emit
//   [64..]  the forward's global-merge counters, two per group: arrivals,
//           departures
constexpr int kSyncStatusWord = 0;
constexpr int kSyncTicketBase = 16;
constexpr int kSyncMergeBase = 64;
constexpr int kSyncWordsPerGroup = 2;
constexpr int kSyncMergeGroups = (TSFA_SYNC_BYTES / 4 - kSyncMergeBase) / kSyncWordsPerGroup;  // 480

// Records the text of a failing CUDA runtime call for tsfa_last_error() and
// maps it to TSFA_ERR_CUDA.
int record_cuda_error(cudaError_t e, const char* where);
#define TSFA_CUDA_CHECK(call)                                            \
  do {                                                                   \
    cudaError_t e_ = (call);                                             \
    if (e_ != cudaSuccess) return ::tsfa::record_cuda_error(e_, #call);  \
  } while (0)

__host__ __device__ inline int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline int cdiv(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Tensor.to(torch.bool) on one element: nonzero is visible; for floating types
// +-0 is invisible and NaN is visible (only the sign bit is ignored).
__device__ __forceinline__ bool mask_elem_visible(const char* row, int64_t col, int dtype) {
  switch (dtype) {
    case TSFA_MASK_B8: return reinterpret_cast<const uint8_t*>(row)[col] != 0;
    case TSFA_MASK_I16: return reinterpret_cast<const uint16_t*>(row)[col] != 0;
    case TSFA_MASK_I32: return reinterpret_cast<const uint32_t*>(row)[col] != 0;
    case TSFA_MASK_I64: return reinterpret_cast<const unsigned long long*>(row)[col] != 0ull;
    case TSFA_MASK_F16:
    case TSFA_MASK_BF16: return (reinterpret_cast<const uint16_t*>(row)[col] & 0x7fffu) != 0;
    case TSFA_MASK_F32: return (reinterpret_cast<const uint32_t*>(row)[col] & 0x7fffffffu) != 0;
    case TSFA_MASK_F64:
      return (reinterpret_cast<const unsigned long long*>(row)[col] & 0x7fffffffffffffffull) != 0ull;
    default: return false;
  }
}

__host__ __device__ inline int mask_elem_bytes(int dtype) {
  switch (dtype) {
    case TSFA_MASK_B8: return 1;
    case TSFA_MASK_I16: case TSFA_MASK_F16: case TSFA_MASK_BF16: return 2;
    case TSFA_MASK_I32: case TSFA_MASK_F32: return 4;
    case TSFA_MASK_I64: case TSFA_MASK_F64: return 8;
    default: return 0;
  }
}

// Metadata pointers as seen by the forward kernels.
struct MetaView {
  const int32_t* row_ptr;
  const int32_t* col_idx;
  const int8_t* blk_type;
  const int32_t* payload;
  const int32_t* offset;
  int n_q_blocks, n_tree_blocks, block_m, block_n;
  // Per-batch trees: elements between batch element b's metadata set and
  // b + 1's (row_ptr / col_idx, blk_type and offset / payload); all zero
  // when one tree serves every batch element.
  int64_t rp_bstride, tile_bstride, payload_bstride;
};

// Strides between consecutive masks / metadata sets of a per-batch build:
// the mask in bytes, the outputs in elements (row_ptr, the tile arrays,
// the payload).
struct MetaBatch {
  int64_t mask_bytes = 0, rp = 0, tile = 0, payload = 0;
};

// Paged K/V: copy the tree keys' K and V (keys prefix_len .. prefix_len + T - 1
// of every (batch, kv-head)) from the page pools into dense [B][Hkv][T][D]
// buffers; keys past kv_len, past a batch element's page list or on a page
// id outside the pool read as zeros.
struct TreeGather {
  const char* k_pages;
  const char* v_pages;
  int64_t ks[4], vs[4];  // element strides (page, token, head, dim)
  int page_shift, num_pages;
  const int32_t* page_indptr;
  const int32_t* page_indices;
  int B, Hkv, T, D, prefix_len, kv_len;
  char* tree_k;
  char* tree_v;
  int ctas;  // CTAs of the gather role
};

// The metadata set of batch element b.
__host__ __device__ __forceinline__ MetaView meta_of_batch(const MetaView& m, int b) {
  MetaView r = m;
  r.row_ptr += b * m.rp_bstride;
  r.col_idx += b * m.tile_bstride;
  r.blk_type += b * m.tile_bstride;
  r.offset += b * m.tile_bstride;
  r.payload += b * m.payload_bstride;
  return r;
}

// Debug builds (-DTSFA_DEBUG) check every metadata index and value the
// forward reads before using it: row_ptr order and range, col_idx against
// n_tree_blocks, blk_type against the two codes, mixed_mask_offset and the
// payload word against the payload the CSR can address (nnz * W words).  A
// failed check records TSFA_ERR_DEVICE_BOUNDS in the workspace status block
// (status[1] = the check, status[2] = the index, status[3] = the CTA) and the
// tile is skipped as if it were ZERO: no access outside the metadata is made.
// Release builds compile none of it.
enum BoundsCheck : int {
  kCheckRowPtr = 101, kCheckColIdx = 102, kCheckBlkType = 103, kCheckOffset = 104, kCheckPayloadWord = 105
};
#ifdef TSFA_DEBUG
__device__ __noinline__ inline void bounds_report(int* status, int check, long long index) {
  if (status && atomicCAS(status, 0, TSFA_ERR_DEVICE_BOUNDS) == 0) {
    status[1] = check;
    status[2] = (int)index;
    status[3] = (int)(blockIdx.y * gridDim.x + blockIdx.x);
  }
}
// nnz of the metadata set, after checking that it fits the tile grid.
__device__ __forceinline__ int checked_nnz(const MetaView& mv, int* status) {
  const int nnz = __ldg(mv.row_ptr + mv.n_q_blocks);
  if (nnz < 0 || (long long)nnz > (long long)mv.n_q_blocks * mv.n_tree_blocks) {
    bounds_report(status, kCheckRowPtr, mv.n_q_blocks);
    return -1;
  }
  return nnz;
}
// CSR row qb spans [lo, hi) inside [0, nnz).
__device__ __forceinline__ bool row_ok(const MetaView& mv, int qb, int lo, int hi, int* status) {
  const int nnz = checked_nnz(mv, status);
  if (qb < 0 || qb >= mv.n_q_blocks || nnz < 0 || lo < 0 || hi < lo || hi > nnz) {
    bounds_report(status, kCheckRowPtr, qb);
    return false;
  }
  return true;
}
#endif

// Entry index of tree block `tb` in CSR row `qb` (col_idx is ascending within a
// row: the reference appends tb in increasing order, tsfa.py:108-120), or -1.
__device__ __forceinline__ int csr_find(const MetaView& mv, int qb, int tb, int* dbg_status = nullptr) {
  int lo = __ldg(mv.row_ptr + qb), hi = __ldg(mv.row_ptr + qb + 1) - 1;
#ifdef TSFA_DEBUG
  if (!row_ok(mv, qb, lo, hi + 1, dbg_status)) return -1;
#endif
  while (lo <= hi) {
    int mid = (lo + hi) >> 1;
    int c = __ldg(mv.col_idx + mid);
#ifdef TSFA_DEBUG
    if (c < 0 || c >= mv.n_tree_blocks) {
      bounds_report(dbg_status, kCheckColIdx, mid);
      return -1;
    }
#endif
    if (c == tb) return mid;
    if (c < tb) lo = mid + 1; else hi = mid - 1;
  }
  return -1;
}

// Visibility bits of tree row `t` for tree columns [c0, c0 + nbits), nbits <= 64,
// clipped to the tree length T: bit i <-> column c0 + i.  Walks the CSR row of
// t's q-block and decodes FULL tiles as all-ones and MIXED tiles from their
// row-major bitset (bit (r * BN + c) of the payload at offset[ridx], as in
// tsfa.py:313-318).
__device__ __forceinline__ unsigned long long tree_row_bits(const MetaView& mv, int t, int c0, int nbits,
                                                            int T, int* dbg_status = nullptr) {
  unsigned long long bits = 0ull;
  const int BM = mv.block_m, BN = mv.block_n;
  const int qb = t / BM, rl = t - qb * BM;
  int c1 = min(c0 + nbits, T);
  if (c1 <= c0) return 0ull;
  for (int tb = c0 / BN; tb * BN < c1; ++tb) {
    int idx = csr_find(mv, qb, tb, dbg_status);
    if (idx < 0) continue;
    int cs = max(c0, tb * BN), ce = min(c1, tb * BN + BN);
    int len = ce - cs;
    if (len <= 0) continue;
    int dst = cs - c0;
    const int type = __ldg(mv.blk_type + idx);
#ifdef TSFA_DEBUG
    if (type != TSFA_FULL_BLOCK && type != TSFA_MIXED_BLOCK) {
      bounds_report(dbg_status, kCheckBlkType, idx);
      continue;
    }
#endif
    if (type == TSFA_FULL_BLOCK) {
      unsigned long long ones = (len >= 64) ? ~0ull : ((1ull << len) - 1ull);
      bits |= ones << dst;
    } else {
      const int off = __ldg(mv.offset + idx);
#ifdef TSFA_DEBUG
      const long long W = ((long long)BM * BN + 31) / 32;
      const int nnz = checked_nnz(mv, dbg_status);
      if (off < 0 || nnz < 0 || (long long)off + W > (long long)nnz * W) {
        bounds_report(dbg_status, kCheckOffset, idx);
        continue;
      }
#endif
      const int32_t* words = mv.payload + off;
      long long bitpos = (long long)rl * BN + (cs - tb * BN);
      while (len > 0) {
        int w = (int)(bitpos >> 5), sh = (int)(bitpos & 31);
#ifdef TSFA_DEBUG
        if ((long long)w >= W) {
          bounds_report(dbg_status, kCheckPayloadWord, w);
          break;
        }
#endif
        int take = min(32 - sh, len);
        unsigned int v = ((unsigned int)__ldg(words + w)) >> sh;
        if (take < 32) v &= (1u << take) - 1u;
        bits |= (unsigned long long)v << dst;
        dst += take;
        bitpos += take;
        len -= take;
      }
    }
  }
  return bits;
}

}  // namespace tsfa
