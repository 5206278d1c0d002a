// Forward-pass plan shared by the host launcher and the kernel.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tsfa_common.cuh"

namespace tsfa {

// Work decomposition.  The G query heads of one kv-head are folded into the
// row dimension: a row tile holds t_per_tile tree rows x G heads, row
// r = g + G * t_local, so K/V are read once per tile for all of them.  A
// "group" is one (batch, kv-head, row tile); its key tiles -- prefix first,
// then the tree tiles its CSR rows touch -- are split evenly over n_splits
// CTAs.  The splits' partial (O, m, l) are merged with log-sum-exp weights,
// so nothing but the output and (in the global mode) the partials reach
// global memory.  Two ways to merge:
//   cluster  the splits of a group form one thread-block cluster and exchange
//            rows through distributed shared memory (bulk copies);
//   global   the grid is a cooperative launch (every CTA resident at once) of
//            up to one CTA per SM, more splits than cluster co-scheduling
//            allows; each split bulk-stores its rows to `partials`, counts
//            itself in on the group's arrival counter, and each CTA merges
//            its slice of rows from bulk loads of every split's partial.
struct FwdParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t sq[4], sk[4], sv[4], so[4];
  int B, Hq, Hkv, G, T, kv_len, P;
  float scale_log2;  // sm_scale * log2(e): scores live in the exp2 domain
  MetaView mv;
  int t_per_tile;      // tree rows per row tile: floor(128 / G)
  int n_row_tiles;     // row tiles per (batch, kv-head)
  int n_prefix_tiles;  // cdiv(P, 128)
  int n_tree_tiles;    // cdiv(T, 128)
  int n_splits;        // splits per group (1 = no split)
  int pair;            // 1 (n_splits == 1, contiguous K/V): a CTA takes two row tiles, sharing each K/V tile
  int global_merge;    // 1: merge through `partials` (cooperative launch); 0: through the cluster
  uint8_t* partials;   // global merge: [group][split][128 rows][2 D + 16 bytes]: O fp16 (scaled per half row),
                       // then m, l0, l1 fp32 and the halves' scale exponents int16
  unsigned int* gsync; // global merge: per group {arrivals, departures}, left at zero
  int* status;         // workspace status block (device-side timeouts)
  // Limit of every bounded wait in the kernel (kWaitLimitNs unless a test
  // shortens it) and a test-only fault: TSFA_FAULT_WITHHOLD_TREE_LIST makes
  // the tree-list warp never publish its list, so the waits on it run out.
  unsigned long long wait_limit_ns;
  int fault;
  // Paged K/V (paged = 1): the K / V maps cover page pools [page][token][head][dim];
  // key n of batch element b is token n % page_size of page
  // page_indices[page_indptr[b] + n / page_size].
  int paged;
  int page_shift;            // log2(page_size)
  int num_pages;
  const int32_t* page_indptr;   // [B + 1]
  const int32_t* page_indices;
  const void* tree_k;           // [B][Hkv][T][D]: the tree keys' K / V, gathered by the metadata kernel
  const void* tree_v;
};

constexpr int kMaxTreeTileList = 64;  // tree tiles per row tile: T <= 8192
constexpr int kMaxSplits = 16;         // largest (non-portable) cluster

}  // namespace tsfa
