// Forward-pass plan shared by the host launcher and the kernels.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "tsfa_common.cuh"

namespace tsfa {

// Work decomposition.  The G query heads of one kv-head are folded into the
// row dimension: folded row f = t * G + g (t-major, so one row tile covers few
// tree rows and the tree tiles it needs stay sparse).  A "group" is one
// (batch, kv-head, row tile); its keys -- prefix tiles then tree tiles, in
// kKeys-wide steps -- are split into `n_splits` contiguous ranges, one CTA
// each.  With more than one split every CTA writes an unnormalised partial
// (O, m, l) and the last CTA of the group merges them (log-sum-exp).
struct FwdParams {
  const void* q;
  const void* k;
  const void* v;
  void* o;
  int64_t sq[4], sk[4], sv[4], so[4];
  int B, Hq, Hkv, G, T, kv_len, P;
  float scale_log2;  // sm_scale * log2(e): scores live in the exp2 domain
  MetaView mv;
  int rows_per_unit;    // G * T
  int t_per_tile;       // tree rows per row tile (tcgen05 kernel: floor(128 / G))
  int n_row_tiles;      // row tiles per (batch, kv-head)
  int n_prefix_tiles;   // cdiv(P, kKeys)
  int n_tree_tiles;     // cdiv(T, kKeys)
  int n_splits;
  int tiles_per_split;
  float* part_o;        // [groups * n_splits, kRows, D]
  float2* part_ml;      // [groups * n_splits, kRows]  (m in exp2 domain, l)
  unsigned int* tickets;  // [groups]
  int* status;
};

constexpr int kMaxTreeTileList = 256;  // tree tiles per row tile (T <= 16384 with 64-key tiles)
constexpr int kMaxSplits = 32;

}  // namespace tsfa
