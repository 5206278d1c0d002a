// libtsfa C ABI: argument checks, work plans, workspace layouts, launches.
//
// Mirrors the launch wrapper run_tree_sparse_kernel
// (eagle_tree_sparse_bridge.py:76-159): the same shape assertions
// (bridge.py:85-89), P = kv_len - q_len with a ValueError when negative
// (bridge.py:91-93), metadata from the mask (bridge.py:95-100) and the forward
// over every (batch, q-head, tree row) -- but the metadata is built on the
// device and nothing is copied through the host.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "tsfa_fwd.cuh"

namespace tsfa {
size_t meta_area_bytes(int64_t ntiles, int64_t W);
int meta_build_launch(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                      int32_t block_m, int32_t block_n, const TsfaMeta& out, unsigned int* ticket, char* area,
                      size_t area_bytes, cudaStream_t stream);
int meta_build_batched_launch(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                              int32_t block_m, int32_t block_n, const TsfaMeta& out, int nbatch, const MetaBatch& mb,
                              unsigned int* ticket, char* area, size_t area_bytes, cudaStream_t stream,
                              const TreeGather* gather);
int fwd_tc_launch(const FwdParams& p, int head_dim, int dtype, bool after_meta, cudaStream_t stream);
bool fwd_tc_can_cooperate(int head_dim, int dtype, int ctas);
int fwd_tc_pick_splits(int head_dim, int dtype, int groups, int want);
int pack_tile_launch(const void* tile, int dtype, int64_t row_stride, int rows, int cols, int32_t* out,
                     cudaStream_t stream);

extern thread_local uint64_t g_wait_limit_ns;
extern thread_local int g_fault;
extern thread_local int32_t g_last_plan[4];
extern thread_local int g_force_merge;

namespace {

constexpr int kRowTile = 128;  // MMA M / TMEM lanes: folded (t, g) rows per CTA
constexpr int kKeyTile = 128;  // keys per step
constexpr int kCtasPerSm = 1;  // ~193 KB of shared memory and 512 TMEM columns per CTA

// ---------------------------------------------------------------- metadata
struct MetaLayout {
  TsfaMetaDims d;
  size_t off_row_ptr, off_col, off_type, off_payload, off_offset, off_counts, off_area, area_bytes, end;
};

// `nb` metadata sets back to back in each array (per-batch trees; set i of
// row_ptr at element i * (n_q_blocks + 1), of the tile arrays at i *
// tile_capacity, of the payload at i * payload_capacity, counts at 2 i).
MetaLayout meta_layout(int64_t q_len, int block_m, int block_n, size_t base, int64_t nb = 1) {
  MetaLayout L;
  tsfa_meta_dims((int32_t)q_len, block_m, block_n, &L.d);
  size_t o = align_up(base, 256);
  L.off_row_ptr = o;
  o = align_up(o + (size_t)(nb * (L.d.n_q_blocks + 1)) * 4, 256);
  L.off_col = o;
  o = align_up(o + (size_t)(nb * L.d.tile_capacity) * 4, 256);
  L.off_type = o;
  o = align_up(o + (size_t)(nb * L.d.tile_capacity), 256);
  L.off_payload = o;
  o = align_up(o + (size_t)(nb * L.d.payload_capacity) * 4, 256);
  L.off_offset = o;
  o = align_up(o + (size_t)(nb * L.d.tile_capacity) * 4, 256);
  L.off_counts = o;
  o = align_up(o + (size_t)nb * 8, 256);
  L.off_area = o;
  L.area_bytes = meta_area_bytes(L.d.tile_capacity, L.d.words_per_tile);
  o = align_up(o + L.area_bytes, 256);
  L.end = o;
  return L;
}

// ---------------------------------------------------------------- forward
struct FwdPlan {
  int G, t_per_tile, n_row_tiles, groups, n_prefix_tiles, n_tree_tiles;
  int wide;              // splits per group of the global merge (one CTA per SM), 1 = none
  size_t off_partials;   // global merge: the splits' partial rows
  size_t end;            // workspace bytes: status block [+ partials]
};

int check_fwd_args(const TsfaFwdArgs* a) {
  if (!a) return TSFA_ERR_VALUE;
  if (a->batch < 0 || a->num_heads <= 0 || a->num_kv_heads <= 0 || a->q_len < 0 || a->kv_len < 0)
    return TSFA_ERR_ASSERT;
  if (a->num_heads % a->num_kv_heads != 0) return TSFA_ERR_ASSERT;  // kv_h = h // G must stay in range
  if (a->num_heads / a->num_kv_heads > kRowTile) return TSFA_ERR_UNSUPPORTED;  // one row tile holds a whole group
  if (a->prefix_len < 0 || a->prefix_len > a->kv_len) return TSFA_ERR_VALUE;  // bridge.py:91-93
  if (a->head_dim != 64 && a->head_dim != 128) return TSFA_ERR_UNSUPPORTED;
  if (a->dtype != TSFA_DTYPE_BF16 && a->dtype != TSFA_DTYPE_F16) return TSFA_ERR_UNSUPPORTED;
  if (a->block_m <= 0 || a->block_n <= 0) return TSFA_ERR_VALUE;
  if (a->batch * (int64_t)a->num_kv_heads > 65535) return TSFA_ERR_UNSUPPORTED;
  if (cdiv64(a->q_len, kKeyTile) > kMaxTreeTileList) return TSFA_ERR_UNSUPPORTED;
  const int64_t* st[4] = {a->q_stride, a->k_stride, a->v_stride, a->o_stride};
  for (int i = 0; i < 4; ++i) {
    if (st[i][3] != 1) return TSFA_ERR_UNSUPPORTED;
    for (int j = 0; j < 3; ++j)
      if (st[i][j] % 8 != 0) return TSFA_ERR_UNSUPPORTED;  // 16-byte aligned rows
  }
  const void* ptrs[4] = {a->q, a->k, a->v, a->o};
  for (int i = 0; i < 4; ++i)
    if ((reinterpret_cast<uintptr_t>(ptrs[i]) & 15u) != 0) return TSFA_ERR_UNSUPPORTED;
  return TSFA_OK;
}

// with_partials: reserve the global merge's partial rows (tsfa_fwd and the
// whole op); the per-batch op's forward merges through clusters, so its
// workspace holds none.
FwdPlan fwd_plan(const TsfaFwdArgs* a, size_t base, bool with_partials) {
  FwdPlan P;
  P.G = a->num_heads / a->num_kv_heads;
  P.t_per_tile = kRowTile / P.G;  // a row tile holds t_per_tile tree rows x G heads
  P.n_row_tiles = cdiv(a->q_len, P.t_per_tile);
  P.groups = a->batch * a->num_kv_heads * P.n_row_tiles;
  P.n_prefix_tiles = cdiv(a->prefix_len, kKeyTile);
  P.n_tree_tiles = cdiv(a->q_len, kKeyTile);
  // the global merge: as many splits as key tiles allow with one CTA per SM
  const int n_tiles = P.n_prefix_tiles + P.n_tree_tiles;
  P.wide = P.groups > 0 ? std::min(std::min(kMaxSplits, n_tiles), kCtasPerSm * kSmCount / P.groups) : 1;
  if (!with_partials || P.wide < 2 || P.groups > kSyncMergeGroups) P.wide = 1;
  P.off_partials = align_up(base, 256);
  const size_t row_bytes = (size_t)a->head_dim * 2 + 16;  // O in fp16, then m, l0, l1 and two scale exponents
  P.end = P.off_partials + (P.wide > 1 ? (size_t)P.groups * P.wide * kRowTile * row_bytes : 0);
  P.end = align_up(P.end, 256);
  return P;
}

// Split-KV width: enough clusters of CTAs to fill the SMs in one wave, capped
// by the key tiles and by what the device can co-schedule; cached per
// (device, shape class) because the occupancy query is not free.
int pick_splits(const TsfaFwdArgs* a, const FwdPlan& P) {
  const int n_tiles = P.n_prefix_tiles + P.n_tree_tiles;
  const int want = std::min(std::min(kMaxSplits, n_tiles), std::max(1, kCtasPerSm * kSmCount / std::max(P.groups, 1)));
  if (want < 2) return 1;
  static std::mutex mu;
  static std::map<std::tuple<int, int, int, int, int>, int> cache;
  int dev = 0;
  cudaGetDevice(&dev);
  const auto key = std::make_tuple(dev, a->head_dim, a->dtype, P.groups, want);
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
  }
  const int ns = fwd_tc_pick_splits(a->head_dim, a->dtype, P.groups, want);
  std::lock_guard<std::mutex> lk(mu);
  cache[key] = ns;
  return ns;
}

// after_meta: the metadata comes from the kernel launched just before on the
// same stream; the forward overlaps it (programmatic dependent launch).
int fwd_launch(const TsfaFwdArgs* a, const MetaView& mv, char* ws, const FwdPlan& P, bool after_meta,
               cudaStream_t stream, const TsfaPagedKV* kv = nullptr, const void* tree_k = nullptr,
               const void* tree_v = nullptr) {
  if (P.groups == 0) return TSFA_OK;  // q_len == 0 or batch == 0: nothing to write
  FwdParams p;
  p.q = a->q;
  p.k = a->k;
  p.v = a->v;
  p.o = a->o;
  for (int i = 0; i < 4; ++i) {
    p.sq[i] = a->q_stride[i];
    p.sk[i] = a->k_stride[i];
    p.sv[i] = a->v_stride[i];
    p.so[i] = a->o_stride[i];
  }
  p.B = a->batch;
  p.Hq = a->num_heads;
  p.Hkv = a->num_kv_heads;
  p.G = P.G;
  p.T = a->q_len;
  p.kv_len = a->kv_len;
  p.P = a->prefix_len;
  p.scale_log2 = a->sm_scale * 1.4426950408889634f;
  p.mv = mv;
  p.t_per_tile = P.t_per_tile;
  p.n_row_tiles = P.n_row_tiles;
  p.n_prefix_tiles = P.n_prefix_tiles;
  p.n_tree_tiles = P.n_tree_tiles;
  // The global merge (a cooperative launch of one CTA per SM) when it gives
  // more splits than cluster co-scheduling and the workspace holds its
  // partial rows (tsfa_fwd and the whole op; not the per-batch op).  Behind
  // the metadata kernel the cooperative launch also carries the programmatic
  // serialization attribute: its CTAs start beside the metadata kernel, and
  // only the tree tiles wait for it.
  const int ns_cluster = pick_splits(a, P);
  p.global_merge = g_force_merge != 1 && g_force_merge != 3 && P.wide > ns_cluster &&
                   fwd_tc_can_cooperate(a->head_dim, a->dtype, P.groups * P.wide) ? 1 : 0;
  p.n_splits = p.global_merge ? P.wide : (g_force_merge == 3 ? 1 : ns_cluster);
  // Row-tile pairs: without a split, when even the pairs fill every SM at
  // least once (a CTA then streams each K/V tile once for 256 rows).  With
  // head_dim 128 the pairs round P once on tree tiles: only where every row
  // sees >= 1024 prefix keys besides its tree keys.
  const int64_t pairs = (int64_t)a->batch * a->num_kv_heads * ((P.n_row_tiles + 1) / 2);
  const bool pair_ok = pairs >= kSmCount && (a->head_dim == 64 || a->prefix_len >= 1024);
  p.pair = (p.n_splits == 1 && !kv && P.n_row_tiles >= 2 && (pair_ok || g_force_merge == 3)) ? 1 : 0;
  p.partials = reinterpret_cast<uint8_t*>(ws + P.off_partials);
  p.gsync = reinterpret_cast<unsigned int*>(ws) + kSyncMergeBase;
  p.status = reinterpret_cast<int*>(ws);
  p.wait_limit_ns = g_wait_limit_ns ? g_wait_limit_ns : kDefaultWaitLimitNs;
  p.fault = g_fault;
  p.paged = 0;
  p.page_shift = 0;
  p.num_pages = 0;
  p.page_indptr = p.page_indices = nullptr;
  p.tree_k = tree_k;
  p.tree_v = tree_v;
  if (kv) {  // K/V maps over the page pools: strides (page, token, head, dim)
    p.paged = 1;
    p.k = kv->k_pages;
    p.v = kv->v_pages;
    for (int i = 0; i < 4; ++i) {
      p.sk[i] = kv->k_stride[i];
      p.sv[i] = kv->v_stride[i];
    }
    int shift = 0;
    while ((1 << shift) < kv->page_size) ++shift;
    p.page_shift = shift;
    p.num_pages = kv->num_pages;
    p.page_indptr = kv->page_indptr;
    p.page_indices = kv->page_indices;
  }
  auto record_plan = [&] {
    g_last_plan[0] = p.n_splits;
    g_last_plan[1] = p.pair ? 3 : p.n_splits <= 1 ? 0 : (p.global_merge ? 2 : 1);
    g_last_plan[2] = p.pair ? (P.n_row_tiles + 1) / 2 : P.n_row_tiles * p.n_splits;
    g_last_plan[3] = a->batch * a->num_kv_heads;
  };
  record_plan();
  // (the test fault stands for a refusal by the device: nothing launched)
  int st = (g_fault == TSFA_FAULT_REFUSE_COOPERATIVE && p.global_merge)
               ? TSFA_ERR_CUDA
               : fwd_tc_launch(p, a->head_dim, a->dtype, after_meta, stream);
  if (st == TSFA_ERR_CUDA && p.global_merge) {
    // The device refused the cooperative launch at run time (another context
    // holding SMs, say; nothing was launched): merge through clusters, which
    // needs only each cluster co-resident.
    cudaGetLastError();
    p.global_merge = 0;
    p.n_splits = ns_cluster;
    record_plan();
    st = fwd_tc_launch(p, a->head_dim, a->dtype, after_meta, stream);
  }
  return st;
}

}  // namespace
}  // namespace tsfa

namespace tsfa {
namespace {
thread_local char g_last_error[256] = "";
}
// Test-only settings of the launches made by the calling thread
// (tsfa_debug_inject): the bounded waits' limit and an injected fault.
thread_local uint64_t g_wait_limit_ns = 0;  // 0: the kernels' own limit
thread_local int g_fault = TSFA_FAULT_NONE;
// The calling thread's last forward launch: splits per row tile, merge mode
// (0 none, 1 cluster, 2 global), grid x, grid y (tsfa_debug_last_plan).
thread_local int32_t g_last_plan[4] = {0, 0, 0, 0};
// Merge mode of the calling thread's later forward launches
// (tsfa_debug_force_merge): 0 the library's choice, 1 the cluster merge,
// 3 one split with row-tile pairs (where the shapes allow them).
thread_local int g_force_merge = 0;
int record_cuda_error(cudaError_t e, const char* where) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%d)", where, cudaGetErrorString(e), (int)e);
  return TSFA_ERR_CUDA;
}
}  // namespace tsfa

using namespace tsfa;

extern "C" const char* tsfa_last_error(void) { return g_last_error; }

extern "C" const char* tsfa_status_string(int status) {
  switch (status) {
    case TSFA_OK: return "ok";
    case TSFA_ERR_VALUE: return "invalid value (mask shape, block size or lengths)";
    case TSFA_ERR_ASSERT: return "shape mismatch between query/key/value";
    case TSFA_ERR_UNSUPPORTED: return "unsupported head_dim, dtype or memory layout";
    case TSFA_ERR_WORKSPACE: return "workspace missing or too small";
    case TSFA_ERR_CUDA: return "CUDA error";
    case TSFA_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case TSFA_ERR_DEVICE_BOUNDS: return "a metadata index failed its device-side bounds check (debug build)";
    default: return "unknown status";
  }
}

extern "C" int tsfa_abi_version(void) { return TSFA_ABI_VERSION; }

extern "C" int tsfa_meta_dims(int32_t q_len, int32_t block_m, int32_t block_n, TsfaMetaDims* out) {
  if (!out) return TSFA_ERR_VALUE;
  if (block_m <= 0 || block_n <= 0 || q_len < 0) return TSFA_ERR_VALUE;  // tsfa.py:87-88
  out->n_q_blocks = cdiv64(q_len, block_m);
  out->n_tree_blocks = cdiv64(q_len, block_n);
  out->words_per_tile = cdiv64((int64_t)block_m * block_n, 32);
  out->tile_capacity = out->n_q_blocks * out->n_tree_blocks;
  out->payload_capacity = out->tile_capacity * out->words_per_tile;
  return TSFA_OK;
}

extern "C" int tsfa_meta_workspace_bytes(int32_t q_len, int32_t block_m, int32_t block_n, size_t* bytes) {
  TsfaMetaDims d;
  const int st = tsfa_meta_dims(q_len, block_m, block_n, &d);
  if (st != TSFA_OK) return st;
  if (!bytes) return TSFA_ERR_VALUE;
  *bytes = TSFA_SYNC_BYTES + meta_area_bytes(d.tile_capacity, d.words_per_tile);
  return TSFA_OK;
}

static int meta_checks(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                       int32_t block_m, int32_t block_n, TsfaMetaDims* d) {
  const int st = tsfa_meta_dims(q_len, block_m, block_n, d);
  if (st != TSFA_OK) return st;
  if (mask_elem_bytes(mask_dtype) == 0) return TSFA_ERR_UNSUPPORTED;
  if (d->words_per_tile > (1ll << 24) || d->payload_capacity > (1ll << 31) - 1) return TSFA_ERR_UNSUPPORTED;
  if (q_len > 0 && (!tree_mask || mask_row_stride < q_len)) return TSFA_ERR_VALUE;
  return TSFA_OK;
}

extern "C" int tsfa_meta_build(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                               int32_t block_m, int32_t block_n, const TsfaMeta* out, void* workspace,
                               size_t workspace_bytes, void* stream) {
  TsfaMetaDims d;
  const int st = meta_checks(tree_mask, mask_dtype, mask_row_stride, q_len, block_m, block_n, &d);
  if (st != TSFA_OK) return st;
  if (!out || !out->row_ptr || !out->counts) return TSFA_ERR_VALUE;
  if (d.tile_capacity > 0 && (!out->col_idx || !out->blk_type || !out->mixed_mask_offset)) return TSFA_ERR_VALUE;
  size_t need = 0;
  tsfa_meta_workspace_bytes(q_len, block_m, block_n, &need);
  if (!workspace || workspace_bytes < need) return TSFA_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  return meta_build_launch(tree_mask, mask_dtype, mask_row_stride, q_len, block_m, block_n, *out,
                           reinterpret_cast<unsigned int*>(ws) + kSyncTicketBase, ws + TSFA_SYNC_BYTES,
                           workspace_bytes - TSFA_SYNC_BYTES, static_cast<cudaStream_t>(stream));
}

extern "C" int tsfa_pack_block_mask(const void* tile, int32_t mask_dtype, int64_t row_stride, int32_t rows,
                                    int32_t cols, int32_t* out_words, void* stream) {
  if (rows < 0 || cols < 0) return TSFA_ERR_VALUE;
  if (mask_elem_bytes(mask_dtype) == 0) return TSFA_ERR_UNSUPPORTED;
  if ((int64_t)rows * cols > (1ll << 31) - 1) return TSFA_ERR_UNSUPPORTED;
  if ((int64_t)rows * cols > 0 && (!tile || !out_words || row_stride < cols)) return TSFA_ERR_VALUE;
  return pack_tile_launch(tile, mask_dtype, row_stride, rows, cols, out_words, static_cast<cudaStream_t>(stream));
}

extern "C" int tsfa_fwd_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes) {
  const int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  if (!bytes) return TSFA_ERR_VALUE;
  *bytes = fwd_plan(args, TSFA_SYNC_BYTES, true).end;
  return TSFA_OK;
}

extern "C" int tsfa_fwd(const TsfaFwdArgs* args, void* workspace, size_t workspace_bytes, void* stream) {
  const int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  if (args->n_q_blocks != cdiv(args->q_len, args->block_m) || args->n_tree_blocks != cdiv(args->q_len, args->block_n))
    return TSFA_ERR_VALUE;
  if (args->q_len > 0 && (!args->row_ptr || !args->col_idx || !args->blk_type)) return TSFA_ERR_VALUE;
  const FwdPlan P = fwd_plan(args, TSFA_SYNC_BYTES, true);
  if (!workspace || workspace_bytes < P.end) return TSFA_ERR_WORKSPACE;
  MetaView mv;
  mv.row_ptr = args->row_ptr;
  mv.col_idx = args->col_idx;
  mv.blk_type = args->blk_type;
  mv.payload = args->mixed_mask_payload;
  mv.offset = args->mixed_mask_offset;
  mv.n_q_blocks = args->n_q_blocks;
  mv.n_tree_blocks = args->n_tree_blocks;
  mv.block_m = args->block_m;
  mv.block_n = args->block_n;
  mv.rp_bstride = mv.tile_bstride = mv.payload_bstride = 0;  // one tree for every batch element
  char* ws = static_cast<char*>(workspace);
  return fwd_launch(args, mv, ws, P, false, static_cast<cudaStream_t>(stream));
}

// Whole-op workspace: [status block + K1 arrival counter | the global merge's
// partial rows | metadata buffers + K1 area].
static void run_layout(const TsfaFwdArgs* a, FwdPlan* P, MetaLayout* L) {
  *P = fwd_plan(a, TSFA_SYNC_BYTES, true);
  *L = meta_layout(a->q_len, a->block_m, a->block_n, P->end);
}

extern "C" int tsfa_run_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes) {
  const int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  if (!bytes) return TSFA_ERR_VALUE;
  FwdPlan P;
  MetaLayout L;
  run_layout(args, &P, &L);
  *bytes = L.end;
  return TSFA_OK;
}

// Paged K/V: the whole-op workspace, then the tree keys' K and V gathered
// from the pages ([B][Hkv][T][D] each).  Returns the bytes needed.
static size_t paged_layout(const TsfaFwdArgs* a, const MetaLayout& L, size_t* off_tree, size_t* tree_bytes) {
  *tree_bytes = align_up((size_t)a->batch * a->num_kv_heads * a->q_len * a->head_dim * 2, 256);
  *off_tree = align_up(L.end, 256);
  return *off_tree + 2 * *tree_bytes;
}

extern "C" int tsfa_run_paged_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes) {
  const int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  if (!bytes) return TSFA_ERR_VALUE;
  FwdPlan P;
  MetaLayout L;
  run_layout(args, &P, &L);
  size_t o, t;
  *bytes = paged_layout(args, L, &o, &t);
  return TSFA_OK;
}

static int run_tree_sparse_impl(const TsfaFwdArgs* args, const void* tree_mask, int32_t mask_dtype,
                                int64_t mask_row_stride, void* workspace, size_t workspace_bytes, void* stream,
                                const TsfaPagedKV* kv) {
  int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  TsfaMetaDims d;
  st = meta_checks(tree_mask, mask_dtype, mask_row_stride, args->q_len, args->block_m, args->block_n, &d);
  if (st != TSFA_OK) return st;
  FwdPlan P;
  MetaLayout L;
  run_layout(args, &P, &L);
  size_t off_tree = 0, tree_bytes = 0;
  const size_t need = kv ? paged_layout(args, L, &off_tree, &tree_bytes) : L.end;
  if (!workspace || workspace_bytes < need) return TSFA_ERR_WORKSPACE;
  char* ws = static_cast<char*>(workspace);
  unsigned int* tickets = reinterpret_cast<unsigned int*>(ws) + kSyncTicketBase;
  TreeGather g{};
  if (kv) {
    g.k_pages = static_cast<const char*>(kv->k_pages);
    g.v_pages = static_cast<const char*>(kv->v_pages);
    for (int i = 0; i < 4; ++i) {
      g.ks[i] = kv->k_stride[i];
      g.vs[i] = kv->v_stride[i];
    }
    while ((1 << g.page_shift) < kv->page_size) ++g.page_shift;
    g.num_pages = kv->num_pages;
    g.page_indptr = kv->page_indptr;
    g.page_indices = kv->page_indices;
    g.B = args->batch;
    g.Hkv = args->num_kv_heads;
    g.T = args->q_len;
    g.D = args->head_dim;
    g.prefix_len = args->prefix_len;
    g.kv_len = args->kv_len;
    g.tree_k = ws + off_tree;
    g.tree_v = ws + off_tree + tree_bytes;
    const int64_t chunks = (int64_t)g.B * g.Hkv * g.T * (g.D / 8);
    g.ctas = (int)std::min<int64_t>(16, std::max<int64_t>(1, (chunks + 1023) / 1024));
  }
  TsfaMeta m;
  m.row_ptr = reinterpret_cast<int32_t*>(ws + L.off_row_ptr);
  m.col_idx = reinterpret_cast<int32_t*>(ws + L.off_col);
  m.blk_type = reinterpret_cast<int8_t*>(ws + L.off_type);
  m.mixed_mask_payload = reinterpret_cast<int32_t*>(ws + L.off_payload);
  m.mixed_mask_offset = reinterpret_cast<int32_t*>(ws + L.off_offset);
  m.counts = reinterpret_cast<int32_t*>(ws + L.off_counts);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = meta_build_batched_launch(tree_mask, mask_dtype, mask_row_stride, args->q_len, args->block_m, args->block_n, m,
                                 1, MetaBatch{}, tickets, ws + L.off_area, L.area_bytes, s, kv ? &g : nullptr);
  if (st != TSFA_OK) return st;
  MetaView mv;
  mv.row_ptr = m.row_ptr;
  mv.col_idx = m.col_idx;
  mv.blk_type = m.blk_type;
  mv.payload = m.mixed_mask_payload;
  mv.offset = m.mixed_mask_offset;
  mv.n_q_blocks = (int)d.n_q_blocks;
  mv.n_tree_blocks = (int)d.n_tree_blocks;
  mv.block_m = args->block_m;
  mv.block_n = args->block_n;
  mv.rp_bstride = mv.tile_bstride = mv.payload_bstride = 0;  // one tree for every batch element
  return fwd_launch(args, mv, ws, P, true, s, kv, kv ? g.tree_k : nullptr, kv ? g.tree_v : nullptr);
}

extern "C" int tsfa_run_tree_sparse(const TsfaFwdArgs* args, const void* tree_mask, int32_t mask_dtype,
                                    int64_t mask_row_stride, void* workspace, size_t workspace_bytes,
                                    void* stream) {
  return run_tree_sparse_impl(args, tree_mask, mask_dtype, mask_row_stride, workspace, workspace_bytes, stream,
                              nullptr);
}

// Paged K/V: the pools replace args->k / args->v; the dense arguments' checks
// run on a copy with those pointers and strides neutral.
extern "C" int tsfa_run_tree_sparse_paged(const TsfaFwdArgs* args, const TsfaPagedKV* kv, const void* tree_mask,
                                          int32_t mask_dtype, int64_t mask_row_stride, void* workspace,
                                          size_t workspace_bytes, void* stream) {
  if (!args || !kv) return TSFA_ERR_VALUE;
  TsfaFwdArgs a = *args;
  a.k = a.v = nullptr;
  for (int i = 0; i < 4; ++i) a.k_stride[i] = a.v_stride[i] = (i == 3) ? 1 : 0;
  if (kv->page_size < 8 || kv->page_size > (1 << 24) || (kv->page_size & (kv->page_size - 1)) != 0)
    return TSFA_ERR_UNSUPPORTED;
  if (kv->num_pages < 1) return TSFA_ERR_VALUE;
  const int64_t* st[2] = {kv->k_stride, kv->v_stride};
  for (int i = 0; i < 2; ++i) {
    if (st[i][3] != 1) return TSFA_ERR_UNSUPPORTED;
    for (int j = 0; j < 3; ++j)
      if (st[i][j] % 8 != 0 || st[i][j] < 0) return TSFA_ERR_UNSUPPORTED;  // 16-byte aligned rows (TMA)
  }
  if (((reinterpret_cast<uintptr_t>(kv->k_pages) | reinterpret_cast<uintptr_t>(kv->v_pages)) & 15u) != 0)
    return TSFA_ERR_UNSUPPORTED;
  if (!kv->k_pages || !kv->v_pages || !kv->page_indptr || !kv->page_indices) return TSFA_ERR_VALUE;
  return run_tree_sparse_impl(&a, tree_mask, mask_dtype, mask_row_stride, workspace, workspace_bytes, stream, kv);
}

// ---------------------------------------------------------------- per-batch trees
// Whole-op workspace with one metadata set per batch element.
static void run_layout_batched(const TsfaFwdArgs* a, FwdPlan* P, MetaLayout* L) {
  *P = fwd_plan(a, TSFA_SYNC_BYTES, false);
  *L = meta_layout(a->q_len, a->block_m, a->block_n, P->end, std::max<int64_t>(a->batch, 1));
}

extern "C" int tsfa_run_batched_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes) {
  const int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  if (!bytes) return TSFA_ERR_VALUE;
  FwdPlan P;
  MetaLayout L;
  run_layout_batched(args, &P, &L);
  *bytes = L.end;
  return TSFA_OK;
}

extern "C" int tsfa_run_tree_sparse_batched(const TsfaFwdArgs* args, const void* tree_masks, int32_t mask_dtype,
                                            int64_t mask_batch_stride, int64_t mask_row_stride, void* workspace,
                                            size_t workspace_bytes, void* stream) {
  int st = check_fwd_args(args);
  if (st != TSFA_OK) return st;
  TsfaMetaDims d;
  st = meta_checks(tree_masks, mask_dtype, mask_row_stride, args->q_len, args->block_m, args->block_n, &d);
  if (st != TSFA_OK) return st;
  // the masks are only read: a stride of 0 (one mask for every element) is fine
  if (mask_batch_stride < 0) return TSFA_ERR_VALUE;
  FwdPlan P;
  MetaLayout L;
  run_layout_batched(args, &P, &L);
  if (!workspace || workspace_bytes < L.end) return TSFA_ERR_WORKSPACE;
  if (args->batch == 0 || args->q_len == 0) return TSFA_OK;  // nothing to write
  char* ws = static_cast<char*>(workspace);
  unsigned int* tickets = reinterpret_cast<unsigned int*>(ws) + kSyncTicketBase;
  TsfaMeta m;
  m.row_ptr = reinterpret_cast<int32_t*>(ws + L.off_row_ptr);
  m.col_idx = reinterpret_cast<int32_t*>(ws + L.off_col);
  m.blk_type = reinterpret_cast<int8_t*>(ws + L.off_type);
  m.mixed_mask_payload = reinterpret_cast<int32_t*>(ws + L.off_payload);
  m.mixed_mask_offset = reinterpret_cast<int32_t*>(ws + L.off_offset);
  m.counts = reinterpret_cast<int32_t*>(ws + L.off_counts);
  MetaBatch mb;
  mb.mask_bytes = mask_batch_stride * mask_elem_bytes(mask_dtype);
  mb.rp = d.n_q_blocks + 1;
  mb.tile = d.tile_capacity;
  mb.payload = d.payload_capacity;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = meta_build_batched_launch(tree_masks, mask_dtype, mask_row_stride, args->q_len, args->block_m, args->block_n,
                                 m, args->batch, mb, tickets, ws + L.off_area, L.area_bytes, s, nullptr);
  if (st != TSFA_OK) return st;
  MetaView mv;
  mv.row_ptr = m.row_ptr;
  mv.col_idx = m.col_idx;
  mv.blk_type = m.blk_type;
  mv.payload = m.mixed_mask_payload;
  mv.offset = m.mixed_mask_offset;
  mv.n_q_blocks = (int)d.n_q_blocks;
  mv.n_tree_blocks = (int)d.n_tree_blocks;
  mv.block_m = args->block_m;
  mv.block_n = args->block_n;
  mv.rp_bstride = mb.rp;
  mv.tile_bstride = mb.tile;
  mv.payload_bstride = mb.payload;
  return fwd_launch(args, mv, ws, P, true, s);
}

extern "C" int tsfa_read_device_status_detail(void* workspace, void* stream, int32_t detail[4]) {
  if (!workspace || !detail) return TSFA_ERR_VALUE;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int32_t v[4] = {0, 0, 0, 0};
  TSFA_CUDA_CHECK(cudaMemcpyAsync(v, workspace, sizeof(v), cudaMemcpyDeviceToHost, s));
  TSFA_CUDA_CHECK(cudaStreamSynchronize(s));
  for (int i = 0; i < 4; ++i) detail[i] = v[i];
  // after a device error every counter of the sync block may be stale: clear it all
  if (v[0] != TSFA_OK) TSFA_CUDA_CHECK(cudaMemsetAsync(workspace, 0, TSFA_SYNC_BYTES, s));
  return TSFA_OK;
}

extern "C" int tsfa_read_device_status(void* workspace, void* stream, int32_t* device_status) {
  if (!device_status) return TSFA_ERR_VALUE;
  int32_t d[4];
  const int st = tsfa_read_device_status_detail(workspace, stream, d);
  if (st == TSFA_OK) *device_status = d[0];
  return st;
}

extern "C" int tsfa_debug_last_plan(int32_t plan[4]) {
  if (!plan) return TSFA_ERR_VALUE;
  for (int i = 0; i < 4; ++i) plan[i] = g_last_plan[i];
  return TSFA_OK;
}

extern "C" int tsfa_debug_force_merge(int32_t mode) {
  if (mode != 0 && mode != 1 && mode != 3) return TSFA_ERR_VALUE;
  g_force_merge = mode;
  return TSFA_OK;
}

extern "C" int tsfa_debug_inject(int32_t fault, uint64_t wait_limit_ns) {
  if (fault != TSFA_FAULT_NONE && fault != TSFA_FAULT_WITHHOLD_TREE_LIST && fault != TSFA_FAULT_REFUSE_COOPERATIVE)
    return TSFA_ERR_VALUE;
  g_fault = fault;
  g_wait_limit_ns = wait_limit_ns;
  return TSFA_OK;
}

// ---------------------------------------------------------------- no-allocation variant
// tsfa_run_tree_sparse over a library-owned workspace: a file-scope device
// array, so the call needs no allocation by anyone.  The array is zeroed when
// the module loads; set-up additionally clears its sync block on the first
// call's stream.  Concurrent calls share the array and race.
namespace {
static __device__ __align__(256) unsigned char g_noalloc_ws[TSFA_NOALLOC_WORKSPACE_BYTES];

constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoallocMaxDevices] = {};

// Address of the current device's copy of g_noalloc_ws.  It is looked up on
// every call (cudaGetSymbolAddress is a host-side table lookup once the
// module is loaded), so a context created after cudaDeviceReset, or another
// context current on the thread, gets its own copy's address, never a stale
// one.  The sync block is cleared on `stream` the first time an address is
// seen on a device (a freshly loaded module also starts zeroed).
int noalloc_workspace(cudaStream_t stream, void** ptr) {
  int dev = 0;
  TSFA_CUDA_CHECK(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kNoallocMaxDevices) return TSFA_ERR_UNSUPPORTED;
  void* p = nullptr;
  TSFA_CUDA_CHECK(cudaGetSymbolAddress(&p, g_noalloc_ws));
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] != p) {
    TSFA_CUDA_CHECK(cudaMemsetAsync(p, 0, TSFA_SYNC_BYTES, stream));
    g_noalloc_ptr[dev] = p;
  }
  *ptr = p;
  return TSFA_OK;
}
}  // namespace

extern "C" int tsfa_run_tree_sparse_noalloc(const TsfaFwdArgs* args, const void* tree_mask, int32_t mask_dtype,
                                            int64_t mask_row_stride, void* stream) {
  size_t need = 0;
  int st = tsfa_run_workspace_bytes(args, &need);
  if (st != TSFA_OK) return st;
  if (need > (size_t)TSFA_NOALLOC_WORKSPACE_BYTES) return TSFA_ERR_WORKSPACE;
  void* ws = nullptr;
  st = noalloc_workspace(static_cast<cudaStream_t>(stream), &ws);
  if (st != TSFA_OK) return st;
  return tsfa_run_tree_sparse(args, tree_mask, mask_dtype, mask_row_stride, ws, TSFA_NOALLOC_WORKSPACE_BYTES, stream);
}

extern "C" int tsfa_noalloc_read_device_status(void* stream, int32_t detail[4]) {
  if (!detail) return TSFA_ERR_VALUE;
  void* ws = nullptr;
  const int st = noalloc_workspace(static_cast<cudaStream_t>(stream), &ws);
  if (st != TSFA_OK) return st;
  return tsfa_read_device_status_detail(ws, stream, detail);
}
