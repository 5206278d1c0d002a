// Forward kernel for sm_100a: TMA + tcgen05/TMEM, warp-specialised, split-KV
// with a log-sum-exp merge of the splits' partial rows: through distributed
// shared memory within a thread-block cluster (bulk copies), or through L2
// between the CTAs of a cooperative grid.  Instantiated per head_dim, dtype,
// contiguous or paged K/V, merge mode and row-tile pairing, so a launch
// carries only its own code paths.
//
// Semantics are those of block_sparse_tree_fwd_kernel
// (tree_sparse_flashattn.py:163-339): prefix keys [0, P) visible and masked
// to n < P (tsfa.py:266-270); tree keys P + c visible iff the CSR entry of the
// row's q-block says so (FULL, or the MIXED bitset bit, tsfa.py:284-318) and
// n < kv_len; online softmax with p = 0 where s = -inf and the -inf/-inf alpha
// guard (tsfa.py:272-279, 320-327); O = acc / l without an l == 0 guard
// (tsfa.py:329).
//
// One CTA = one row tile (128 rows r = g + G * t_local: the G query heads of a
// kv-head folded into MMA M, so K/V are read once for all of them) x one
// cost-balanced slice of the group's 128-key tiles (prefix first, then the
// tree tiles its CSR rows touch).  The slices of a group form one cluster
// (cluster merge) or meet through L2 (global merge).  Without a split, a CTA
// may instead take a pair of row tiles (kPair below).
//
//   warp 0      TMA producer: Q once, K tiles into a 3-slot ring (a slot
//               recycles once S has read it), V tiles into a 3-slot ring
//               (2 slots with a split merge or a pair; recycles after P.V).
//   warp 1      TMEM allocator + tcgen05.mma issuer (one lane):
//                 S[a&1]   = Q K_a^T     (SS, K-major SW128, M=128 N=128)
//                 O[a&1]  += P_a V_a      (TS: P from TMEM, V MN-major, N=D)
//               in the order S(0) S(1) PV(0) S(2) PV(1) S(3) ...; S(a+2)
//               reuses the S buffer of P(a) and waits for P(a).V.
//   warps 2-9   softmax in two sets: warps 2-5 take the key tiles 0, 2, 4,
//               ..., warps 6-9 the tiles 1, 3, 5, ...; one thread per row
//               (TMEM lane = row) over the tile's 128 keys.  Each set has its
//               own S buffer, running max, row sum and O accumulator in TMEM,
//               so the two warps sharing a scheduler are on different tiles.
//               A thread exponentiates its keys two at a time (packed fp32
//               scaling and sums, 2^x on MUFU; full prefix tiles run a compact
//               instantiation of the tile body without masking or residual),
//               packs P to bf16 (round to nearest, as the reference's
//               p.to(v.dtype)) over the first 64 columns of its S buffer.  O
//               is rescaled lazily (row max grew by > 2^8), warp-collectively.
//               Tree tiles add the residual P - P_hi (second P.V, from shared
//               memory), keeping ~16 mantissa bits on rows that see a handful
//               of keys.  The epilogue combines the two sets' states per row
//               (their (m, l) meet in TMEM).
//   epilogue    one split: normalise + store.  Several: every CTA stages its
//               partial rows (O in fp16 scaled per half row, m, l) in shared
//               memory.  Cluster: cluster barrier; lane c of warp 0
//               bulk-copies the rows of CTA c's slice into CTA c's inbox
//               (completion counted on its merge mbarrier); each CTA merges
//               its slice; cluster barrier.  Global: thread 0 bulk-stores the
//               rows to the workspace, counts in, waits (bounded) for the
//               group, bulk-loads its slice of every split's rows and counts
//               out; each CTA merges its slice.
//
// Every mbarrier wait is bounded in wall time; one that runs out raises the
// CTA's abort flag and writes the status block (site, tile, CTA), and all
// roles wind down (the producer lets its own copies land) before TMEM is
// freed.  Decisions that guard warp-collective tcgen05.ld/st are warp-uniform.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <type_traits>

#include <map>
#include <mutex>
#include <set>
#include <utility>

#include "tsfa_fwd.cuh"
#include "tsfa_sm100.cuh"

namespace tsfa {
namespace tc {

using namespace sm100;

static_assert(kWaitLimitNs == kDefaultWaitLimitNs, "one default limit for host and device");

constexpr int kRows = 128;
constexpr int kKeys = 128;
constexpr int kKStages = 3;
constexpr int kVStagesMax = 3;
// V ring slots of an instantiation: three where one split streams many tiles
// from L2 (a V tile then takes ~2 us to land, longer than two tiles of the
// loop); two with the split merges (measured no better with three) and with
// row-tile pairs (their second Q tile takes the third slot's room).
__host__ __device__ constexpr int v_stages(bool no_merge, bool pair) { return no_merge && !pair ? 3 : 2; }
constexpr int kThreads = 352;         // producer, MMA, 8 softmax warps, tree-list warp
constexpr int kListWarp = 10;
constexpr int kSoftmaxThreads = 256;  // two sets of 128: one thread per row in each
constexpr int kSetThreads = 128;
constexpr float kRescaleLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: S buffers of the two softmax sets at 0 and 128 (fp32 scores;
// P(a), bf16 pairs, overwrites the first 64 columns of its buffer and is the
// A operand of P.V), then the sets' O accumulators at 256 and 256 + D.
constexpr uint32_t kColO = 256;
constexpr unsigned kFull = 0xffffffffu;

// Tensor maps of one launch.  The paged instantiation adds the tree keys
// gathered into the workspace (dense); the contiguous one carries none of
// the paged state, so its kernel and parameter block are those of a build
// without paging.
template <bool kPaged>
struct TmaMaps {
  CUtensorMap q, k, v;
};
template <>
struct TmaMaps<true> {
  CUtensorMap q, k, v;
  CUtensorMap kt, vt;
};

// VS: V ring slots; QT: Q tiles (2: a row-tile pair).
template <int D, int VS = 2, int QT = 1>
struct Layout {
  static constexpr int kBox = kRows * 128;  // 128 rows x 128 B: one 64-column SW128 box (16 KB)
  static constexpr int kDH = D / 64;        // 64-column halves of head_dim
  static constexpr int kTile = kDH * kBox;  // one K or V tile (128 keys)
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + QT * kTile;
  static constexpr int kV = kK + kKStages * kTile;
  // P lives in TMEM.  Its rounding residual on tree tiles (128 rows x 128
  // keys, K-major SW128) is an SS operand: with D = 128 a K slot is exactly
  // that size, so the residual goes into the tile's own K slot (S has consumed
  // it; the slot's release is deferred to after P.V); with D = 64 it has its
  // own buffer.
  static constexpr bool kPLInK = (D == 128);
  static constexpr int kPL = kV + VS * kTile;
  static constexpr int kBytes = kPLInK ? kPL : kPL + 2 * 2 * kBox;  // D = 64: one residual buffer per set
  static constexpr int kAlloc = kBytes + 1024;  // room to align the base to 1024 B
  // Split merge, after the CTA's main loop, over the K/V rings.  A partial
  // row is the unnormalised O in fp16, each half row (the D/2 columns one
  // thread holds) scaled by 2^-e so that its largest magnitude lands in
  // [2^14, 2^15), then (m, l0, l1) in fp32 and the two halves' e as int16 --
  // half the bytes of an fp32 row (the exchange is bound by L2 bandwidth) at
  // 2^-12 relative rounding against the half row's largest value:
  //   staging [128 rows][row]: this CTA's rows
  //   inbox   [ns][cdiv(128, ns)][row]: every split's rows of the slice this
  //           CTA merges
  static constexpr int kRowBytes = 2 * D + 16;  // multiple of 16 for bulk copies
  static constexpr int kRowMl = 2 * D;          // byte offset of (m, l0, l1, e0 | e1)
  static constexpr int kStage = kK;
  static constexpr int kInbox = kStage + ((kRows * kRowBytes + 1023) / 1024) * 1024;
  static_assert(kInbox + (kRows + kMaxSplits) * kRowBytes <= kBytes, "merge buffers must fit");
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kKStages], k_empty[kKStages];
  uint64_t v_full[kVStagesMax], v_empty[kVStagesMax];
  // per softmax set s (tiles a = s, s + 2, ...): S(a) complete / P(a) written /
  // P(a).V complete
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t list_ready, merge;
  uint64_t mma_drain;  // after a failed wait: every MMA the issuer started has completed
};

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  // round-to-nearest pack (residuals, outputs)
  static __device__ __forceinline__ uint32_t two(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  // the value a round-to-nearest pack keeps of x
  static __device__ __forceinline__ float kept(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
};
template <>
struct Pack<__half> {
  static constexpr bool kBf16 = false;
  static __device__ __forceinline__ uint32_t two(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float kept(float x) { return __half2float(__float2half_rn(x)); }
};

// Wait sites reported in the workspace status block when a wait gives up.
enum WaitSite : int {
  kSiteListProducer = 1, kSiteKvEmpty, kSiteQFull, kSiteListMma, kSiteKFull, kSiteSEmpty, kSitePFull, kSiteVFull,
  kSiteSFull, kSitePvDone, kSitePvDoneEpi, kSiteListSoftmax, kSiteMerge, kSiteRowMax
};

// First key tile of split s: the tiles (prefix first, then tree) are cut into
// ns contiguous slices of about equal cost, a tree tile costing kTreeCost
// prefix tiles (bitset decode, the second, residual P.V, and the wait for the
// metadata kernel that the prefix tiles do not have).
constexpr int kTreeCost = 4;

__device__ __forceinline__ int split_begin(int s, int ns, int n_pre_tiles, int n_tree_tiles) {
  const int total = n_pre_tiles + kTreeCost * n_tree_tiles;
  const int target = (int)((int64_t)s * total / ns);
  return target <= n_pre_tiles ? target : n_pre_tiles + (target - n_pre_tiles + kTreeCost - 1) / kTreeCost;
}
__device__ __forceinline__ int rows_begin(int c, int ns) { return c * kRows / ns; }

// status[0] = TSFA_ERR_DEVICE_TIMEOUT; status[1..3] = first site, tile, CTA.
__device__ __forceinline__ void raise_abort(volatile int* flag, int* status, int site, int tile) {
  *flag = 1;
  if (atomicCAS(status, 0, TSFA_ERR_DEVICE_TIMEOUT) == 0) {
    status[1] = site;
    status[2] = tile;
    status[3] = (int)(blockIdx.y * gridDim.x + blockIdx.x);
  }
}

// One 128-key K or V tile (keys n0 .. n0 + 127 of (b, kvh)) into `dst`:
// kDH boxes of 128 rows x 64 columns, completing on `bar` (which expects
// kTile bytes).  Dense: one 4-D box per 64 columns.  Paged: boxes of
// min(page_size, 128) tokens, each from its page; keys at or past kv_len,
// and page slots past the batch element's page list, read a page coordinate
// past the pool, which the copy fills with zeros (bytes still counted).
template <int D, bool kPaged>
__device__ __forceinline__ void load_kv_tile(const FwdParams& p, uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                             int n0, int kvh, int b, int pg_lo, int pg_n) {
  using L = Layout<D>;
  if constexpr (!kPaged) {
    for (int h = 0; h < L::kDH; ++h) tma_load_4d(dst + h * L::kBox, map, bar, h * 64, n0, kvh, b);
    return;
  }
  const int ps = 1 << p.page_shift;
  const int rows = ps < kKeys ? ps : kKeys;  // tokens per box
  for (int j = 0; j < kKeys / rows; ++j) {
    const int n = n0 + j * rows;
    const int pi = n >> p.page_shift;  // page of the batch element's list
    const int page = (n < p.kv_len && pi < pg_n) ? __ldg(p.page_indices + pg_lo + pi) : p.num_pages;
    const int slot = n & (ps - 1);
    for (int h = 0; h < L::kDH; ++h) tma_load_4d(dst + h * L::kBox + j * rows * 128, map, bar, h * 64, kvh, slot, page);
  }
}

// Split merge of a launch, fixed per instantiation so that each kernel holds
// only its own epilogue (code a launch never runs still costs it
// instruction fetches).
enum MergeMode : int { kMergeNone = 0, kMergeCluster = 1, kMergeGlobal = 2 };

// kPair: one CTA takes two row tiles (a row-tile pair) over every key tile of
// its group, without a split: both row tiles share each K and V tile it
// loads, halving the K/V bytes streamed per flop.  Softmax set s then holds
// row tile s (its own Q tile, S buffer, row state and O) and takes every key
// tile; "tile a" of the loops is virtual: key tile a >> 1 for row tile a & 1.
// With D = 128 the tree tiles' rounding residual has no room in shared memory
// (the second Q tile takes it): P is rounded once there, as the reference
// does, and the host picks pairs only where every row sees >= 1024 prefix keys.
template <int D, typename T, bool kPaged, int kMerge, bool kPair = false>
__global__ void __launch_bounds__(kThreads, 1) fwd_tc_kernel(const __grid_constant__ FwdParams p,
                                                             const __grid_constant__ TmaMaps<kPaged> maps) {
  static_assert(!kPair || (kMerge == kMergeNone && !kPaged), "row-tile pairs: contiguous K/V, no split");
  constexpr int VS = v_stages(kMerge == kMergeNone, kPair);
  constexpr int QT = kPair ? 2 : 1;  // Q tiles (row tiles) of a CTA
  using L = Layout<D, VS, QT>;
  // key tile and Q tile of the loops' tile a
  auto kt = [](int a) { return kPair ? a >> 1 : a; };
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base for the SW128 tiles; offsetting the shared array
  // itself (no integer round trip) keeps every access a shared-memory one
  uint8_t* smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sPL = smem + L::kPL;  // D = 64 only
  __shared__ Bars bars;
  __shared__ uint32_t s_tmem;
  __shared__ int s_tree_list[kMaxTreeTileList];
  __shared__ int s_tree_count;
  __shared__ int s_abort_storage;
  volatile int* s_abort = &s_abort_storage;
  float o[D / 2];  // softmax threads: their half row of O (registers)

  // A kernel launched after this one with programmatic stream serialization
  // (the next call's metadata kernel) may become resident now; it waits for
  // this grid to complete before it touches anything.
  griddep_launch_dependents();
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint64_t wl = p.wait_limit_ns;  // limit of every bounded wait of this launch
  const int ns = p.n_splits;
  const int split = blockIdx.x % ns;  // == rank in the cluster
  const int rtile = blockIdx.x / ns;
  const int unit = blockIdx.y;
  const int b = unit / p.Hkv, kvh = unit - b * p.Hkv;
  const MetaView mv = meta_of_batch(p.mv, b);  // this batch element's tree
  // paged K/V: this batch element's page list (used by thread 0, the producer)
  int pg_lo = 0, pg_n = 0;
  if (kPaged && tid == 0) {
    pg_lo = __ldg(p.page_indptr + b);
    pg_n = __ldg(p.page_indptr + b + 1) - pg_lo;
  }
  const int G = p.G, TPT = p.t_per_tile, R = G * TPT;
  const int t0 = rtile * TPT * QT;                 // first tree row of the CTA's (first) row tile
  const int t_hi = min(t0 + QT * TPT, p.T) - 1;  // last tree row of its row tiles
  const int j0 = split_begin(split, ns, p.n_prefix_tiles, p.n_tree_tiles);  // cost-balanced slice
  const int j1 = split_begin(split + 1, ns, p.n_prefix_tiles, p.n_tree_tiles);
  const int n_pre = max(0, min(j1, p.n_prefix_tiles) - j0);
  const int tr0 = max(j0, p.n_prefix_tiles) - p.n_prefix_tiles;
  const int tr1 = max(j1, p.n_prefix_tiles) - p.n_prefix_tiles;

  if (tid == 0) {
    mbar_init(&bars.q_full, 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&bars.k_full[s], 1);
      mbar_init(&bars.k_empty[s], 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(&bars.v_full[s], 1);
      mbar_init(&bars.v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars.s_full[s], 1);
      mbar_init(&bars.p_full[s], kSetThreads);
      mbar_init(&bars.pv_done[s], 1);
    }
    mbar_init(&bars.list_ready, 1);
    mbar_init(&bars.merge, 1);
    mbar_init(&bars.mma_drain, 1);
    s_abort_storage = 0;
    s_tree_count = 0;
    fence_mbar_init();
    if constexpr (kMerge == kMergeCluster) {
      // the merge barrier completes when the other splits' rows of this CTA's
      // slice have landed in its inbox
      const int my_rows = rows_begin(split + 1, ns) - rows_begin(split, ns);
      mbar_arrive_expect_tx(&bars.merge, (uint32_t)((ns - 1) * my_rows * L::kRowBytes));
    }
    // The first copies do not depend on the tree list: start them before the
    // CTA-wide setup barrier (Q, K and V of the first prefix tiles: every ring
    // slot).
    mbar_arrive_expect_tx(&bars.q_full, (uint32_t)(QT * L::kDH * 128 * R));
    for (int qt = 0; qt < QT; ++qt)
      for (int h = 0; h < L::kDH; ++h)
        tma_load_4d(sQ + qt * L::kTile + h * L::kBox, &maps.q, &bars.q_full, h * 64, kvh * G, t0 + qt * TPT, b);
    for (int a = 0; a < min(kKStages, n_pre); ++a) {
      mbar_arrive_expect_tx(&bars.k_full[a], (uint32_t)L::kTile);
      load_kv_tile<D, kPaged>(p, sK + a * L::kTile, &maps.k, &bars.k_full[a], (j0 + a) * kKeys, kvh, b, pg_lo, pg_n);
    }
    for (int a = 0; a < min(VS, n_pre); ++a) {
      mbar_arrive_expect_tx(&bars.v_full[a], (uint32_t)L::kTile);
      load_kv_tile<D, kPaged>(p, sV + a * L::kTile, &maps.v, &bars.v_full[a], (j0 + a) * kKeys, kvh, b, pg_lo, pg_n);
    }
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------ producer
    // (one thread: it polls the barriers and issues every copy)
    // Key tiles: K(0) K(1) K(2) and the first VS V tiles at setup, then K(3)
    // V(VS) K(4) ... -- K runs up to three key tiles ahead of V, in the order
    // the MMA warp consumes them.  K(j) reuses the slot of K(j - 3) once its
    // S MMAs have read it; V(j) the slot of V(j - VS) once its P.V MMAs have.
    bool ok = true;
    int site = 0, at = 0;
    int kq = min(kKStages, n_pre), vq = min(VS, n_pre);  // next K / V tile to issue
    bool k_done = false;
    int n_total = n_pre;
    bool have_list = false;
    for (;;) {
      const bool do_k = !k_done && kq < vq + kKStages;
      const int a = do_k ? kq : vq;
      if (a >= n_pre && !have_list) {
        ok = mbar_wait(&bars.list_ready, 0, s_abort, wl);
        if (!ok) {
          site = kSiteListProducer;
          at = a;
          break;
        }
        n_total = n_pre + s_tree_count;
        have_list = true;
      }
      if (a >= n_total) {
        if (do_k && vq < n_total) {  // every K is out; V still has tiles
          k_done = true;
          continue;
        }
        break;
      }
      const int nst = do_k ? kKStages : VS;
      const int stage = a % nst;
      if (a >= nst) {
        uint64_t* empty = do_k ? &bars.k_empty[stage] : &bars.v_empty[stage];
        ok = mbar_wait(empty, ((a - nst) / nst) & 1, s_abort, wl);
        if (!ok) {
          site = kSiteKvEmpty;
          at = a;
          break;
        }
      }
      const int n0 = a < n_pre ? (j0 + a) * kKeys : p.P + s_tree_list[a - n_pre] * kKeys;
      uint64_t* full = do_k ? &bars.k_full[stage] : &bars.v_full[stage];
      uint8_t* dst = (do_k ? sK : sV) + stage * L::kTile;
      const CUtensorMap* map = do_k ? &maps.k : &maps.v;
      mbar_arrive_expect_tx(full, (uint32_t)L::kTile);
      if constexpr (kPaged) {
        if (a >= n_pre) {
        // a tree tile of a paged cache starts at key P + 128 jt, which need
        // not be a page boundary: it comes from the copy of the tree keys
        // the metadata kernel gathered (this load follows list_ready, which
        // follows the wait for that kernel); rows >= T fill with zeros
          const CUtensorMap* tmap = do_k ? &maps.kt : &maps.vt;
          for (int h = 0; h < L::kDH; ++h)
            tma_load_4d(dst + h * L::kBox, tmap, full, h * 64, n0 - p.P, kvh, b);
        } else {
          load_kv_tile<D, kPaged>(p, dst, map, full, n0, kvh, b, pg_lo, pg_n);
        }
      } else {
        load_kv_tile<D, kPaged>(p, dst, map, full, n0, kvh, b, pg_lo, pg_n);
      }
      if (do_k) ++kq; else ++vq;
    }
    if (!ok) {
      raise_abort(s_abort, p.status, site, at);
      // let this CTA's own copies land before the shared memory goes away
      mbar_wait(&bars.q_full, 0, nullptr, wl);
      for (int a = max(0, kq - kKStages); a < kq; ++a) mbar_wait(&bars.k_full[a % kKStages], (a / kKStages) & 1, nullptr, wl);
      for (int a = max(0, vq - VS); a < vq; ++a) mbar_wait(&bars.v_full[a % VS], (a / VS) & 1, nullptr, wl);
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer
    // (one thread: it polls the barriers and issues every MMA and commit)
    constexpr uint32_t idS = idesc_f16(Pack<T>::kBf16, 128, kKeys, false);
    constexpr uint32_t idPV = idesc_f16(Pack<T>::kBf16, 128, D, true);
    const uint32_t aQ = smem_addr(sQ), aK = smem_addr(sK), aV = smem_addr(sV), aPL = smem_addr(sPL);
    int site = 0, at = 0;
    bool ok = mbar_wait(&bars.q_full, 0, s_abort, wl);
    if (!ok) site = kSiteQFull;
    int n_total = QT * n_pre;  // loop tiles (pairs: two per key tile)
    bool have_list = false;
    auto fail = [&](int s_, int a) -> bool {
      site = s_;
      at = a;
      return false;
    };
    auto ensure = [&](int a) -> bool {
      if (kt(a) >= n_pre && !have_list) {
        if (!mbar_wait(&bars.list_ready, 0, s_abort, wl)) return fail(kSiteListMma, a);
        n_total = QT * (n_pre + s_tree_count);
        have_list = true;
      }
      return true;
    };
    // Tile a belongs to softmax set a & 1: S(a) into that set's S buffer,
    // P(a).V into that set's O.  S(a) overwrites the columns P(a - 2) held:
    // it is issued only once P(a - 2).V has completed.
    auto issue_s = [&](int a) -> bool {
      const int ks = kt(a) % kKStages, sb = a & 1;
      if (!mbar_wait(&bars.k_full[ks], (kt(a) / kKStages) & 1, s_abort, wl)) return fail(kSiteKFull, a);
      if (a >= 2 && !mbar_wait(&bars.pv_done[sb], ((a - 2) >> 1) & 1, s_abort, wl)) return fail(kSiteSEmpty, a);
      tc_fence_after();
      {
        const uint32_t kbase = aK + ks * L::kTile;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kBox + (kk & 3) * 32;
          umma_f16_ss(tmem + (uint32_t)sb * kKeys, sw128_desc(aQ + (kPair ? sb * L::kTile : 0) + off, 16, 1024),
                      sw128_desc(kbase + off, 16, 1024), idS, kk > 0);
        }
        umma_commit(&bars.s_full[sb]);
        // K slot free once S(a) is done (pairs: once both row tiles' S are)
        if (kPair ? (a & 1) != 0 : !(L::kPLInK && a >= n_pre)) umma_commit(&bars.k_empty[ks]);
      }
      return true;
    };
    auto issue_pv = [&](int a) -> bool {
      const int ks = kt(a) % kKStages, vs = kt(a) % VS, sb = a & 1;
      const uint32_t vbase = aV + vs * L::kTile;
      const uint32_t dO = tmem + kColO + (uint32_t)sb * D;
      if (!mbar_wait(&bars.p_full[sb], (a >> 1) & 1, s_abort, wl)) return fail(kSitePFull, a);
      if (!mbar_wait(&bars.v_full[vs], (kt(a) / VS) & 1, s_abort, wl)) return fail(kSiteVFull, a);
      tc_fence_after();
      {
        // O_s += P V with P from TMEM (TS); tree tiles add P_lo V from shared memory (SS)
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)
          umma_f16_ts(dO, tmem + (uint32_t)sb * kKeys + kk * 8, sw128_desc(vbase + kk * 16 * 128, L::kBox, 1024), idPV,
                      (a >= 2 || kk > 0) ? 1u : 0u);
        if ((!kPair || !L::kPLInK) && kt(a) >= n_pre) {  // pairs with D = 128: no residual (no room)
          const uint32_t aLo = L::kPLInK ? aK + ks * L::kTile : aPL + (uint32_t)(sb * 2 * L::kBox);
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            const uint32_t poff = (kk >> 2) * L::kBox + (kk & 3) * 32;
            umma_f16_ss(dO, sw128_desc(aLo + poff, 16, 1024), sw128_desc(vbase + kk * 16 * 128, L::kBox, 1024), idPV,
                        1u);
          }
        }
        if (!kPair && L::kPLInK && a >= n_pre) umma_commit(&bars.k_empty[ks]);  // held the residual of P
        if (!kPair || (a & 1) != 0) umma_commit(&bars.v_empty[vs]);  // pairs: once both row tiles' P.V are done
        umma_commit(&bars.pv_done[sb]);
      }
      return true;
    };
    if (ok) ok = ensure(0);
    if (ok && n_total > 0) ok = issue_s(0);
    if (ok) ok = ensure(1);
    if (ok && n_total > 1) ok = issue_s(1);
    for (int a = 0; ok && a < n_total; ++a) {
      ok = issue_pv(a);
      if (ok) ok = ensure(a + 2);
      if (ok && a + 2 < n_total) ok = issue_s(a + 2);
    }
    if (!ok) {
      raise_abort(s_abort, p.status, site, at);
      // nobody waits for the MMAs already issued: let them complete before
      // TMEM is freed
      umma_commit(&bars.mma_drain);
      mbar_wait(&bars.mma_drain, 0, nullptr, wl);
    }
  } else if (warp == kListWarp) {
    // ------------------------------------------------------------ tree list
    // The tree tiles this CTA's slice needs: the union of the CSR entries of
    // the row tile's q-blocks, clipped to [tr0, tr1).  The metadata may come
    // from the kernel just before this one on the stream (programmatic
    // dependent launch): only this warp and the softmax threads, before their
    // first tree tile, wait for it -- the prefix sweep does not.
    unsigned long long bits = 0ull;  // bit jt - tr0 (tr1 - tr0 <= kMaxTreeTileList = 64)
    if (tr1 > tr0) {
      griddep_wait();
      const int BM = mv.block_m, BN = mv.block_n;
      int e0 = __ldg(mv.row_ptr + t0 / BM);
      int e1 = __ldg(mv.row_ptr + t_hi / BM + 1);
#ifdef TSFA_DEBUG
      // the rows' entries must lie in [0, nnz): otherwise skip them all
      if (!row_ok(mv, t0 / BM, e0, e1, p.status)) e1 = e0;
#endif
      for (int e = e0 + lane; e < e1; e += 32) {
        const int tb = __ldg(mv.col_idx + e);
#ifdef TSFA_DEBUG
        if (tb < 0 || tb >= mv.n_tree_blocks) {
          bounds_report(p.status, kCheckColIdx, e);
          continue;
        }
#endif
        const int lo = (tb * BN) / kKeys, hi = min((tb * BN + BN - 1) / kKeys, p.n_tree_tiles - 1);
        for (int jt = max(lo, tr0); jt <= min(hi, tr1 - 1); ++jt) bits |= 1ull << (jt - tr0);
      }
    }
    const unsigned lo32 = __reduce_or_sync(kFull, (unsigned)bits);
    const unsigned hi32 = __reduce_or_sync(kFull, (unsigned)(bits >> 32));
    if (lane == 0) {
      const unsigned long long all = ((unsigned long long)hi32 << 32) | lo32;
      int c = 0;
      for (int jt = tr0; jt < tr1; ++jt)
        if ((all >> (jt - tr0)) & 1ull) s_tree_list[c++] = jt;
      s_tree_count = c;
      // the test fault withholds the list: every wait on it must run out
      if (p.fault != TSFA_FAULT_WITHHOLD_TREE_LIST) mbar_arrive(&bars.list_ready);
    }
  } else if (warp >= 2) {
    // ------------------------------------------------------------ softmax
    // Two sets of four warps.  Set s takes the key tiles a = s, s + 2, ...
    // with one thread per row (TMEM lane = row) over all 128 keys of a tile,
    // and keeps its own running max, row sum and O accumulator (TMEM O_s).
    // The two warps that share a scheduler belong to different sets, so they
    // work on different tiles and hide each other's latencies; the two
    // partial states of a row are combined once, in the epilogue.  (Pairs:
    // set s holds row tile s and takes every key tile; nothing to combine.)
    const int st = tid - 64;               // 0..255
    const int set = st >> 7;               // this thread's set; in the epilogue its O-column half
    const int half = set;
    const int r = 32 * (warp & 3) + lane;  // TMEM lane == row of the tile
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const uint32_t colS = (uint32_t)set * kKeys;      // this set's S buffer; P(a) overwrites its first 64 columns
    const uint32_t colO = kColO + (uint32_t)set * D;  // this set's O accumulator
    const int tl = r / G;
    const int t = t0 + (kPair ? set * TPT : 0) + tl;
    const bool row_valid = (r < R) && (t < p.T);
    const float sl2 = p.scale_log2;
    constexpr int DH = D / 2;  // O columns this thread finishes in the epilogue

    int n_total = QT * n_pre;  // + the tree tiles, once the tree-list warp has published them
    bool have_list = false;

    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int site = 0, at = 0;
    // One tile of the softmax; false if a wait gave up (site / at set).
    // kGeneral: masked keys (the last, partial prefix tile; tree tiles) and
    // the tree tiles' rounding residual.  Full prefix tiles -- most of the
    // work -- run the compact instantiation, which keeps their loop small in
    // the instruction caches.
    auto softmax_tile = [&](int a, auto general) -> bool {
      constexpr bool kGeneral = decltype(general)::value;
      const bool is_tree = kGeneral && kt(a) >= n_pre;
      const int n0 = is_tree ? p.P + s_tree_list[kt(a) - n_pre] * kKeys : (j0 + kt(a)) * kKeys;
      // keys of the tile the row sees: all of a full prefix tile; else a
      // mask.  The compact body takes every key: its rows past the row tile
      // (row_valid false) get numbers in their own TMEM lanes only, and those
      // rows are never stored.  The general body only ever runs on masked
      // tiles (its first tile, n_full below, is the partial prefix tile or a
      // tree tile), so it carries no unmasked path.
      const bool full = !kGeneral;
      unsigned long long vis_lo = 0ull, vis_hi = 0ull;
      if (!full && row_valid) {
        if (!is_tree) {
          const int nv = p.P - n0;  // 0 < nv < 128: keys n < P (tsfa.py:270)
          vis_lo = nv >= 64 ? ~0ull : ((1ull << nv) - 1ull);
          vis_hi = nv > 64 ? ((1ull << (nv - 64)) - 1ull) : 0ull;
        } else {
          const int lim = min(kKeys, p.kv_len - n0);
          vis_lo = tree_row_bits(mv, t, n0 - p.P, min(64, lim), p.T, p.status);
          vis_hi = lim > 64 ? tree_row_bits(mv, t, n0 - p.P + 64, lim - 64, p.T, p.status) : 0ull;
        }
      }
      // tcgen05.ld / st are warp-collective (.sync.aligned): every decision
      // that guards one is warp-uniform.
      if (!__all_sync(kFull, mbar_wait(&bars.s_full[set], (a >> 1) & 1, s_abort, wl))) {
        ok = false;
        site = kSiteSFull;
        at = a;
        return false;
      }
      tc_fence_after();
      // Two passes over the S buffer, 64 scores at a time (128 live scores
      // would not fit the register budget of 352 threads): the row max, then
      // the exponentials.  P for keys [64 h, 64 h + 64) goes to columns
      // [32 h, 32 h + 32), which held scores the pass has already read.  The
      // loops over h are not unrolled: the kernel is bound by instruction
      // fetch as much as by anything at small sizes (each body runs cold at
      // least once per CTA), and one copy of each half's code fetches half the
      // bytes.
      auto load64 = [&](int h, float* x) {
        uint32_t* xr = reinterpret_cast<uint32_t*>(x);
        tmem_ld32(tmem + lane_base + colS + 64 * h, xr);
        tmem_ld32(tmem + lane_base + colS + 64 * h + 32, xr + 32);
        tmem_ld_wait();
        if (!full) {
          const unsigned long long vm = h ? vis_hi : vis_lo;
#pragma unroll
          for (int i = 0; i < 64; ++i) x[i] = ((vm >> i) & 1ull) ? x[i] : -INFINITY;
        }
      };
      float mx = -INFINITY;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float x[64];
        load64(h, x);
        // eight independent chains of three-input max
        float mx8[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = max3f(x[j], x[8 + j], x[16 + j]);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = max3f(mx8[j], x[24 + j], x[32 + j]);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = max3f(mx8[j], x[40 + j], x[48 + j]);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx8[j] = fmaxf(mx8[j], x[56 + j]);
        mx = max3f(mx, max3f(mx8[0], mx8[1], mx8[2]), max3f(mx8[3], mx8[4], max3f(mx8[5], mx8[6], mx8[7])));
      }
      const float m_new = fmaxf(m_run, mx * sl2);  // scale > 0: max commutes with it
      // Lazy rescale: the reference max m_run only moves when the row max
      // grows by more than 2^8 (p stays <= 256 otherwise).  A row whose O is
      // still exactly zero (m_run = -inf) just adopts the new max.
      const bool need = (m_run != -INFINITY) && (m_new > m_run + kRescaleLog2);
      const float alpha = need ? ex2_approx(m_run - m_new) : 1.f;
      if (need || m_run == -INFINITY) m_run = m_new;
      // This set's previous P.V (tile a - 2) has completed: the MMA issuer
      // started S(a) only after it.  So O_s may be rescaled, and P(a) (and,
      // with D = 64, this set's residual buffer) written, without a wait.
      const bool resc = __any_sync(kFull, need);  // the whole warp touches TMEM
      if (resc && a >= 2) {
#pragma unroll 1
        for (int i = 0; i < D / 32; ++i) {
          uint32_t ov[32];
          tmem_ld32(tmem + lane_base + colO + 32 * i, ov);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = __float_as_uint(__uint_as_float(ov[j]) * alpha);
          tmem_st32(tmem + lane_base + colO + 32 * i, ov);
        }
        tmem_st_wait();
      }
      // p = 2^(s * scale_log2 - m) two keys at a time: one packed FMA, then
      // 2^x on MUFU (every key: the FMA pipe carries the packed scaling and
      // sums, and moving some keys' 2^x onto it as a polynomial measured
      // slower at every split of the two pipes).  s = -inf gives 0 (a row
      // that has seen nothing uses 0 as its offset).  P is rounded to nearest, as the reference's
      // p.to(v.dtype); tree tiles also store the residual p - P_hi, as a
      // K-major SW128 tile in shared memory (16-byte chunk c of row r at chunk
      // c ^ (r & 7) of the row's line).
      const float moff = (m_run == -INFINITY) ? 0.f : m_run;
      const float2 sc2 = make_float2(sl2, sl2), off2 = make_float2(-moff, -moff);
      float2 rs[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) rs[j] = make_float2(0.f, 0.f);
      uint8_t* lo_buf = L::kPLInK ? sK + (a % kKStages) * L::kTile : sPL + set * 2 * L::kBox;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        float x[64];
        load64(h, x);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float2 e = fma2(make_float2(x[2 * j], x[2 * j + 1]), sc2, off2);
          e.x = ex2_approx(e.x);
          e.y = ex2_approx(e.y);
          x[2 * j] = e.x;
          x[2 * j + 1] = e.y;
          rs[j & 3] = add2(rs[j & 3], e);
        }
        if ((!kPair || !L::kPLInK) && is_tree) {  // (pairs with D = 128 round P once, as the reference)
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t z[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
              z[j] = Pack<T>::two(x[c * 8 + 2 * j] - Pack<T>::kept(x[c * 8 + 2 * j]),
                                  x[c * 8 + 2 * j + 1] - Pack<T>::kept(x[c * 8 + 2 * j + 1]));
            *reinterpret_cast<uint4*>(lo_buf + h * L::kBox + r * 128 + ((c ^ (r & 7)) << 4)) =
                make_uint4(z[0], z[1], z[2], z[3]);
          }
        }
        uint32_t w[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = Pack<T>::two(x[2 * j], x[2 * j + 1]);
        tmem_st32(tmem + lane_base + colS + 32 * h, w);
      }
      tmem_st_wait();
      const float2 rsum = add2(add2(rs[0], rs[1]), add2(rs[2], rs[3]));
      l_run = l_run * alpha + (rsum.x + rsum.y);
      if constexpr (kGeneral && kPaged) {
        if (n0 + kKeys > p.kv_len) {
          // Paged K/V: the last used page may hold stale values (even NaN)
          // past kv_len, and a 0 in P does not cancel a NaN in V.  Zero the
          // V rows of keys >= kv_len before P(a).V reads them (keys past the
          // page list were already filled with zeros by the copy).
          const int vs = kt(a) % VS;
          if (!__all_sync(kFull, mbar_wait(&bars.v_full[vs], (kt(a) / VS) & 1, s_abort, wl))) {
            ok = false;
            site = kSiteVFull;
            at = a;
            return false;
          }
          const int z0 = max(0, p.kv_len - n0), zrows = kKeys - z0;
          uint8_t* vt = sV + vs * L::kTile;
          for (int i = st & (kSetThreads - 1); i < L::kDH * zrows * 8; i += kSetThreads) {
            const int box = i / (zrows * 8), rem = i - box * zrows * 8;
            *reinterpret_cast<uint4*>(vt + box * L::kBox + (z0 + (rem >> 3)) * 128 + (rem & 7) * 16) =
                make_uint4(0u, 0u, 0u, 0u);
          }
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars.p_full[set]);
      return true;
    };
    // Prefix tiles whose 128 keys all lie below P: the compact body, also in
    // splits that go on to tree tiles.
    const int n_full = QT * max(0, min(n_pre, p.P / kKeys - j0));
    int a = set;
    for (; ok && a < n_full; a += 2) ok = softmax_tile(a, std::false_type{});
    for (; ok; a += 2) {
      if (kt(a) >= n_pre && !have_list) {
        if (!__all_sync(kFull, mbar_wait(&bars.list_ready, 0, s_abort, wl))) {
          ok = false;
          site = kSiteListSoftmax;
          at = a;
          break;
        }
        n_total = QT * (n_pre + s_tree_count);
        have_list = true;
        if (s_tree_count > 0) griddep_wait();  // tree tiles read the metadata
      }
      if (a >= n_total) break;
      ok = softmax_tile(a, std::true_type{});
    }

    if (!ok) raise_abort(s_abort, p.status, site, at);

    if constexpr (kPair) {
      // ------------------------------------------------ epilogue (row-tile pair)
      // Set s holds row tile s whole: after the set's last P.V each thread
      // normalises its row's D columns (O_s / l) and stores them, 32 columns
      // at a time.  A row that saw no key stores 0 / 0 = NaN, as tsfa.py:329.
      const bool ran = ok && n_total > set;  // warp-uniform
      if (ran) {
        const int a_last = n_total - 2 + set;  // n_total is even: both sets ran as many tiles
        if (!__all_sync(kFull, mbar_wait(&bars.pv_done[set], (a_last >> 1) & 1, s_abort, wl))) {
          ok = false;
          raise_abort(s_abort, p.status, kSitePvDoneEpi, n_total);
        }
      }
      tc_fence_after();
      const float inv = 1.f / l_run;
      const int g = r - tl * G;
      T* dst = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)(kvh * G + g) * p.so[1] + (int64_t)t * p.so[2];
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ov[32];
        if (ran && ok) {
          tmem_ld32(tmem + lane_base + colO + 32 * c, ov);
          tmem_ld_wait();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) ov[j] = 0u;
        }
        if (*s_abort == 0 && row_valid) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = Pack<T>::two(__uint_as_float(ov[8 * q + 0]) * inv, __uint_as_float(ov[8 * q + 1]) * inv);
            w.y = Pack<T>::two(__uint_as_float(ov[8 * q + 2]) * inv, __uint_as_float(ov[8 * q + 3]) * inv);
            w.z = Pack<T>::two(__uint_as_float(ov[8 * q + 4]) * inv, __uint_as_float(ov[8 * q + 5]) * inv);
            w.w = Pack<T>::two(__uint_as_float(ov[8 * q + 6]) * inv, __uint_as_float(ov[8 * q + 7]) * inv);
            *reinterpret_cast<uint4*>(dst + 32 * c + 8 * q) = w;
          }
        }
      }
    } else {
    // ---------------------------------------------------------- epilogue
    // Combine the row's two partial states (m_s, l_s, O_s): M = max(m_0, m_1),
    // weights 2^(m_s - M) (0 for a set that saw nothing: m_s = -inf).  Each
    // thread then forms its half of the row's columns from both accumulators.
    // The sets' (m, l) of the row meet in TMEM: columns 64-65 of each set's S
    // buffer, dead since the set's last softmax (its last P sits in columns
    // 0-63, no S of the set follows).
    {
      const uint32_t ml2[2] = {__float_as_uint(m_run), __float_as_uint(l_run)};
      tmem_st2(tmem + lane_base + colS + 64, ml2);
      tmem_st_wait();
    }
    tc_fence_before();
    named_barrier(1, kSoftmaxThreads);  // every softmax thread gets here exactly once
    tc_fence_after();
    float2 ma, mb;
    {
      uint32_t a2[2], b2[2];
      tmem_ld2(tmem + lane_base + 64, a2);
      tmem_ld2(tmem + lane_base + kKeys + 64, b2);
      tmem_ld_wait();
      ma = make_float2(__uint_as_float(a2[0]), __uint_as_float(a2[1]));
      mb = make_float2(__uint_as_float(b2[0]), __uint_as_float(b2[1]));
    }
    const float m_row = fmaxf(ma.x, mb.x);
    const float wa = (ma.x == -INFINITY) ? 0.f : ex2_approx(ma.x - m_row);
    const float wb = (mb.x == -INFINITY) ? 0.f : ex2_approx(mb.x - m_row);
    m_run = m_row;
    // the row sum goes with half 0; the merge adds the two halves' sums
    const float l_half = half == 0 ? ma.y * wa + mb.y * wb : 0.f;
#pragma unroll
    for (int i = 0; i < DH; ++i) o[i] = 0.f;
    const int n_sets = min(n_total, 2);  // sets that ran at least one tile
    if (ok && n_sets > 0) {
      // the last P.V of each set that ran
      for (int s = 0; s < n_sets && ok; ++s) {
        const int a_last = n_total - 1 - ((n_total - 1 - s) & 1);
        ok = __all_sync(kFull, mbar_wait(&bars.pv_done[s], (a_last >> 1) & 1, s_abort, wl));
      }
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int i = 0; i < DH / 32; ++i) {
          uint32_t oa[32], ob[32];
          tmem_ld32(tmem + lane_base + kColO + half * DH + 32 * i, oa);
          if (n_sets > 1) tmem_ld32(tmem + lane_base + kColO + D + half * DH + 32 * i, ob);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j)
            o[32 * i + j] = wa * __uint_as_float(oa[j]) + (n_sets > 1 ? wb * __uint_as_float(ob[j]) : 0.f);
        }
      } else {
        raise_abort(s_abort, p.status, kSitePvDoneEpi, n_total);
      }
    }
    if constexpr (kMerge == kMergeNone) {
      // row sum = the two halves' sums (same m_run on both threads), exchanged
      // through the K ring (free: every MMA has completed)
      float* lx = reinterpret_cast<float*>(smem + L::kStage);
      lx[half * kRows + r] = l_half;
      named_barrier(1, kSoftmaxThreads);  // every softmax thread gets here exactly once
      const float l_row = lx[r] + lx[kRows + r];
      if (*s_abort == 0 && row_valid) {
        const int g = r - tl * G;
        T* dst = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)(kvh * G + g) * p.so[1] +
                 (int64_t)t * p.so[2] + half * DH;
        const float inv = 1.f / l_row;  // l == 0 (row sees no key) gives NaN, as tsfa.py:329
#pragma unroll
        for (int c = 0; c < DH / 8; ++c) {
          uint4 w;
          w.x = Pack<T>::two(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
          w.y = Pack<T>::two(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          w.z = Pack<T>::two(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          w.w = Pack<T>::two(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + 8 * c) = w;
        }
      }
    } else {
      // this CTA's unnormalised O half row and (m, l_half) into the staging
      // row -- or, for a row of the slice this CTA merges itself, straight
      // into its own inbox slot (the K/V rings are free: every MMA has
      // completed)
      const int my_lo = rows_begin(split, ns);
      const bool mine = kMerge == kMergeCluster && r >= my_lo && r < rows_begin(split + 1, ns);
      const int rps = (kRows + ns - 1) / ns;
      uint8_t* srow = smem + (mine ? L::kInbox + (split * rps + r - my_lo) * L::kRowBytes : L::kStage + r * L::kRowBytes);
      // the half row's scale 2^-e: e from the exponent field of its largest
      // magnitude (fmaxf skips NaN), clamped so 2^-e and 2^e stay normal
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < DH; ++i) amax = fmaxf(amax, fabsf(o[i]));
      const int e = min(max((int)((__float_as_uint(amax) >> 23) & 0xffu) - 127 - 14, -100), 100);
      const float sc = __uint_as_float((uint32_t)(127 - e) << 23);
#pragma unroll
      for (int c = 0; c < DH / 8; ++c)
        *reinterpret_cast<uint4*>(srow + half * DH * 2 + 16 * c) =
            make_uint4(Pack<__half>::two(o[8 * c] * sc, o[8 * c + 1] * sc), Pack<__half>::two(o[8 * c + 2] * sc, o[8 * c + 3] * sc),
                       Pack<__half>::two(o[8 * c + 4] * sc, o[8 * c + 5] * sc),
                       Pack<__half>::two(o[8 * c + 6] * sc, o[8 * c + 7] * sc));
      float* ml = reinterpret_cast<float*>(srow + L::kRowMl);
      if (half == 0) ml[0] = m_run;
      ml[1 + half] = l_half;
      reinterpret_cast<int16_t*>(ml + 3)[half] = (int16_t)e;
      fence_proxy_async_smem();  // read by the bulk copies below
    }
    }  // not a row-tile pair
  }

  __syncwarp();  // warps 0 and 1 reconverge (one lane of each ran its role)
  // Every split's copy of row i of the slice is inbox row sp * rps + i.  One
  // thread per (row, 8 columns), a single pass: the thread forms the split
  // weights 2^(m_s - M) from the copies' maxima itself (broadcast loads shared
  // by the 16 threads of a row), accumulates the weighted O and the weighted
  // row sums, and divides once.
  auto merge_slice = [&](bool landed, int rps, int r_lo, int nr) {
    if (!landed || *s_abort != 0) return;
    const uint8_t* inbox = smem + L::kInbox;
    constexpr int C8 = D / 8;
    const int SS = rps * L::kRowBytes;  // bytes between two splits' copies of a row
    T* const obase = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)(kvh * G) * p.so[1];
    for (int item = tid; item < nr * C8; item += kThreads) {
      const int i = item / C8, c8 = (item - i * C8) * 8;
      const int rr = r_lo + i, tl = rr / G;
      const int tt = t0 + tl, gg = rr - tl * G;
      if (rr >= R || tt >= p.T) continue;
      const uint8_t* src = inbox + i * L::kRowBytes;
      float M = -INFINITY;
      for (int sp = 0; sp < ns; ++sp) M = fmaxf(M, *reinterpret_cast<const float*>(src + sp * SS + L::kRowMl));
      float4 a0 = make_float4(0.f, 0.f, 0.f, 0.f), a1 = a0;
      float lsum = 0.f;
      const int hh = c8 / (D / 2);  // the half row these 8 columns belong to
#pragma unroll 3
      for (int sp = 0; sp < ns; ++sp) {
        const uint8_t* sr = src + sp * SS;
        const float* ml = reinterpret_cast<const float*>(sr + L::kRowMl);
        const float m_s = ml[0];
        const float w = (m_s == -INFINITY) ? 0.f : ex2_approx(m_s - M);  // a split that saw nothing: 0
        lsum = fmaf(w, ml[1] + ml[2], lsum);
        // the O values carry the half row's factor 2^-e: weigh them by w 2^e
        const int e = reinterpret_cast<const int16_t*>(ml + 3)[hh];
        const float wo = w * __uint_as_float((uint32_t)(127 + e) << 23);
        const uint4 v = *reinterpret_cast<const uint4*>(sr + 2 * c8);
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
        const float2 f2 = __half22float2(*reinterpret_cast<const __half2*>(&v.z));
        const float2 f3 = __half22float2(*reinterpret_cast<const __half2*>(&v.w));
        a0.x = fmaf(wo, f0.x, a0.x);
        a0.y = fmaf(wo, f0.y, a0.y);
        a0.z = fmaf(wo, f1.x, a0.z);
        a0.w = fmaf(wo, f1.y, a0.w);
        a1.x = fmaf(wo, f2.x, a1.x);
        a1.y = fmaf(wo, f2.y, a1.y);
        a1.z = fmaf(wo, f3.x, a1.z);
        a1.w = fmaf(wo, f3.y, a1.w);
      }
      // lsum == 0 (the row sees no key at all): NaN, as tsfa.py:329
      const float inv = 1.f / lsum;
      uint4 o8;
      o8.x = Pack<T>::two(a0.x * inv, a0.y * inv);
      o8.y = Pack<T>::two(a0.z * inv, a0.w * inv);
      o8.z = Pack<T>::two(a1.x * inv, a1.y * inv);
      o8.w = Pack<T>::two(a1.z * inv, a1.w * inv);
      *reinterpret_cast<uint4*>(obase + (int64_t)gg * p.so[1] + (int64_t)tt * p.so[2] + c8) = o8;
    }
  };

  if constexpr (kMerge == kMergeGlobal) {
    // -------------------------------------------------- global merge (LSE)
    // (1) thread 0 bulk-stores the CTA's staged rows to its partial, waits for
    //     the store, and counts the CTA in on the group's arrival counter;
    // (2) thread 0 waits (bounded) until every split of the group has
    //     arrived -- the launch is cooperative, so they are all resident --
    //     and bulk-loads the rows of this CTA's slice from every split's
    //     partial into the inbox (bytes counted on the merge barrier), then
    //     counts the CTA out on the group's departure counter: the last CTA
    //     of the group to do so resets both counters to zero;
    // (3) merge_slice, as in the cluster merge.
    const int rps = (kRows + ns - 1) / ns;
    const int r_lo = rows_begin(split, ns), nr = rows_begin(split + 1, ns) - r_lo;
    const int gidx = (int)blockIdx.y * p.n_row_tiles + rtile;
    unsigned int* arrive = p.gsync + kSyncWordsPerGroup * gidx;
    unsigned int* depart = arrive + 1;
    uint8_t* gbase = p.partials + (size_t)gidx * ns * kRows * L::kRowBytes;
    __syncthreads();  // every staging row is written (and fenced for the async proxy)
    if (tid == 0) {
      bool ok = *s_abort == 0;
      if (ok) {
        bulk_store_s2g(gbase + (size_t)split * kRows * L::kRowBytes, smem_addr(smem + L::kStage),
                       (uint32_t)(kRows * L::kRowBytes));
        bulk_commit_group();
        bulk_wait_group_all();
        fence_proxy_async_global();
        __threadfence();
        atomicAdd(arrive, 1u);
        const uint64_t t_start = globaltimer_ns();
        while (ld_acquire_gpu(arrive) < (unsigned int)ns) {
          if (*s_abort != 0 || globaltimer_ns() - t_start > wl) {
            ok = false;
            break;
          }
        }
      }
      if (ok) {
        fence_proxy_async_global();
        mbar_arrive_expect_tx(&bars.merge, (uint32_t)(ns * nr * L::kRowBytes));
        for (int sp = 0; sp < ns; ++sp)
          bulk_load_g2s(smem_addr(smem + L::kInbox) + (uint32_t)(sp * rps * L::kRowBytes),
                        gbase + ((size_t)sp * kRows + r_lo) * L::kRowBytes, (uint32_t)(nr * L::kRowBytes),
                        &bars.merge);
      } else {
        raise_abort(s_abort, p.status, kSiteMerge, split);
      }
      // Past the wait on `arrive`: count out while the loads are in flight;
      // the last CTA of the group to do so resets both counters.
      if (atomicAdd(depart, 1u) == (unsigned int)ns - 1) {
        *arrive = 0u;
        *depart = 0u;
      }
    }
    const bool landed = __all_sync(kFull, mbar_wait(&bars.merge, 0, s_abort, wl));
    if (!landed && lane == 0) raise_abort(s_abort, p.status, kSiteMerge, split);
    merge_slice(landed, rps, r_lo, nr);
  } else if constexpr (kMerge == kMergeCluster) {
    // -------------------------------------------------- cluster merge (LSE)
    // (1) cluster barrier: every CTA has left its main loop and staged its
    //     rows, and its inbox (over the K/V rings) is free;
    // (2) lane c of warp 0 sends CTA c the staged rows of c's slice (owner c
    //     merges rows [c*128/ns, (c+1)*128/ns)) with one bulk shared::cta ->
    //     shared::cluster copy; the bytes complete on c's merge barrier
    //     (expected since setup);
    // (3) each owner merges its rows from its inbox (its own rows were staged
    //     there directly) with merge_slice;
    // (4) cluster barrier (execution only: each copy's landing was observed
    //     by its owner's merge barrier): no CTA leaves while a copy out of its
    //     shared memory may still be in flight.
    cluster_sync();
    const int rps = (kRows + ns - 1) / ns;  // inbox rows per source split
    const int r_lo = rows_begin(split, ns), nr = rows_begin(split + 1, ns) - r_lo;
    if (warp == 0 && lane < ns && lane != split && *s_abort == 0) {
      const int c = lane;
      const int c_lo = rows_begin(c, ns), c_rows = rows_begin(c + 1, ns) - c_lo;
      bulk_copy_s2cluster(mapa_shared(smem_addr(smem + L::kInbox) + (uint32_t)(split * rps * L::kRowBytes), (uint32_t)c),
                          smem_addr(smem + L::kStage) + (uint32_t)(c_lo * L::kRowBytes),
                          (uint32_t)(c_rows * L::kRowBytes), mapa_shared(smem_addr(&bars.merge), (uint32_t)c));
    }
    // The wait ignores this CTA's own abort flag: peers that did not abort
    // still send their rows, and they must land before this CTA's shared
    // memory goes away.  (A peer that aborted sends nothing: the wait then
    // runs out at the limit.)
    const bool landed = __all_sync(kFull, mbar_wait(&bars.merge, 0, nullptr, wl));
    if (!landed && lane == 0) raise_abort(s_abort, p.status, kSiteMerge, split);
    merge_slice(landed, rps, r_lo, nr);
    cluster_sync_relaxed();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  });
  return fn;
}

// 4-D map, dims ordered (d, dim1, dim2, dim3) by the caller, SW128 boxes.
bool encode_4d(CUtensorMap* m, const void* base, bool bf16, const uint64_t dims[4], const uint64_t strides_bytes[3],
               const uint32_t box[4]) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gd[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t gs[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t bx[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t es[4] = {1, 1, 1, 1};
  const CUresult r = fn(m, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                        const_cast<void*>(base), gd, gs, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <bool kPaged, int kMerge, bool kPair = false>
void* kernel_for_t(int head_dim, bool bf16) {
  if (head_dim == 128)
    return bf16 ? reinterpret_cast<void*>(&fwd_tc_kernel<128, __nv_bfloat16, kPaged, kMerge, kPair>)
                : reinterpret_cast<void*>(&fwd_tc_kernel<128, __half, kPaged, kMerge, kPair>);
  return bf16 ? reinterpret_cast<void*>(&fwd_tc_kernel<64, __nv_bfloat16, kPaged, kMerge, kPair>)
              : reinterpret_cast<void*>(&fwd_tc_kernel<64, __half, kPaged, kMerge, kPair>);
}
// pair: row-tile pairs (contiguous K/V, one split only)
void* kernel_for(int head_dim, bool bf16, bool paged, int merge, bool pair = false) {
  if (pair) return kernel_for_t<false, kMergeNone, true>(head_dim, bf16);
  if (paged) {
    switch (merge) {
      case kMergeNone: return kernel_for_t<true, kMergeNone>(head_dim, bf16);
      case kMergeGlobal: return kernel_for_t<true, kMergeGlobal>(head_dim, bf16);
      default: return kernel_for_t<true, kMergeCluster>(head_dim, bf16);
    }
  }
  switch (merge) {
    case kMergeNone: return kernel_for_t<false, kMergeNone>(head_dim, bf16);
    case kMergeGlobal: return kernel_for_t<false, kMergeGlobal>(head_dim, bf16);
    default: return kernel_for_t<false, kMergeCluster>(head_dim, bf16);
  }
}

// Dynamic shared memory of an instantiation (its V ring and Q tiles).
template <int D>
int smem_bytes_t(int merge, bool pair) {
  if (pair) return Layout<D, v_stages(true, true), 2>::kAlloc;
  return merge == kMergeNone ? Layout<D, v_stages(true, false), 1>::kAlloc : Layout<D, v_stages(false, false), 1>::kAlloc;
}
int smem_bytes(int head_dim, int merge, bool pair = false) {
  return head_dim == 128 ? smem_bytes_t<128>(merge, pair) : smem_bytes_t<64>(merge, pair);
}

// Shared-memory opt-in and non-portable cluster sizes for this kernel, once
// per (device, kernel).
int prepare_kernel(void* kern, int smem) {
  static std::mutex mu;
  static std::set<std::pair<int, void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({dev, kern})) return 0;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  if (e != cudaSuccess) {
    record_cuda_error(e, "cudaFuncSetAttribute(fwd kernel)");
    return -1;
  }
  done.insert({dev, kern});
  return 0;
}

}  // namespace tc

// Whether `ctas` CTAs of the forward kernel can be launched cooperatively
// (all resident at once), once per (device, kernel).
bool fwd_tc_can_cooperate(int head_dim, int dtype, int ctas) {
  using namespace tc;
  void* kern = kernel_for(head_dim, dtype == TSFA_DTYPE_BF16, false, kMergeGlobal);
  const int smem = smem_bytes(head_dim, kMergeGlobal);
  if (prepare_kernel(kern, smem) != 0) {
    cudaGetLastError();
    return false;
  }
  static std::mutex mu;
  static std::map<std::pair<int, void*>, int> cache;  // resident CTAs, 0 = no cooperative launch
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lk(mu);
  auto it = cache.find({dev, kern});
  if (it == cache.end()) {
    int coop = 0, sms = 0, per_sm = 0;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, (size_t)smem) != cudaSuccess) {
      cudaGetLastError();
      coop = 0;
    }
    it = cache.emplace(std::make_pair(dev, kern), coop ? sms * per_sm : 0).first;
  }
  return ctas <= it->second;
}

// Largest cluster size n <= want such that `groups` clusters of n CTAs are
// resident at once (one wave), per cudaOccupancyMaxActiveClusters.
int fwd_tc_pick_splits(int head_dim, int dtype, int groups, int want) {
  using namespace tc;
  void* kern = kernel_for(head_dim, dtype == TSFA_DTYPE_BF16, false, kMergeCluster);
  const int smem = smem_bytes(head_dim, kMergeCluster);
  if (prepare_kernel(kern, smem) != 0) {
    cudaGetLastError();
    return 1;
  }
  for (int n = want; n >= 2; --n) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(n * groups), 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = (size_t)smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = (unsigned)n;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (clusters >= groups) return n;
  }
  return 1;
}

int fwd_tc_launch(const FwdParams& p, int head_dim, int dtype, bool after_meta, cudaStream_t stream) {
  using namespace tc;
  const bool bf16 = dtype == TSFA_DTYPE_BF16;
  const int D = head_dim;
  TmaMaps<true> maps;  // the paged set; a contiguous launch passes its first three maps
  {
    // Q: dims (d, head, t, batch); box (64, G, t_per_tile, 1) -> rows g + G * t_local
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.Hq, (uint64_t)p.T, (uint64_t)p.B};
    const uint64_t st[3] = {(uint64_t)p.sq[1] * 2, (uint64_t)p.sq[2] * 2, (uint64_t)p.sq[0] * 2};
    const uint32_t box[4] = {64u, (uint32_t)p.G, (uint32_t)p.t_per_tile, 1u};
    if (!encode_4d(&maps.q, p.q, bf16, dims, st, box)) return TSFA_ERR_CUDA;
  }
  if (p.paged) {
    // K / V page pools: dims (d, kv-head, token in page, page); box
    // (64, 1, min(page_size, 128), 1) lands that many key rows of 128 B.
    // Boxes start at multiples of 8 rows (page_size >= 8), 1024-byte
    // aligned in shared memory as the SW128 pattern needs.
    const uint64_t ps = 1ull << p.page_shift;
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.Hkv, ps, (uint64_t)p.num_pages};
    const uint32_t box[4] = {64u, 1u, (uint32_t)(ps < (uint64_t)kKeys ? ps : (uint64_t)kKeys), 1u};
    const uint64_t sk[3] = {(uint64_t)p.sk[2] * 2, (uint64_t)p.sk[1] * 2, (uint64_t)p.sk[0] * 2};
    const uint64_t sv[3] = {(uint64_t)p.sv[2] * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
    if (!encode_4d(&maps.k, p.k, bf16, dims, sk, box)) return TSFA_ERR_CUDA;
    if (!encode_4d(&maps.v, p.v, bf16, dims, sv, box)) return TSFA_ERR_CUDA;
    // the gathered tree keys: dense [B][Hkv][T][D], box (64, 128, 1, 1)
    const uint64_t tdims[4] = {(uint64_t)D, (uint64_t)(p.T > 0 ? p.T : 1), (uint64_t)p.Hkv, (uint64_t)p.B};
    const uint64_t ts[3] = {(uint64_t)D * 2, (uint64_t)D * 2 * tdims[1], (uint64_t)D * 2 * tdims[1] * p.Hkv};
    const uint32_t tbox[4] = {64u, (uint32_t)kKeys, 1u, 1u};
    if (!encode_4d(&maps.kt, p.tree_k, bf16, tdims, ts, tbox)) return TSFA_ERR_CUDA;
    if (!encode_4d(&maps.vt, p.tree_v, bf16, tdims, ts, tbox)) return TSFA_ERR_CUDA;
  } else {
    // K / V: dims (d, key, kv-head, batch); box (64, 128, 1, 1)
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.kv_len, (uint64_t)p.Hkv, (uint64_t)p.B};
    const uint32_t box[4] = {64u, (uint32_t)kKeys, 1u, 1u};
    const uint64_t sk[3] = {(uint64_t)p.sk[2] * 2, (uint64_t)p.sk[1] * 2, (uint64_t)p.sk[0] * 2};
    const uint64_t sv[3] = {(uint64_t)p.sv[2] * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
    if (!encode_4d(&maps.k, p.k, bf16, dims, sk, box)) return TSFA_ERR_CUDA;
    if (!encode_4d(&maps.v, p.v, bf16, dims, sv, box)) return TSFA_ERR_CUDA;
  }
  const int merge = p.n_splits <= 1 ? kMergeNone : (p.global_merge ? kMergeGlobal : kMergeCluster);
  const bool pair = p.pair != 0 && merge == kMergeNone && !p.paged;
  void* kern = kernel_for(D, bf16, p.paged != 0, merge, pair);
  const int smem = smem_bytes(D, merge, pair);
  if (prepare_kernel(kern, smem) != 0) return TSFA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(pair ? (p.n_row_tiles + 1) / 2 : p.n_row_tiles * p.n_splits), (unsigned)(p.B * p.Hkv), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int na = 0;
  if (merge == kMergeGlobal) {
    // every CTA of the grid resident at once: the splits wait for each other
    attr[na].id = cudaLaunchAttributeCooperative;
    attr[na].val.cooperative = 1;
    ++na;
  }
  if (merge == kMergeCluster) {
    // the splits of a row tile form one cluster
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = (unsigned)p.n_splits;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  // after the metadata kernel: start as soon as it lets us (it does so at its
  // start); only the tree-list warp and the tree tiles wait for its results
  attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[na].val.programmaticStreamSerializationAllowed = 1;
  if (after_meta) ++na;
  cfg.attrs = attr;
  cfg.numAttrs = (unsigned)na;
  void* args[2] = {const_cast<FwdParams*>(&p), &maps};
  cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
  if (e != cudaSuccess && after_meta) {  // without the overlap, should the pair of attributes be refused
    cudaGetLastError();
    cfg.numAttrs = (unsigned)(na - 1);  // the programmatic serialization attribute is the last
    e = cudaLaunchKernelExC(&cfg, kern, args);
  }
  TSFA_CUDA_CHECK(e);
  TSFA_CUDA_CHECK(cudaGetLastError());
  return TSFA_OK;
}

}  // namespace tsfa
