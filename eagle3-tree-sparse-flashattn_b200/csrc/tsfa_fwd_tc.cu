// Forward kernel for sm_100a: TMA + tcgen05/TMEM, warp-specialised, split-KV
// over a thread-block cluster with a DSMEM log-sum-exp merge.
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
// kv-head folded into MMA M) x one contiguous slice of the group's 128-key
// tiles.  The slices of a group are the CTAs of one cluster.
//
//   warp 0      TMA producer: Q once, then K/V tiles into a 2-stage ring.
//   warp 1      TMEM allocator + tcgen05.mma issuer (one lane):
//                 S[a&1] = Q K_a^T       (SS, K-major SW128, M=128 N=128)
//                 O     += P_a V_a       (SS, P K-major, V MN-major, N=D)
//               S is double-buffered in TMEM so S(a+1) overlaps softmax(a).
//   warps 2-5   softmax: thread = TMEM lane = row.  tcgen05.ld the S row,
//               mask (bitsets decoded in registers), one FFMA + ex2 per key,
//               P (bf16/fp16) to SW128 shared memory.  O stays in TMEM and is
//               rescaled lazily (row max grew by > 2^8), warp-collectively.
//               Tree tiles also write the rounding residual of P and the MMA
//               warp adds P_lo V (keeps ~16 mantissa bits on rows that see a
//               handful of keys).
//   epilogue    with one split: normalise + store.  With a cluster: every CTA
//               parks its unnormalised O (fp32) and (m, l) in shared memory,
//               cluster barrier, CTA c merges rows [c*128/n, (c+1)*128/n)
//               from all CTAs' shared memory, cluster barrier, exit.
//
// Every mbarrier wait is bounded in wall time; one that runs out raises the
// CTA's abort flag and writes the status block (site, tile, CTA), and all
// roles wind down (the producer lets its own copies land) before TMEM is
// freed.  Decisions that guard warp-collective tcgen05.ld/st are warp-uniform.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <mutex>
#include <set>
#include <utility>

#include "tsfa_fwd.cuh"
#include "tsfa_sm100.cuh"

namespace tsfa {
namespace tc {

using namespace sm100;

constexpr int kRows = 128;
constexpr int kKeys = 128;
constexpr int kStages = 2;
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr float kRescaleLog2 = 8.f;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColO = 256;  // S buffers at columns 0 and 128
constexpr unsigned kFull = 0xffffffffu;

struct TmaMaps {
  CUtensorMap q, k, v;
};

template <int D>
struct Layout {
  static constexpr int kBox = kRows * 128;  // 128 rows x 128 B: one 64-column SW128 box (16 KB)
  static constexpr int kDH = D / 64;        // 64-column halves of head_dim
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kDH * kBox;
  static constexpr int kV = kK + kStages * kDH * kBox;
  static constexpr int kP = kV + kStages * kDH * kBox;  // P: 128 rows x 128 keys
  static constexpr int kPL = kP + 2 * kBox;             // residual of P (tree tiles)
  static constexpr int kBytes = kPL + 2 * kBox;
  static constexpr int kAlloc = kBytes + 1024;  // room to align the base to 1024 B
  // merge staging (after the last MMA): O partial fp32 [128][D] over K, (m, l) over V
  static constexpr int kMergeO = kK;
  static constexpr int kMergeML = kV;
  static_assert(kRows * D * 4 <= kStages * kDH * kBox, "O partial must fit the K ring");
};

struct Bars {
  uint64_t q_full;
  uint64_t k_full[kStages], v_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], s_empty[2];
  uint64_t p_full, o_done, list_ready;
};

template <typename T>
struct Pack;
template <>
struct Pack<__nv_bfloat16> {
  static constexpr bool kBf16 = true;
  static __device__ __forceinline__ uint32_t two(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo_of(uint32_t w) { return __uint_as_float(w << 16); }
  static __device__ __forceinline__ float hi_of(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }
};
template <>
struct Pack<__half> {
  static constexpr bool kBf16 = false;
  static __device__ __forceinline__ uint32_t two(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo_of(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
  }
  static __device__ __forceinline__ float hi_of(uint32_t w) {
    return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
  }
};

// Wait sites reported in the workspace status block when a wait gives up.
enum WaitSite : int {
  kSiteListProducer = 1, kSiteKvEmpty, kSiteQFull, kSiteListMma, kSiteKFull, kSiteSEmpty, kSitePFull, kSiteVFull,
  kSiteSFull, kSiteODone, kSiteODoneEpi
};

// status[0] = TSFA_ERR_DEVICE_TIMEOUT; status[1..3] = first site, tile, CTA.
__device__ __forceinline__ void raise_abort(volatile int* flag, int* status, int site, int tile) {
  *flag = 1;
  if (atomicCAS(status, 0, TSFA_ERR_DEVICE_TIMEOUT) == 0) {
    status[1] = site;
    status[2] = tile;
    status[3] = (int)(blockIdx.y * gridDim.x + blockIdx.x);
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads, 1) fwd_tc_kernel(const __grid_constant__ FwdParams p,
                                                             const __grid_constant__ TmaMaps maps) {
  using L = Layout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem + L::kQ;
  uint8_t* sK = smem + L::kK;
  uint8_t* sV = smem + L::kV;
  uint8_t* sP = smem + L::kP;
  uint8_t* sPL = smem + L::kPL;
  __shared__ Bars bars;
  __shared__ uint32_t s_tmem;
  __shared__ int s_tree_list[kMaxTreeTileList];
  __shared__ unsigned int s_bitmap[kMaxTreeTileList / 32];
  __shared__ int s_tree_count;
  __shared__ int s_abort_storage;
  volatile int* s_abort = &s_abort_storage;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int ns = p.n_splits;
  const int split = blockIdx.x % ns;  // == rank in the cluster
  const int rtile = blockIdx.x / ns;
  const int unit = blockIdx.y;
  const int b = unit / p.Hkv, kvh = unit - b * p.Hkv;
  const int G = p.G, TPT = p.t_per_tile, R = G * TPT;
  const int t0 = rtile * TPT;
  const int t_hi = min(t0 + TPT, p.T) - 1;
  const int n_tiles = p.n_prefix_tiles + p.n_tree_tiles;
  const int j0 = (int)((int64_t)split * n_tiles / ns);  // balanced slice of the key tiles
  const int j1 = (int)((int64_t)(split + 1) * n_tiles / ns);
  const int n_pre = max(0, min(j1, p.n_prefix_tiles) - j0);
  const int tr0 = max(j0, p.n_prefix_tiles) - p.n_prefix_tiles;
  const int tr1 = max(j1, p.n_prefix_tiles) - p.n_prefix_tiles;

  if (tid == 0) {
    mbar_init(&bars.q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars.k_full[s], 1);
      mbar_init(&bars.v_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars.s_full[s], 1);
      mbar_init(&bars.s_empty[s], kSoftmaxThreads);
    }
    mbar_init(&bars.p_full, kSoftmaxThreads);
    mbar_init(&bars.o_done, 1);
    mbar_init(&bars.list_ready, 1);
    s_abort_storage = 0;
    s_tree_count = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&maps.q);
    prefetch_tmap(&maps.k);
    prefetch_tmap(&maps.v);
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    bool ok = true;
    int issued = 0, site = 0, at = 0;
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars.q_full, (uint32_t)(L::kDH * 128 * R));
      for (int h = 0; h < L::kDH; ++h) tma_load_4d(sQ + h * L::kBox, &maps.q, &bars.q_full, h * 64, kvh * G, t0, b);
    }
    __syncwarp();
    int n_total = n_pre;
    bool have_list = false;
    for (int a = 0;; ++a) {
      if (a == n_pre && !have_list) {
        ok = __all_sync(kFull, mbar_wait(&bars.list_ready, 0, s_abort));
        if (!ok) {
          site = kSiteListProducer;
          at = a;
          break;
        }
        n_total = n_pre + s_tree_count;
        have_list = true;
      }
      if (a >= n_total) break;
      const int stage = a & 1;
      if (a >= kStages) {
        ok = __all_sync(kFull, mbar_wait(&bars.kv_empty[stage], ((a - kStages) >> 1) & 1, s_abort));
        if (!ok) {
          site = kSiteKvEmpty;
          at = a;
          break;
        }
      }
      const int n0 = a < n_pre ? (j0 + a) * kKeys : p.P + s_tree_list[a - n_pre] * kKeys;
      if (lane == 0) {
        uint8_t* kd = sK + stage * L::kDH * L::kBox;
        uint8_t* vd = sV + stage * L::kDH * L::kBox;
        mbar_arrive_expect_tx(&bars.k_full[stage], (uint32_t)(L::kDH * L::kBox));
        for (int h = 0; h < L::kDH; ++h) tma_load_4d(kd + h * L::kBox, &maps.k, &bars.k_full[stage], h * 64, n0, kvh, b);
        mbar_arrive_expect_tx(&bars.v_full[stage], (uint32_t)(L::kDH * L::kBox));
        for (int h = 0; h < L::kDH; ++h) tma_load_4d(vd + h * L::kBox, &maps.v, &bars.v_full[stage], h * 64, n0, kvh, b);
      }
      __syncwarp();
      issued = a + 1;
    }
    if (!ok) {
      if (lane == 0) raise_abort(s_abort, p.status, site, at);
      // let this CTA's own copies land before the shared memory goes away
      mbar_wait(&bars.q_full, 0, nullptr);
      for (int a = max(0, issued - kStages); a < issued; ++a) {
        mbar_wait(&bars.k_full[a & 1], (a >> 1) & 1, nullptr);
        mbar_wait(&bars.v_full[a & 1], (a >> 1) & 1, nullptr);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idS = idesc_f16(Pack<T>::kBf16, 128, kKeys, false);
    constexpr uint32_t idPV = idesc_f16(Pack<T>::kBf16, 128, D, true);
    const uint32_t aQ = smem_addr(sQ), aK = smem_addr(sK), aV = smem_addr(sV), aP = smem_addr(sP),
                   aPL = smem_addr(sPL);
    int site = 0, at = 0;
    bool ok = __all_sync(kFull, mbar_wait(&bars.q_full, 0, s_abort));
    if (!ok) site = kSiteQFull;
    int n_total = n_pre;
    bool have_list = false;
    auto fail = [&](int s_, int a) -> bool {
      site = s_;
      at = a;
      return false;
    };
    auto ensure = [&](int a) -> bool {
      if (a >= n_pre && !have_list) {
        if (!__all_sync(kFull, mbar_wait(&bars.list_ready, 0, s_abort))) return fail(kSiteListMma, a);
        n_total = n_pre + s_tree_count;
        have_list = true;
      }
      return true;
    };
    auto issue_s = [&](int a) -> bool {
      const int stage = a & 1;
      if (!__all_sync(kFull, mbar_wait(&bars.k_full[stage], (a >> 1) & 1, s_abort))) return fail(kSiteKFull, a);
      if (a >= 2 && !__all_sync(kFull, mbar_wait(&bars.s_empty[a & 1], ((a - 2) >> 1) & 1, s_abort)))
        return fail(kSiteSEmpty, a);
      tc_fence_after();
      if (lane == 0) {
        const uint32_t kbase = aK + stage * L::kDH * L::kBox;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * L::kBox + (kk & 3) * 32;
          umma_f16_ss(tmem + (uint32_t)(a & 1) * kKeys, sw128_desc(aQ + off, 16, 1024),
                      sw128_desc(kbase + off, 16, 1024), idS, kk > 0);
        }
        umma_commit(&bars.s_full[a & 1]);
      }
      __syncwarp();
      return true;
    };
    auto issue_pv = [&](int a) -> bool {
      const int stage = a & 1;
      const uint32_t vbase = aV + stage * L::kDH * L::kBox;
      if (!__all_sync(kFull, mbar_wait(&bars.p_full, a & 1, s_abort))) return fail(kSitePFull, a);
      if (!__all_sync(kFull, mbar_wait(&bars.v_full[stage], (a >> 1) & 1, s_abort))) return fail(kSiteVFull, a);
      tc_fence_after();
      if (lane == 0) {
        const int parts = a >= n_pre ? 2 : 1;  // tree tiles: P_hi V + P_lo V
        for (int part = 0; part < parts; ++part) {
          const uint32_t pbase = part ? aPL : aP;
#pragma unroll
          for (int kk = 0; kk < kKeys / 16; ++kk) {
            const uint32_t poff = (kk >> 2) * L::kBox + (kk & 3) * 32;
            umma_f16_ss(tmem + kColO, sw128_desc(pbase + poff, 16, 1024),
                        sw128_desc(vbase + kk * 16 * 128, L::kBox, 1024), idPV,
                        (a > 0 || part > 0 || kk > 0) ? 1u : 0u);
          }
        }
        umma_commit(&bars.kv_empty[stage]);
        umma_commit(&bars.o_done);
      }
      __syncwarp();
      return true;
    };
    if (ok) ok = ensure(0);
    if (ok && n_total > 0) ok = issue_s(0);
    for (int a = 0; ok && a < n_total; ++a) {
      ok = ensure(a + 1);
      if (ok && a + 1 < n_total) ok = issue_s(a + 1);
      if (ok) ok = issue_pv(a);
    }
    if (!ok && lane == 0) raise_abort(s_abort, p.status, site, at);
  } else {
    // ------------------------------------------------------------ softmax
    const int st = tid - 64;               // 0..127
    const int r = 32 * (warp & 3) + lane;  // TMEM lane == row of the tile
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    const int tl = r / G;
    const int t = t0 + tl;
    const bool row_valid = (r < R) && (t < p.T);
    const float sl2 = p.scale_log2;

    // tree tiles this row tile needs: union of the CSR entries of its q-blocks
    if (st < kMaxTreeTileList / 32) s_bitmap[st] = 0u;
    named_barrier(1, kSoftmaxThreads);
    if (tr1 > tr0) {
      const int BM = p.mv.block_m, BN = p.mv.block_n;
      const int e0 = __ldg(p.mv.row_ptr + t0 / BM);
      const int e1 = __ldg(p.mv.row_ptr + t_hi / BM + 1);
      for (int e = e0 + st; e < e1; e += kSoftmaxThreads) {
        const int tb = __ldg(p.mv.col_idx + e);
        const int lo = (tb * BN) / kKeys, hi = min((tb * BN + BN - 1) / kKeys, p.n_tree_tiles - 1);
        for (int jt = max(lo, tr0); jt <= min(hi, tr1 - 1); ++jt) atomicOr(&s_bitmap[jt >> 5], 1u << (jt & 31));
      }
    }
    named_barrier(1, kSoftmaxThreads);
    if (st == 0) {
      int c = 0;
      for (int jt = tr0; jt < tr1; ++jt)
        if ((s_bitmap[jt >> 5] >> (jt & 31)) & 1u) s_tree_list[c++] = jt;
      s_tree_count = c;
      mbar_arrive(&bars.list_ready);
    }
    named_barrier(1, kSoftmaxThreads);
    const int n_total = n_pre + s_tree_count;

    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    int site = 0, at = 0;
    for (int a = 0; a < n_total && ok; ++a) {
      const bool is_tree = a >= n_pre;
      const int n0 = is_tree ? p.P + s_tree_list[a - n_pre] * kKeys : (j0 + a) * kKeys;
      // keys of this tile the row sees: all of a full prefix tile; else a mask
      const bool full = row_valid && !is_tree && n0 + kKeys <= p.P;
      unsigned long long vis_lo = 0ull, vis_hi = 0ull;
      if (!full && row_valid) {
        if (!is_tree) {
          const int nv = p.P - n0;  // 0 < nv < 128: keys n < P (tsfa.py:270)
          vis_lo = nv >= 64 ? ~0ull : ((1ull << nv) - 1ull);
          vis_hi = nv > 64 ? ((1ull << (nv - 64)) - 1ull) : 0ull;
        } else {
          const int c0 = n0 - p.P;
          const int lim = min(kKeys, p.kv_len - n0);
          vis_lo = tree_row_bits(p.mv, t, c0, min(64, lim), p.T);
          vis_hi = lim > 64 ? tree_row_bits(p.mv, t, c0 + 64, lim - 64, p.T) : 0ull;
        }
      }
      // tcgen05.ld / st are warp-collective (.sync.aligned): every decision
      // that guards one is warp-uniform.
      if (!__all_sync(kFull, mbar_wait(&bars.s_full[a & 1], (a >> 1) & 1, s_abort))) {
        ok = false;
        site = kSiteSFull;
        at = a;
        break;
      }
      tc_fence_after();
      float x[kKeys];
      {
        uint32_t* xr = reinterpret_cast<uint32_t*>(x);
#pragma unroll
        for (int i = 0; i < kKeys / 32; ++i)
          tmem_ld32(tmem + lane_base + (uint32_t)(a & 1) * kKeys + 32 * i, xr + 32 * i);
        tmem_ld_wait();
      }
      tc_fence_before();
      mbar_arrive(&bars.s_empty[a & 1]);
      if (!full) {
#pragma unroll
        for (int i = 0; i < 64; ++i) x[i] = ((vis_lo >> i) & 1ull) ? x[i] : -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; ++i) x[64 + i] = ((vis_hi >> i) & 1ull) ? x[64 + i] : -INFINITY;
      }
      // row max of the raw scores: 8 independent chains
      float mx8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) mx8[j] = x[j];
#pragma unroll
      for (int i = 8; i < kKeys; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], x[i]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const float m_new = fmaxf(m_run, mx * sl2);  // scale > 0: max commutes with it
      if (a > 0) {
        // P's buffers and O are free once the previous P.V finished
        if (!__all_sync(kFull, mbar_wait(&bars.o_done, (a - 1) & 1, s_abort))) {
          ok = false;
          site = kSiteODone;
          at = a;
          break;
        }
        tc_fence_after();
      }
      // Lazy rescale: the reference max m_run only moves when the row max
      // grows by more than 2^8 (p stays <= 256 otherwise).  A row whose O is
      // still exactly zero (m_run = -inf) just adopts the new max.
      const bool need = (m_run != -INFINITY) && (m_new > m_run + kRescaleLog2);
      if (m_run == -INFINITY) m_run = m_new;
      if (__any_sync(kFull, need)) {
        const float alpha = need ? ex2_approx(m_run - m_new) : 1.f;
#pragma unroll
        for (int i = 0; i < D / 32; ++i) {
          uint32_t o[32];
          tmem_ld32(tmem + lane_base + kColO + 32 * i, o);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] = __float_as_uint(__uint_as_float(o[j]) * alpha);
          tmem_st32(tmem + lane_base + kColO + 32 * i, o);
        }
        tmem_st_wait();
        if (need) {
          l_run *= alpha;
          m_run = m_new;
        }
      }
      // p = 2^(s * scale_log2 - m): one FFMA + ex2 per key.  s = -inf gives 0;
      // a row that has seen nothing (m_run = -inf) uses 0 as its offset.
      const float moff = (m_run == -INFINITY) ? 0.f : m_run;
      float rs8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) rs8[j] = 0.f;
#pragma unroll
      for (int i = 0; i < kKeys; ++i) {
        x[i] = ex2_approx(fmaf(x[i], sl2, -moff));
        rs8[i & 7] += x[i];
      }
      l_run += ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      // P row into the K-major SW128 layout: 16-byte chunk c of row r sits at
      // chunk (c ^ (r & 7)) of the row's 128-byte line; tree tiles also store
      // the rounding residual p - rn(p) into the second buffer.
#pragma unroll
      for (int c = 0; c < kKeys / 8; ++c) {
        uint32_t w[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) w[j] = Pack<T>::two(x[c * 8 + 2 * j], x[c * 8 + 2 * j + 1]);
        const uint32_t off = (c >> 3) * L::kBox + r * 128 + (((c & 7) ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(sP + off) = make_uint4(w[0], w[1], w[2], w[3]);
        if (is_tree) {
          uint32_t z[4];
#pragma unroll
          for (int j = 0; j < 4; ++j)
            z[j] = Pack<T>::two(x[c * 8 + 2 * j] - Pack<T>::lo_of(w[j]), x[c * 8 + 2 * j + 1] - Pack<T>::hi_of(w[j]));
          *reinterpret_cast<uint4*>(sPL + off) = make_uint4(z[0], z[1], z[2], z[3]);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bars.p_full);
    }
    if (!ok) raise_abort(s_abort, p.status, site, at);

    // ---------------------------------------------------------- epilogue
    float o[D];
#pragma unroll
    for (int i = 0; i < D; ++i) o[i] = 0.f;
    if (ok && n_total > 0) {
      ok = __all_sync(kFull, mbar_wait(&bars.o_done, (n_total - 1) & 1, s_abort));
      if (ok) {
        tc_fence_after();
        uint32_t* orr = reinterpret_cast<uint32_t*>(o);
#pragma unroll
        for (int i = 0; i < D / 32; ++i) tmem_ld32(tmem + lane_base + kColO + 32 * i, orr + 32 * i);
        tmem_ld_wait();
      } else {
        raise_abort(s_abort, p.status, kSiteODoneEpi, n_total);
      }
    }
    if (ns == 1) {
      named_barrier(1, kSoftmaxThreads);  // every softmax thread gets here exactly once
      if (*s_abort == 0 && row_valid) {
        const int g = r - tl * G;
        T* dst = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)(kvh * G + g) * p.so[1] +
                 (int64_t)t * p.so[2];
        const float inv = 1.f / l_run;  // l == 0 (row sees no key) gives NaN, as tsfa.py:329
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          uint4 w;
          w.x = Pack<T>::two(o[8 * c + 0] * inv, o[8 * c + 1] * inv);
          w.y = Pack<T>::two(o[8 * c + 2] * inv, o[8 * c + 3] * inv);
          w.z = Pack<T>::two(o[8 * c + 4] * inv, o[8 * c + 5] * inv);
          w.w = Pack<T>::two(o[8 * c + 6] * inv, o[8 * c + 7] * inv);
          *reinterpret_cast<uint4*>(dst + 8 * c) = w;
        }
      }
    } else {
      // park the split's unnormalised O (fp32, row-major) and (m, l); the K
      // and V rings are free: every MMA has completed (o_done above)
      float* po = reinterpret_cast<float*>(smem + L::kMergeO) + r * D;
#pragma unroll
      for (int c = 0; c < D / 4; ++c)
        *reinterpret_cast<float4*>(po + 4 * c) = make_float4(o[4 * c], o[4 * c + 1], o[4 * c + 2], o[4 * c + 3]);
      reinterpret_cast<float2*>(smem + L::kMergeML)[r] = make_float2(m_run, l_run);
    }
  }

  if (ns > 1) {
    // -------------------------------------------------- cluster merge (LSE)
    cluster_sync();  // every CTA's partial is in its shared memory
    if (warp >= 2 && *s_abort == 0) {
      const int wq = warp - 2;  // 4 merge warps
      constexpr int VPL = D / 32;
      const uint32_t aO = smem_addr(smem + L::kMergeO), aML = smem_addr(smem + L::kMergeML);
      const int r_lo = split * kRows / ns, r_hi = (split + 1) * kRows / ns;
      for (int rr = r_lo + wq; rr < r_hi; rr += 4) {
        const int tt = t0 + rr / G, gg = rr - (rr / G) * G;
        if (rr >= R || tt >= p.T) continue;
        const float2 ml =
            lane < ns ? ld_dsmem_f2(mapa_shared(aML + rr * 8, (uint32_t)lane)) : make_float2(-INFINITY, 0.f);
        float M = ml.x;
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) M = fmaxf(M, __shfl_xor_sync(kFull, M, d));
        const float w = (ml.x == -INFINITY) ? 0.f : ex2_approx(ml.x - M);  // a split that saw nothing: 0
        float Lsum = w * ml.y;
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) Lsum += __shfl_xor_sync(kFull, Lsum, d);
        float acc[VPL];
#pragma unroll
        for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
        for (int s = 0; s < ns; ++s) {
          const float ws = __shfl_sync(kFull, w, s);
          const uint32_t src = mapa_shared(aO + (uint32_t)(rr * D + lane * VPL) * 4, (uint32_t)s);
          if constexpr (VPL == 4) {
            const float4 xv = ld_dsmem_f4(src);
            acc[0] = fmaf(ws, xv.x, acc[0]);
            acc[1] = fmaf(ws, xv.y, acc[1]);
            acc[2] = fmaf(ws, xv.z, acc[2]);
            acc[3] = fmaf(ws, xv.w, acc[3]);
          } else {
            const float2 xv = ld_dsmem_f2(src);
            acc[0] = fmaf(ws, xv.x, acc[0]);
            acc[1] = fmaf(ws, xv.y, acc[1]);
          }
        }
        const float inv = 1.f / Lsum;  // Lsum == 0 (row sees no key): NaN like tsfa.py:329
        T* dst = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)(kvh * G + gg) * p.so[1] +
                 (int64_t)tt * p.so[2] + lane * VPL;
#pragma unroll
        for (int i = 0; i < VPL; i += 2)
          *reinterpret_cast<uint32_t*>(dst + i) = Pack<T>::two(acc[i] * inv, acc[i + 1] * inv);
      }
    }
    cluster_sync();  // no CTA leaves while others still read its shared memory
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

void* kernel_for(int head_dim, bool bf16) {
  if (head_dim == 128)
    return bf16 ? reinterpret_cast<void*>(&fwd_tc_kernel<128, __nv_bfloat16>)
                : reinterpret_cast<void*>(&fwd_tc_kernel<128, __half>);
  return bf16 ? reinterpret_cast<void*>(&fwd_tc_kernel<64, __nv_bfloat16>)
              : reinterpret_cast<void*>(&fwd_tc_kernel<64, __half>);
}

int smem_bytes(int head_dim) { return head_dim == 128 ? Layout<128>::kAlloc : Layout<64>::kAlloc; }

// Shared-memory opt-in and non-portable cluster sizes for this kernel, once
// per (device, kernel).
int prepare_kernel(void* kern, int smem) {
  static std::mutex mu;
  static std::set<std::pair<int, void*>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({dev, kern})) return 0;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return -1;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) return -1;
  done.insert({dev, kern});
  return 0;
}

}  // namespace tc

// Largest cluster size n <= want such that `groups` clusters of n CTAs are
// resident at once (one wave), per cudaOccupancyMaxActiveClusters.
int fwd_tc_pick_splits(int head_dim, int dtype, int groups, int want) {
  using namespace tc;
  void* kern = kernel_for(head_dim, dtype == TSFA_DTYPE_BF16);
  const int smem = smem_bytes(head_dim);
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

int fwd_tc_launch(const FwdParams& p, int head_dim, int dtype, cudaStream_t stream) {
  using namespace tc;
  const bool bf16 = dtype == TSFA_DTYPE_BF16;
  const int D = head_dim;
  TmaMaps maps;
  {
    // Q: dims (d, head, t, batch); box (64, G, t_per_tile, 1) -> rows g + G * t_local
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.Hq, (uint64_t)p.T, (uint64_t)p.B};
    const uint64_t st[3] = {(uint64_t)p.sq[1] * 2, (uint64_t)p.sq[2] * 2, (uint64_t)p.sq[0] * 2};
    const uint32_t box[4] = {64u, (uint32_t)p.G, (uint32_t)p.t_per_tile, 1u};
    if (!encode_4d(&maps.q, p.q, bf16, dims, st, box)) return TSFA_ERR_CUDA;
  }
  {
    // K / V: dims (d, key, kv-head, batch); box (64, 128, 1, 1)
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)p.kv_len, (uint64_t)p.Hkv, (uint64_t)p.B};
    const uint32_t box[4] = {64u, (uint32_t)kKeys, 1u, 1u};
    const uint64_t sk[3] = {(uint64_t)p.sk[2] * 2, (uint64_t)p.sk[1] * 2, (uint64_t)p.sk[0] * 2};
    const uint64_t sv[3] = {(uint64_t)p.sv[2] * 2, (uint64_t)p.sv[1] * 2, (uint64_t)p.sv[0] * 2};
    if (!encode_4d(&maps.k, p.k, bf16, dims, sk, box)) return TSFA_ERR_CUDA;
    if (!encode_4d(&maps.v, p.v, bf16, dims, sv, box)) return TSFA_ERR_CUDA;
  }
  void* kern = kernel_for(D, bf16);
  const int smem = smem_bytes(D);
  if (prepare_kernel(kern, smem) != 0) return TSFA_ERR_CUDA;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(p.n_row_tiles * p.n_splits), (unsigned)(p.B * p.Hkv), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = (unsigned)p.n_splits;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  void* args[2] = {const_cast<FwdParams*>(&p), &maps};
  if (cudaLaunchKernelExC(&cfg, kern, args) != cudaSuccess) return TSFA_ERR_CUDA;
  return cudaGetLastError() == cudaSuccess ? TSFA_OK : TSFA_ERR_CUDA;
}

}  // namespace tsfa
