// K1: tree-mask -> block-CSR metadata on the device.
//
// Replaces the host double loop of prepare_tree_sparse_metadata
// (tree_sparse_flashattn.py:103-147) and _pack_block_mask_to_int32
// (tree_sparse_flashattn.py:44-64).  One launch, two phases:
//
//   phase A -- pack + count.  Lane l of the ballot for word w of a tile owns
//     flat index i = 32 w + l of the zero-padded BM x BN tile (i = r * BN + c),
//     so the ballot IS payload word w (bit i % 32 of word i / 32, LSB first,
//     bit 31 the int32 sign).  popc of the ballots counts the visible bits of
//     the clipped region, which decides ZERO / FULL / MIXED as tsfa.py:113-134.
//   phase B -- emit.  Block-wide exclusive scans of the "nonzero" and "mixed"
//     flags in row-major tile order give the CSR positions and payload
//     offsets; row_ptr / col_idx / blk_type / offset are written and the MIXED
//     tiles' words copied into the compact payload.
//
// Small problems (every verify shape of the benchmark configs) run as a single
// CTA per mask with the words in shared memory: all 32 warps share the
// (tile, word) units, so a 64 x 64 tile costs 4 ballots per warp.  Per-batch
// trees add one CTA per mask; a paged K/V cache adds CTAs that gather the
// tree keys' K and V into the workspace.  The small path is instantiated per
// mask dtype and launched with programmatic stream serialization: it first
// waits for the kernel ahead of it, then lets the forward start.  Large
// problems spread phase A over the SMs (one warp per tile, words in the
// workspace) and the last CTA to arrive runs phase B.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <set>
#include <utility>

#include "tsfa_common.cuh"
#include "tsfa_sm100.cuh"

namespace tsfa {

constexpr int kMetaThreads = 1024;
constexpr int kSmallMaxTiles = 1024;
constexpr int kSmallMaxWords = 8192;
// Masks of at most this many bytes are first copied to shared memory with
// 16-byte loads (one round of global-memory latency instead of one per eight
// words), then packed from there.
constexpr int kStageBytes = 16384;

struct MetaWs {
  unsigned int* ticket;
  int8_t* tile_class;  // 0 ZERO, 1 FULL, 2 MIXED
  int32_t* mixed_ord;  // ordinal among MIXED tiles, -1 otherwise
  uint32_t* words;     // [ntiles * W]
};

inline size_t meta_ws_layout(int64_t ntiles, int64_t W, size_t* off_class, size_t* off_ord, size_t* off_words) {
  size_t o = TSFA_SYNC_BYTES;
  *off_class = o;
  o = align_up(o + (size_t)ntiles, 256);
  *off_ord = o;
  o = align_up(o + (size_t)ntiles * 4, 256);
  *off_words = o;
  o = align_up(o + (size_t)(ntiles * W) * 4, 256);
  return o;
}

struct MaskSrc {
  const char* base;
  int64_t row_stride_bytes;
  int dtype;
  int T, BM, BN, ntb, W;
};

// Raw bits of mask elements of type DT (compile time) and their visibility:
// nonzero, ignoring the sign bit of floating types (Tensor.to(torch.bool)).
template <int DT> struct MaskRaw;
template <> struct MaskRaw<TSFA_MASK_B8> { using U = uint8_t; static constexpr uint64_t kMask = 0xffull; };
template <> struct MaskRaw<TSFA_MASK_I16> { using U = uint16_t; static constexpr uint64_t kMask = 0xffffull; };
template <> struct MaskRaw<TSFA_MASK_I32> { using U = uint32_t; static constexpr uint64_t kMask = 0xffffffffull; };
template <> struct MaskRaw<TSFA_MASK_I64> { using U = unsigned long long; static constexpr uint64_t kMask = ~0ull; };
template <> struct MaskRaw<TSFA_MASK_F16> { using U = uint16_t; static constexpr uint64_t kMask = 0x7fffull; };
template <> struct MaskRaw<TSFA_MASK_BF16> { using U = uint16_t; static constexpr uint64_t kMask = 0x7fffull; };
template <> struct MaskRaw<TSFA_MASK_F32> { using U = uint32_t; static constexpr uint64_t kMask = 0x7fffffffull; };
template <> struct MaskRaw<TSFA_MASK_F64> { using U = unsigned long long; static constexpr uint64_t kMask = 0x7fffffffffffffffull; };

// a / d for 0 <= a < 2^24 and 0 < d < 2^24 through the float reciprocal: the
// estimate is within one of the quotient, and one correction step fixes it.
struct FastDiv {
  int d;
  float inv;
};
__device__ __forceinline__ FastDiv make_fastdiv(int d) { return FastDiv{d, 1.f / (float)d}; }
__device__ __forceinline__ int fdiv(int a, FastDiv f) {
  int q = __float2int_rz((float)a * f.inv);
  const int r = a - q * f.d;
  q += (r >= f.d) - (r < 0);
  return q;
}

// Phase A of the single-CTA path: warp `warp` of `nw` builds a contiguous
// range of words (u = tile * W + w, tiles row-major), walking (tile, w)
// incrementally.  Eight words per round: their mask elements are loaded
// unconditionally (lanes outside the mask read its first element and are
// masked off afterwards), so the loads of a round are in flight together.
template <int DT, bool kStaged>
__device__ __forceinline__ void small_words(const MaskSrc& m, int ntiles, uint32_t* s_words, int warp, int nw,
                                            int lane) {
  using U = typename MaskRaw<DT>::U;
  constexpr int K = 8;
  const int units = ntiles * m.W;
  const int area = m.BM * m.BN;
  const int per = (units + nw - 1) / nw;
  const int u_begin = warp * per, u_end = min(units, u_begin + per);
  if (u_begin >= u_end) return;
  const FastDiv dBN = make_fastdiv(m.BN);
  int tile = fdiv(u_begin, make_fastdiv(m.W));
  int w = u_begin - tile * m.W;
  int qb = fdiv(tile, make_fastdiv(m.ntb));
  int tb = tile - qb * m.ntb;
  for (int u = u_begin; u < u_end; u += K) {
    U raw[K];
    unsigned in_bits = 0u;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int flat = w * 32 + lane;
      const int r = fdiv(flat, dBN), c = flat - r * m.BN;
      const int q = qb * m.BM + r, k = tb * m.BN + c;
      const bool in = (u + j < u_end) && flat < area && q < m.T && k < m.T;
      const U* src = reinterpret_cast<const U*>(m.base + (in ? (int64_t)q * m.row_stride_bytes : 0)) + (in ? k : 0);
      raw[j] = kStaged ? *src : __ldg(src);  // staged: a copy in shared memory
      in_bits |= (unsigned)in << j;
      if (++w == m.W) {
        w = 0;
        if (++tb == m.ntb) {
          tb = 0;
          ++qb;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const bool vis = ((in_bits >> j) & 1u) && (((uint64_t)raw[j] & MaskRaw<DT>::kMask) != 0);
      const unsigned int word = __ballot_sync(0xffffffffu, vis);
      if (u + j < u_end && lane == 0) s_words[u + j] = word;
    }
  }
}

// Ballot word w of tile (qb, tb): bit l <-> flat index 32 w + l.
__device__ __forceinline__ unsigned int tile_word(const MaskSrc& m, int qb, int tb, int w, int lane) {
  const int q0 = qb * m.BM, k0 = tb * m.BN;
  const int rows = min(m.BM, m.T - q0), cols = min(m.BN, m.T - k0);
  const int flat = w * 32 + lane;
  bool vis = false;
  if (flat < m.BM * m.BN) {
    const int r = flat / m.BN;
    const int c = flat - r * m.BN;
    if (r < rows && c < cols) vis = mask_elem_visible(m.base + (int64_t)(q0 + r) * m.row_stride_bytes, k0 + c, m.dtype);
  }
  return __ballot_sync(0xffffffffu, vis);
}

__device__ __forceinline__ int tile_class_of(const MaskSrc& m, int qb, int tb, int ones) {
  const int rows = min(m.BM, m.T - qb * m.BM), cols = min(m.BN, m.T - tb * m.BN);
  return ones == 0 ? 0 : (ones == rows * cols ? 1 : 2);
}

// Phase B.  `cls(tile)` and `word(i)` read phase A's results; `ord` is scratch
// for the MIXED ordinal of every tile.
template <class ClsFn, class WordFn>
__device__ void meta_emit(const MaskSrc& m, int nqb, const TsfaMeta& out, ClsFn cls_of, WordFn word_of,
                          int32_t* ord) {
  __shared__ int s_warp_nz[kMetaThreads / 32];
  __shared__ int s_warp_mx[kMetaThreads / 32];
  __shared__ int s_carry[2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int ntb = m.ntb, W = m.W;
  const int ntiles = nqb * ntb;  // < 2^31 (the payload capacity is checked on the host)
  if (threadIdx.x == 0) {
    s_carry[0] = 0;
    s_carry[1] = 0;
    out.row_ptr[0] = 0;
  }
  __syncthreads();
  for (int base = 0; base < ntiles; base += blockDim.x) {
    const int tile = base + threadIdx.x;
    const int cls = tile < ntiles ? cls_of(tile) : 0;
    const int nz = cls != 0, mx = cls == 2;
    int snz = nz, smx = mx;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int a = __shfl_up_sync(0xffffffffu, snz, d);
      const int b = __shfl_up_sync(0xffffffffu, smx, d);
      if (lane >= d) {
        snz += a;
        smx += b;
      }
    }
    if (lane == 31) {
      s_warp_nz[warp] = snz;
      s_warp_mx[warp] = smx;
    }
    __syncthreads();
    if (warp == 0) {
      int a = lane < nw ? s_warp_nz[lane] : 0;
      int b = lane < nw ? s_warp_mx[lane] : 0;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, a, d);
        const int y = __shfl_up_sync(0xffffffffu, b, d);
        if (lane >= d) {
          a += x;
          b += y;
        }
      }
      if (lane < nw) {
        s_warp_nz[lane] = a;
        s_warp_mx[lane] = b;
      }
    }
    __syncthreads();
    const int pos = s_carry[0] + (warp ? s_warp_nz[warp - 1] : 0) + snz - nz;
    const int mpos = s_carry[1] + (warp ? s_warp_mx[warp - 1] : 0) + smx - mx;
    if (tile < ntiles) {
      const int qb = (int)((unsigned)tile / (unsigned)ntb), tb = tile - qb * ntb;
      if (nz) {
        out.col_idx[pos] = tb;
        out.blk_type[pos] = mx ? (int8_t)TSFA_MIXED_BLOCK : (int8_t)TSFA_FULL_BLOCK;
        out.mixed_mask_offset[pos] = mx ? mpos * W : 0;
      }
      ord[tile] = mx ? mpos : -1;
      if (tb == ntb - 1) out.row_ptr[qb + 1] = pos + nz;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      s_carry[0] += s_warp_nz[nw - 1];
      s_carry[1] += s_warp_mx[nw - 1];
    }
    __syncthreads();
  }
  // payload: thread t copies word w of every tile whose MIXED ordinal o >= 0,
  // walking (tile, w) without a division per word
  const int step_t = blockDim.x / W, step_w = blockDim.x - step_t * W;  // blockDim = step_t * W + step_w
  int tile = (int)((unsigned)threadIdx.x / (unsigned)W), w = threadIdx.x - tile * W;
  for (; tile < ntiles;) {
    const int o = ord[tile];
    if (o >= 0) out.mixed_mask_payload[(int64_t)o * W + w] = (int32_t)word_of((int64_t)tile * W + w);
    tile += step_t;
    w += step_w;
    if (w >= W) {
      w -= W;
      ++tile;
    }
  }
  if (threadIdx.x == 0) {
    out.counts[0] = s_carry[0];
    out.counts[1] = s_carry[1];
  }
}

// Gather role: CTA `cta` of g.ctas copies 16-byte chunks of the tree keys'
// K and V rows (16-bit elements) from the pages into the dense buffers.
__device__ __forceinline__ void tree_gather(const TreeGather& g, int cta) {
  const int chunks = g.D / 8;  // 16-byte chunks per row
  const int64_t total = (int64_t)g.B * g.Hkv * g.T * chunks;
  const int ps_mask = (1 << g.page_shift) - 1;
  for (int64_t i = (int64_t)cta * blockDim.x + threadIdx.x; i < total; i += (int64_t)g.ctas * blockDim.x) {
    const int c = (int)(i % chunks);
    const int64_t row = i / chunks;
    const int t = (int)(row % g.T);
    const int64_t bh = row / g.T;
    const int h = (int)(bh % g.Hkv), b = (int)(bh / g.Hkv);
    const int n = g.prefix_len + t;
    uint4 kv = make_uint4(0u, 0u, 0u, 0u), vv = kv;
    if (n < g.kv_len) {
      const int lo = __ldg(g.page_indptr + b), cnt = __ldg(g.page_indptr + b + 1) - lo;
      const int pi = n >> g.page_shift;
      if (pi < cnt) {
        const int page = __ldg(g.page_indices + lo + pi);
        if (page >= 0 && page < g.num_pages) {
          const int slot = n & ps_mask;
          kv = *reinterpret_cast<const uint4*>(g.k_pages + 2 * (page * g.ks[0] + slot * g.ks[1] + h * g.ks[2]) + 16 * c);
          vv = *reinterpret_cast<const uint4*>(g.v_pages + 2 * (page * g.vs[0] + slot * g.vs[1] + h * g.vs[2]) + 16 * c);
        }
      }
    }
    const int64_t off = 2 * (row * g.D) + 16 * c;
    *reinterpret_cast<uint4*>(g.tree_k + off) = kv;
    *reinterpret_cast<uint4*>(g.tree_v + off) = vv;
  }
}

__global__ void __launch_bounds__(kMetaThreads) tree_gather_kernel(TreeGather g) {
  sm100::griddep_launch_dependents();
  tree_gather(g, blockIdx.x);
}

// Single CTA per metadata set: words, popcounts and classes in shared
// memory.  CTA i builds the set of mask i (per-batch trees, MetaBatch
// strides; one CTA and zero strides for a single tree).
// kGather (paged K/V only): CTAs past the n_sets metadata CTAs gather the
// tree keys; the contiguous op's instantiation carries no gather code.
// One instantiation per mask dtype: a launch carries only its own dtype's
// packing code.
template <bool kGather, int DT>
__global__ void __launch_bounds__(kMetaThreads) meta_build_small_kernel(MaskSrc m, int nqb, TsfaMeta out,
                                                                         MetaBatch mb, int n_sets, TreeGather g) {
  // Launched with programmatic stream serialization, this grid may be
  // resident before the kernel ahead of it on the stream has finished: wait
  // for it (it may have written the mask, or still read the metadata this
  // grid overwrites) before anything else.  Then the forward kernel may
  // start: it waits for this grid only before it reads the metadata.
  const int64_t bi = blockIdx.x;
  const int esz = mask_elem_bytes(DT);
  const int row_bytes = m.T * esz;
  const bool staged = (int64_t)row_bytes * m.T <= kStageBytes;
  if (staged && (int)bi < n_sets) {
    // warm L2 with this CTA's mask rows while the kernel ahead of us runs (a
    // prefetch reads nothing into the program; the copy below follows the wait)
    const char* mb0 = m.base + bi * mb.mask_bytes;
    const int lines = (row_bytes + 127) / 128;
    for (int i = threadIdx.x; i < m.T * lines; i += blockDim.x) {
      const int r = i / lines, l = i - r * lines;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(mb0 + (int64_t)r * m.row_stride_bytes + 128 * l));
    }
  }
  sm100::griddep_wait();
  sm100::griddep_launch_dependents();
  if constexpr (kGather) {
    if ((int)blockIdx.x >= n_sets) {
      tree_gather(g, (int)blockIdx.x - n_sets);
      return;
    }
  }
  m.base += bi * mb.mask_bytes;
  out.row_ptr += bi * mb.rp;
  out.col_idx += bi * mb.tile;
  out.blk_type += bi * mb.tile;
  out.mixed_mask_offset += bi * mb.tile;
  out.mixed_mask_payload += bi * mb.payload;
  out.counts += 2 * bi;
  __shared__ uint32_t s_words[kSmallMaxWords];
  __shared__ int s_ones[kSmallMaxTiles];
  __shared__ int32_t s_ord[kSmallMaxTiles];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int ntiles = nqb * m.ntb;
  if (staged) {
    // the mask rows, packed, in shared memory: 16-byte loads when the rows
    // allow them (all issued before the first is used), else element loads
    extern __shared__ __align__(16) uint8_t s_stage[];
    const bool vec = row_bytes % 16 == 0 && m.row_stride_bytes % 16 == 0 &&
                     (reinterpret_cast<uintptr_t>(m.base) & 15u) == 0;
    if (vec) {
      const int chunks = row_bytes / 16, total = chunks * m.T;
      for (int i = threadIdx.x; i < total; i += blockDim.x) {
        const int r = i / chunks, c = i - r * chunks;
        reinterpret_cast<uint4*>(s_stage)[i] =
            __ldg(reinterpret_cast<const uint4*>(m.base + (int64_t)r * m.row_stride_bytes) + c);
      }
    } else {
      for (int i = threadIdx.x; i < row_bytes * m.T; i += blockDim.x) {
        const int r = i / row_bytes, c = i - r * row_bytes;
        s_stage[i] = __ldg(reinterpret_cast<const uint8_t*>(m.base + (int64_t)r * m.row_stride_bytes) + c);
      }
    }
    __syncthreads();
    MaskSrc ms = m;
    ms.base = reinterpret_cast<const char*>(s_stage);
    ms.row_stride_bytes = row_bytes;
    small_words<DT, true>(ms, ntiles, s_words, warp, nw, lane);
  } else {
    small_words<DT, false>(m, ntiles, s_words, warp, nw, lane);
  }
  __syncthreads();
  // classes: a warp per tile sums the popcounts of its words (no shared
  // atomics: every word of a tile would hit the same counter)
  for (int tile = warp; tile < ntiles; tile += nw) {
    int ones = 0;
    for (int i = lane; i < m.W; i += 32) ones += __popc(s_words[tile * m.W + i]);
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) ones += __shfl_xor_sync(0xffffffffu, ones, d);
    if (lane == 0) {
      const int qb = tile / m.ntb, tb = tile - qb * m.ntb;
      s_ones[tile] = tile_class_of(m, qb, tb, ones);
    }
  }
  __syncthreads();
  meta_emit(
      m, nqb, out, [&](int64_t t) { return s_ones[t]; }, [&](int64_t i) { return s_words[i]; }, s_ord);
}

// Grid: phase A with one warp per tile (words unrolled for memory-level
// parallelism), phase B in the last CTA to arrive.
__global__ void __launch_bounds__(kMetaThreads) meta_build_large_kernel(MaskSrc m, int nqb, TsfaMeta out,
                                                                         MetaWs ws) {
  sm100::griddep_launch_dependents();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int64_t ntiles = (int64_t)nqb * m.ntb;
  for (int64_t tile = (int64_t)blockIdx.x * nw + warp; tile < ntiles; tile += (int64_t)gridDim.x * nw) {
    const int qb = (int)(tile / m.ntb), tb = (int)(tile - (int64_t)qb * m.ntb);
    int ones = 0;
    int w = 0;
    for (; w + 8 <= m.W; w += 8) {
      unsigned int v[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = tile_word(m, qb, tb, w + j, lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        ones += __popc(v[j]);
        if (lane == j) ws.words[tile * m.W + w + j] = v[j];
      }
    }
    for (; w < m.W; ++w) {
      const unsigned int v = tile_word(m, qb, tb, w, lane);
      ones += __popc(v);
      if (lane == 0) ws.words[tile * m.W + w] = v;
    }
    if (lane == 0) ws.tile_class[tile] = (int8_t)tile_class_of(m, qb, tb, ones);
  }
  __shared__ int s_last;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicInc(ws.ticket, gridDim.x - 1) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  meta_emit(
      m, nqb, out, [&](int64_t t) { return (int)__ldcg(ws.tile_class + t); },
      [&](int64_t i) { return __ldcg(ws.words + i); }, ws.mixed_ord);
}

// _pack_block_mask_to_int32 for one tile: one warp per output word.
__global__ void pack_tile_kernel(const char* __restrict__ base, int dtype, int64_t row_stride_bytes, int rows,
                                 int cols, int words, int32_t* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int nw = (gridDim.x * blockDim.x) >> 5;
  for (int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < words; w += nw) {
    const int64_t flat = (int64_t)w * 32 + lane;
    bool vis = false;
    if (flat < (int64_t)rows * cols) {
      const int r = (int)(flat / cols), c = (int)(flat - (int64_t)r * cols);
      vis = mask_elem_visible(base + (int64_t)r * row_stride_bytes, c, dtype);
    }
    const unsigned int word = __ballot_sync(0xffffffffu, vis);
    if (lane == 0) out[w] = (int32_t)word;
  }
}

int pack_tile_launch(const void* tile, int dtype, int64_t row_stride, int rows, int cols, int32_t* out,
                     cudaStream_t stream) {
  const int64_t words = cdiv64((int64_t)rows * cols, 32);
  if (words == 0) return TSFA_OK;
  const int threads = 256;
  const int grid = (int)std::min<int64_t>(cdiv64(words * 32, threads), 4 * kSmCount);
  pack_tile_kernel<<<grid, threads, 0, stream>>>(static_cast<const char*>(tile), dtype,
                                                 row_stride * mask_elem_bytes(dtype), rows, cols, (int)words, out);
  TSFA_CUDA_CHECK(cudaGetLastError());
  return TSFA_OK;
}

template <bool kGather>
void* small_kernel_for_t(int32_t dtype) {
  switch (dtype) {
    case TSFA_MASK_B8: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_B8>);
    case TSFA_MASK_I16: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_I16>);
    case TSFA_MASK_I32: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_I32>);
    case TSFA_MASK_I64: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_I64>);
    case TSFA_MASK_F16: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_F16>);
    case TSFA_MASK_BF16: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_BF16>);
    case TSFA_MASK_F32: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_F32>);
    case TSFA_MASK_F64: return reinterpret_cast<void*>(&meta_build_small_kernel<kGather, TSFA_MASK_F64>);
    default: return nullptr;
  }
}
void* small_kernel_for(int32_t dtype, bool gather) {
  return gather ? small_kernel_for_t<true>(dtype) : small_kernel_for_t<false>(dtype);
}

// Opt-in for the staged mask's dynamic shared memory, once per (device, kernel).
int allow_stage_smem(void* kern) {
  static std::mutex mu;
  static std::set<std::pair<int, void*>> done;
  int dev = 0;
  TSFA_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lk(mu);
  if (done.count({dev, kern})) return 0;
  TSFA_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kStageBytes));
  done.insert({dev, kern});
  return 0;
}

// Work area of the large path: tile classes, MIXED ordinals, words.
size_t meta_area_bytes(int64_t ntiles, int64_t W) {
  size_t a, b, c;
  return meta_ws_layout(ntiles, W, &a, &b, &c) - TSFA_SYNC_BYTES;
}

// Launches K1 for `nbatch` masks (mask i at tree_mask + i * mb.mask_bytes,
// its set at `out` + i * the MetaBatch element strides, its counts at
// out.counts + 2 i).  `ticket` is a zero-initialised arrival counter (left at
// zero); `area` (meta_area_bytes) is only touched by the large path, which
// runs the masks one after another.
int meta_build_batched_launch(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                              int32_t block_m, int32_t block_n, const TsfaMeta& out, int nbatch, const MetaBatch& mb,
                              unsigned int* ticket, char* area, size_t area_bytes, cudaStream_t stream,
                              const TreeGather* gather) {
  TreeGather g{};
  if (gather) g = *gather;
  const int64_t nqb = cdiv64(q_len, block_m), ntb = cdiv64(q_len, block_n);
  const int64_t W = cdiv64((int64_t)block_m * block_n, 32);
  const int64_t ntiles = nqb * ntb;
  MaskSrc m;
  m.base = static_cast<const char*>(tree_mask);
  m.row_stride_bytes = mask_row_stride * mask_elem_bytes(mask_dtype);
  m.dtype = mask_dtype;
  m.T = q_len;
  m.BM = block_m;
  m.BN = block_n;
  m.ntb = (int)ntb;
  m.W = (int)W;
  if (nbatch <= 0) return TSFA_OK;
  if (ntiles <= kSmallMaxTiles && ntiles * W <= kSmallMaxWords) {
    const bool gather = g.ctas > 0;
    void* kern = small_kernel_for(mask_dtype, gather);
    if (!kern) return TSFA_ERR_UNSUPPORTED;
    int n_sets = nbatch, nq = (int)nqb;
    void* args[6] = {&m, &nq, const_cast<TsfaMeta*>(&out), const_cast<MetaBatch*>(&mb), &n_sets, &g};
    // early launch behind the previous kernel (the grid waits for it first)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(nbatch + (gather ? g.ctas : 0)));
    // as many threads as the words need (a ballot per word, ~8 per warp):
    // a few warps make the block-wide scans of a small mask cheap, and the
    // forward it releases early is waiting on its result
    int threads = 128;
    while (threads < kMetaThreads && threads * 8 < ntiles * W) threads *= 2;
    cfg.blockDim = dim3((unsigned)(gather ? kMetaThreads : threads));
    // the shared-memory copy of a small mask (with the static arrays above
    // the 48 KB that needs no opt-in: the attribute is set once per device)
    if ((int64_t)q_len * q_len * mask_elem_bytes(mask_dtype) <= kStageBytes) {
      if (allow_stage_smem(kern) != 0) return TSFA_ERR_CUDA;
      cfg.dynamicSmemBytes = kStageBytes;
    }
    cfg.stream = stream;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelExC(&cfg, kern, args);
    if (e != cudaSuccess) {  // plain stream order then
      cudaGetLastError();
      cfg.numAttrs = 0;
      e = cudaLaunchKernelExC(&cfg, kern, args);
    }
    TSFA_CUDA_CHECK(e);
  } else {
    size_t oc, oo, ow;
    meta_ws_layout(ntiles, W, &oc, &oo, &ow);
    if (!area || !ticket || area_bytes < meta_area_bytes(ntiles, W)) return TSFA_ERR_WORKSPACE;
    MetaWs ws;
    ws.ticket = ticket;
    ws.tile_class = reinterpret_cast<int8_t*>(area + (oc - TSFA_SYNC_BYTES));
    ws.mixed_ord = reinterpret_cast<int32_t*>(area + (oo - TSFA_SYNC_BYTES));
    ws.words = reinterpret_cast<uint32_t*>(area + (ow - TSFA_SYNC_BYTES));
    const int warps = kMetaThreads / 32;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(cdiv64(ntiles, warps), 2 * kSmCount));
    for (int i = 0; i < nbatch; ++i) {  // the work area is shared: one mask after another
      MaskSrc mi = m;
      mi.base += i * mb.mask_bytes;
      TsfaMeta oi = out;
      oi.row_ptr += i * mb.rp;
      oi.col_idx += i * mb.tile;
      oi.blk_type += i * mb.tile;
      oi.mixed_mask_offset += i * mb.tile;
      oi.mixed_mask_payload += i * mb.payload;
      oi.counts += 2 * i;
      meta_build_large_kernel<<<grid, kMetaThreads, 0, stream>>>(mi, (int)nqb, oi, ws);
      TSFA_CUDA_CHECK(cudaGetLastError());
    }
    // the last kernel before the forward: its dependency wait covers this
    // gather and, in stream order, the metadata kernels before it
    if (g.ctas > 0) tree_gather_kernel<<<g.ctas, kMetaThreads, 0, stream>>>(g);
  }
  TSFA_CUDA_CHECK(cudaGetLastError());
  return TSFA_OK;
}

int meta_build_launch(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride, int32_t q_len,
                      int32_t block_m, int32_t block_n, const TsfaMeta& out, unsigned int* ticket, char* area,
                      size_t area_bytes, cudaStream_t stream) {
  return meta_build_batched_launch(tree_mask, mask_dtype, mask_row_stride, q_len, block_m, block_n, out, 1,
                                   MetaBatch{}, ticket, area, area_bytes, stream, nullptr);
}

}  // namespace tsfa
