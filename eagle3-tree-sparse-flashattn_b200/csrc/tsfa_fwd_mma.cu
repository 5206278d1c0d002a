// Forward kernel, warp-MMA variant: split-KV prefix sweep + CSR tree walk.
//
// Semantics follow block_sparse_tree_fwd_kernel (tree_sparse_flashattn.py:163-339):
//   prefix keys [0, P) fully visible, masked to n < P (tsfa.py:266-270);
//   tree keys P + c visible iff the CSR/bitset says so and n < kv_len
//   (tsfa.py:284-318); online softmax with p = 0 where s = -inf and
//   alpha = 1 where both maxima are -inf (tsfa.py:272-279, 320-327);
//   O = acc / l with no l == 0 guard (tsfa.py:329).
// Layout: 4 warps x 16 rows = 64 folded rows per CTA, 64-key tiles, K/V
// double-buffered with cp.async into XOR-swizzled shared memory, fragments via
// ldmatrix, bf16/fp16 mma.sync m16n8k16 with fp32 accumulation, P re-used from
// the S accumulators as the A operand of P.V.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "tsfa_fwd.cuh"

namespace tsfa {
namespace mma {

constexpr int kRows = 64;
constexpr int kKeys = 64;
constexpr int kThreads = 128;

template <typename T>
struct Ty;
template <>
struct Ty<__nv_bfloat16> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo(uint32_t x) { return __uint_as_float(x << 16); }
  static __device__ __forceinline__ float hi(uint32_t x) { return __uint_as_float(x & 0xffff0000u); }
  static __device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};
template <>
struct Ty<__half> {
  static __device__ __forceinline__ uint32_t pack(float a, float b) {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float lo(uint32_t x) { return __half2float(__ushort_as_half((unsigned short)(x & 0xffffu))); }
  static __device__ __forceinline__ float hi(uint32_t x) { return __half2float(__ushort_as_half((unsigned short)(x >> 16))); }
  static __device__ __forceinline__ void mma(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t* r) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Byte offset of 16-byte chunk `c` of row `r` in a [rows][D] tile, chunks
// XOR-swizzled by the row's low 3 bits (conflict-free ldmatrix).
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return (uint32_t)(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

template <int D>
struct Smem {
  static constexpr int kTileBytes = kKeys * D * 2;
  static constexpr int kQBytes = kRows * D * 2;
  static constexpr int kBytes = kQBytes + 4 * kTileBytes;  // Q + 2 x (K, V)
};

template <int D, typename T>
__global__ void __launch_bounds__(kThreads, 2) fwd_mma_kernel(const FwdParams p) {
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* sQ = smem;
  unsigned char* sK0 = smem + Smem<D>::kQBytes;
  __shared__ unsigned long long s_tmask[kRows];
  __shared__ int s_tree_list[kMaxTreeTileList];
  __shared__ int s_tree_count;
  __shared__ unsigned int s_tree_bitmap[kMaxTreeTileList / 32];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int split = blockIdx.x % p.n_splits;
  const int rtile = blockIdx.x / p.n_splits;
  const int unit = blockIdx.y;  // b * Hkv + kvh
  const int b = unit / p.Hkv, kvh = unit - b * p.Hkv;
  const int G = p.G;
  const int f0 = rtile * kRows;  // first folded row of this tile
  const int t_lo = f0 / G;
  const int t_hi = min((f0 + kRows - 1) / G, p.T - 1);

  const T* qbase = static_cast<const T*>(p.q) + (int64_t)b * p.sq[0] + (int64_t)kvh * G * p.sq[1];
  const T* kbase = static_cast<const T*>(p.k) + (int64_t)b * p.sk[0] + (int64_t)kvh * p.sk[1];
  const T* vbase = static_cast<const T*>(p.v) + (int64_t)b * p.sv[0] + (int64_t)kvh * p.sv[1];

  // ---- key range of this split: prefix tiles, then active tree tiles -------
  const int n_tiles = p.n_prefix_tiles + p.n_tree_tiles;
  const int j0 = split * p.tiles_per_split;
  const int j1 = min(n_tiles, j0 + p.tiles_per_split);
  const int pre_end = min(j1, p.n_prefix_tiles);
  const int n_pre = max(0, pre_end - j0);
  const int tr0 = max(j0, p.n_prefix_tiles) - p.n_prefix_tiles;  // tree tile range [tr0, tr1)
  const int tr1 = max(j1, p.n_prefix_tiles) - p.n_prefix_tiles;
  if (tid < kMaxTreeTileList / 32) s_tree_bitmap[tid] = 0u;
  __syncthreads();
  if (tr1 > tr0) {
    // A tree tile is needed iff some CSR entry of the q-blocks covering
    // [t_lo, t_hi] overlaps it (ZERO tiles are skipped, tsfa.py:113-114).
    const int BM = p.mv.block_m, BN = p.mv.block_n;
    const int e0 = __ldg(p.mv.row_ptr + t_lo / BM);
    const int e1 = __ldg(p.mv.row_ptr + t_hi / BM + 1);
    for (int e = e0 + tid; e < e1; e += kThreads) {
      const int tb = __ldg(p.mv.col_idx + e);
      const int a = (tb * BN) / kKeys, z = min((tb * BN + BN - 1) / kKeys, p.n_tree_tiles - 1);
      for (int jt = max(a, tr0); jt <= min(z, tr1 - 1); ++jt) atomicOr(&s_tree_bitmap[jt >> 5], 1u << (jt & 31));
    }
  }
  __syncthreads();
  if (tid == 0) {
    int c = 0;
    for (int jt = tr0; jt < tr1; ++jt)
      if (s_tree_bitmap[jt >> 5] >> (jt & 31) & 1u) s_tree_list[c++] = jt;
    s_tree_count = c;
  }
  __syncthreads();
  const int n_active = n_pre + s_tree_count;

  // ---- loaders -------------------------------------------------------------
  auto load_q = [&]() {
    for (int i = tid; i < kRows * CH; i += kThreads) {
      const int r = i / CH, c = i - r * CH;
      const int f = f0 + r, t = f / G, g = f - t * G;
      const bool ok = t < p.T;
      const T* src = ok ? qbase + (int64_t)g * p.sq[1] + (int64_t)t * p.sq[2] + c * 8 : qbase;
      cp_async16(smem_u32(sQ + swz<D>(r, c)), src, ok);
    }
  };
  // key tile a (0-based among active tiles) -> first kv position
  auto tile_key0 = [&](int a) -> int {
    if (a < n_pre) return (j0 + a) * kKeys;
    return p.P + s_tree_list[a - n_pre] * kKeys;
  };
  auto load_kv = [&](int a, int stage) {
    const int n0 = tile_key0(a);
    unsigned char* sk = sK0 + stage * 2 * Smem<D>::kTileBytes;
    unsigned char* sv = sk + Smem<D>::kTileBytes;
    for (int i = tid; i < kKeys * CH; i += kThreads) {
      const int r = i / CH, c = i - r * CH;
      const int n = n0 + r;
      const bool ok = n < p.kv_len;
      const T* ks = ok ? kbase + (int64_t)n * p.sk[2] + c * 8 : kbase;
      const T* vs = ok ? vbase + (int64_t)n * p.sv[2] + c * 8 : vbase;
      cp_async16(smem_u32(sk + swz<D>(r, c)), ks, ok);
      cp_async16(smem_u32(sv + swz<D>(r, c)), vs, ok);
    }
  };

  load_q();
  if (n_active > 0) load_kv(0, 0);
  cp_async_commit();

  // ---- per-thread state: rows r0 = 16 warp + lane/4 and r1 = r0 + 8 --------
  const int rr0 = warp * 16 + (lane >> 2), rr1 = rr0 + 8;
  const int tq0 = (f0 + rr0) / G, tq1 = (f0 + rr1) / G;
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  uint32_t qf[D / 16][4];
  bool q_loaded = false;

  for (int a = 0; a < n_active; ++a) {
    const int stage = a & 1;
    if (a + 1 < n_active) load_kv(a + 1, stage ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    const bool is_tree = a >= n_pre;
    const int n0 = tile_key0(a);
    if (is_tree) {
      // visibility bits of each tree row of this tile for keys [n0, n0 + 64)
      const int nt = t_hi - t_lo + 1;
      for (int i = tid; i < nt; i += kThreads)
        s_tmask[i] = tree_row_bits(p.mv, t_lo + i, n0 - p.P, min(kKeys, p.kv_len - n0), p.T);
    }
    __syncthreads();
    if (!q_loaded) {
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int r = warp * 16 + (lane & 15), c = 2 * ks + (lane >> 4);
        ldsm_x4(smem_u32(sQ + swz<D>(r, c)), qf[ks]);
      }
      q_loaded = true;
    }
    const unsigned char* sk = sK0 + stage * 2 * Smem<D>::kTileBytes;
    const unsigned char* sv = sk + Smem<D>::kTileBytes;

    // S = Q K^T (16 x 64 per warp)
    float s[kKeys / 8][4];
#pragma unroll
    for (int i = 0; i < kKeys / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int nb = 0; nb < kKeys / 16; ++nb) {
        const int mi = lane >> 3;
        const int r = nb * 16 + (mi >> 1) * 8 + (lane & 7), c = 2 * ks + (mi & 1);
        uint32_t bf[4];
        ldsm_x4(smem_u32(sk + swz<D>(r, c)), bf);
        Ty<T>::mma(s[2 * nb], qf[ks], bf[0], bf[1]);
        Ty<T>::mma(s[2 * nb + 1], qf[ks], bf[2], bf[3]);
      }
    }

    // mask + scale into the exp2 domain
    unsigned long long mk0 = ~0ull, mk1 = ~0ull;
    if (is_tree) {
      mk0 = (tq0 < p.T) ? s_tmask[tq0 - t_lo] : 0ull;
      mk1 = (tq1 < p.T) ? s_tmask[tq1 - t_lo] : 0ull;
    } else if (n0 + kKeys > p.P) {
      const int nv = p.P - n0;  // keys n < P are visible (tsfa.py:270)
      const unsigned long long lim = nv >= 64 ? ~0ull : ((1ull << nv) - 1ull);
      mk0 = mk1 = lim;
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int nt = 0; nt < kKeys / 8; ++nt) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int col = nt * 8 + 2 * (lane & 3) + e;
        float x0 = s[nt][e] * p.scale_log2, x1 = s[nt][2 + e] * p.scale_log2;
        if (!((mk0 >> col) & 1ull)) x0 = -INFINITY;
        if (!((mk1 >> col) & 1ull)) x1 = -INFINITY;
        s[nt][e] = x0;
        s[nt][2 + e] = x1;
        mx0 = fmaxf(mx0, x0);
        mx1 = fmaxf(mx1, x1);
      }
    }
#pragma unroll
    for (int d = 1; d <= 2; d <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, d));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, d));
    }
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float al0 = (m0 == -INFINITY && mn0 == -INFINITY) ? 1.f : exp2f(m0 - mn0);
    const float al1 = (m1 == -INFINITY && mn1 == -INFINITY) ? 1.f : exp2f(m1 - mn1);
    float rs0 = 0.f, rs1 = 0.f;
    uint32_t pf[kKeys / 16][4];
    uint32_t pl[kKeys / 16][4];  // tree tiles: residual p - (p rounded), see below
#pragma unroll
    for (int nt = 0; nt < kKeys / 8; ++nt) {
      const float p00 = s[nt][0] == -INFINITY ? 0.f : exp2f(s[nt][0] - mn0);
      const float p01 = s[nt][1] == -INFINITY ? 0.f : exp2f(s[nt][1] - mn0);
      const float p10 = s[nt][2] == -INFINITY ? 0.f : exp2f(s[nt][2] - mn1);
      const float p11 = s[nt][3] == -INFINITY ? 0.f : exp2f(s[nt][3] - mn1);
      rs0 += p00 + p01;
      rs1 += p10 + p11;
      const uint32_t h0 = Ty<T>::pack(p00, p01), h1 = Ty<T>::pack(p10, p11);
      pf[nt >> 1][(nt & 1) * 2 + 0] = h0;
      pf[nt >> 1][(nt & 1) * 2 + 1] = h1;
      if (is_tree) {
        pl[nt >> 1][(nt & 1) * 2 + 0] = Ty<T>::pack(p00 - Ty<T>::lo(h0), p01 - Ty<T>::hi(h0));
        pl[nt >> 1][(nt & 1) * 2 + 1] = Ty<T>::pack(p10 - Ty<T>::lo(h1), p11 - Ty<T>::hi(h1));
      }
    }
    l0 = l0 * al0 + rs0;
    l1 = l1 * al1 + rs1;
    m0 = mn0;
    m1 = mn1;
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      o[dt][0] *= al0;
      o[dt][1] *= al0;
      o[dt][2] *= al1;
      o[dt][3] *= al1;
    }
    // O += P V
#pragma unroll
    for (int ks = 0; ks < kKeys / 16; ++ks) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        const int mi = lane >> 3;
        const int r = ks * 16 + (mi & 1) * 8 + (lane & 7), c = 2 * dp + (mi >> 1);
        uint32_t bf[4];
        ldsm_x4_t(smem_u32(sv + swz<D>(r, c)), bf);
        Ty<T>::mma(o[2 * dp], pf[ks], bf[0], bf[1]);
        Ty<T>::mma(o[2 * dp + 1], pf[ks], bf[2], bf[3]);
        if (is_tree) {
          // Tree rows can see only a handful of keys, where rounding p to the
          // 8-bit mantissa of bf16 (tsfa.py:278 does the same) would cost up
          // to 2^-9 |v|.  P = hi + lo keeps ~16 bits on the (few) tree tiles.
          Ty<T>::mma(o[2 * dp], pl[ks], bf[0], bf[1]);
          Ty<T>::mma(o[2 * dp + 1], pl[ks], bf[2], bf[3]);
        }
      }
    }
    __syncthreads();  // stage may be overwritten by the next prefetch
  }
  cp_async_wait<0>();

  // full row sums (each of the 4 lanes of a row holds a partial)
#pragma unroll
  for (int d = 1; d <= 2; d <<= 1) {
    l0 += __shfl_xor_sync(0xffffffffu, l0, d);
    l1 += __shfl_xor_sync(0xffffffffu, l1, d);
  }
  const int fa = f0 + rr0, fb = f0 + rr1;
  const int ta = fa / G, ga = fa - ta * G, tb_ = fb / G, gb = fb - tb_ * G;

  if (p.n_splits == 1) {
    T* obase = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)kvh * G * p.so[1];
    const float i0 = 1.f / l0, i1 = 1.f / l1;  // no l == 0 guard (tsfa.py:329)
#pragma unroll
    for (int dt = 0; dt < D / 8; ++dt) {
      const int d = dt * 8 + 2 * (lane & 3);
      if (ta < p.T)
        *reinterpret_cast<uint32_t*>(obase + (int64_t)ga * p.so[1] + (int64_t)ta * p.so[2] + d) =
            Ty<T>::pack(o[dt][0] * i0, o[dt][1] * i0);
      if (tb_ < p.T)
        *reinterpret_cast<uint32_t*>(obase + (int64_t)gb * p.so[1] + (int64_t)tb_ * p.so[2] + d) =
            Ty<T>::pack(o[dt][2] * i1, o[dt][3] * i1);
    }
    return;
  }

  // ---- split-KV: write the partial, last CTA of the group merges -----------
  const int group = unit * p.n_row_tiles + rtile;
  const int64_t slot = (int64_t)group * p.n_splits + split;
  float* po = p.part_o + slot * kRows * D;
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) {
    const int d = dt * 8 + 2 * (lane & 3);
    *reinterpret_cast<float2*>(po + rr0 * D + d) = make_float2(o[dt][0], o[dt][1]);
    *reinterpret_cast<float2*>(po + rr1 * D + d) = make_float2(o[dt][2], o[dt][3]);
  }
  if ((lane & 3) == 0) {
    p.part_ml[slot * kRows + rr0] = make_float2(m0, l0);
    p.part_ml[slot * kRows + rr1] = make_float2(m1, l1);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicInc(p.tickets + group, p.n_splits - 1) == (unsigned)(p.n_splits - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // warp w merges rows w, w + 4, ...; lane holds D/32 consecutive columns
  constexpr int VPL = D / 32;
  T* obase = static_cast<T*>(p.o) + (int64_t)b * p.so[0] + (int64_t)kvh * G * p.so[1];
  const int ns = p.n_splits;
  for (int r = warp; r < kRows; r += kThreads / 32) {
    const int f = f0 + r, t = f / G, g = f - t * G;
    if (t >= p.T) continue;
    const int64_t s0 = (int64_t)group * ns;
    float2 ml = lane < ns ? __ldcg(p.part_ml + (s0 + lane) * kRows + r) : make_float2(-INFINITY, 0.f);
    float M = ml.x;
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, d));
    // weight of split s: exp2(m_s - M), 0 for a split that saw no key
    const float w = (ml.x == -INFINITY) ? 0.f : exp2f(ml.x - M);
    float L = w * ml.y;
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1) L += __shfl_xor_sync(0xffffffffu, L, d);
    float acc[VPL];
#pragma unroll
    for (int i = 0; i < VPL; ++i) acc[i] = 0.f;
    for (int sidx = 0; sidx < ns; ++sidx) {
      const float ws = __shfl_sync(0xffffffffu, w, sidx);
      if (ws == 0.f) continue;
      const float* src = p.part_o + ((s0 + sidx) * kRows + r) * D + lane * VPL;
      if constexpr (VPL == 4) {
        const float4 x = __ldcg(reinterpret_cast<const float4*>(src));
        acc[0] += ws * x.x;
        acc[1] += ws * x.y;
        acc[2] += ws * x.z;
        acc[3] += ws * x.w;
      } else {
        const float2 x = __ldcg(reinterpret_cast<const float2*>(src));
        acc[0] += ws * x.x;
        acc[1] += ws * x.y;
      }
    }
    const float inv = 1.f / L;  // L == 0 (no visible key) gives NaN like tsfa.py:329
    T* dst = obase + (int64_t)g * p.so[1] + (int64_t)t * p.so[2] + lane * VPL;
#pragma unroll
    for (int i = 0; i < VPL; i += 2)
      *reinterpret_cast<uint32_t*>(dst + i) = Ty<T>::pack(acc[i] * inv, acc[i + 1] * inv);
  }
}

}  // namespace mma

int fwd_mma_launch(const FwdParams& p, int head_dim, int dtype, cudaStream_t stream) {
  dim3 grid(p.n_row_tiles * p.n_splits, p.B * p.Hkv);
  dim3 block(mma::kThreads);
#define TSFA_LAUNCH(D, T)                                                                                  \
  do {                                                                                                     \
    auto kern = mma::fwd_mma_kernel<D, T>;                                                                 \
    const int smem = mma::Smem<D>::kBytes;                                                                 \
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);        \
    if (e != cudaSuccess) return TSFA_ERR_CUDA;                                                            \
    kern<<<grid, block, smem, stream>>>(p);                                                                \
  } while (0)
  if (head_dim == 128 && dtype == TSFA_DTYPE_BF16) TSFA_LAUNCH(128, __nv_bfloat16);
  else if (head_dim == 128 && dtype == TSFA_DTYPE_F16) TSFA_LAUNCH(128, __half);
  else if (head_dim == 64 && dtype == TSFA_DTYPE_BF16) TSFA_LAUNCH(64, __nv_bfloat16);
  else if (head_dim == 64 && dtype == TSFA_DTYPE_F16) TSFA_LAUNCH(64, __half);
  else return TSFA_ERR_UNSUPPORTED;
#undef TSFA_LAUNCH
  return cudaGetLastError() == cudaSuccess ? TSFA_OK : TSFA_ERR_CUDA;
}

}  // namespace tsfa
