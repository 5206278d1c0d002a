/*
 * tsfa.h -- C ABI of libtsfa.so: tree-sparse attention forward for B200 (sm_100a).
 *
 * The verify step of tree speculative decoding: T draft-tree tokens attend to a
 * dense prefix of P keys and to their own ancestors under tree_mask[T, T].  The
 * tree part is described by the reference's block-CSR metadata
 * (row_ptr / col_idx / blk_type / mixed_mask_payload / mixed_mask_offset, the
 * layout of tree_sparse_flashattn.py:15-41 and README.md:116-133).
 *
 * Conventions
 *   - Every entry point returns an int status: TSFA_OK (0) or a negative code.
 *   - All tensor arguments are device pointers with element strides; the
 *     library never allocates device memory.  Work buffers ("workspace") are
 *     passed in by the caller; their first TSFA_SYNC_BYTES bytes hold
 *     arrival counters that must be zero before the first call on that buffer
 *     (cudaMemset once) -- every kernel leaves them at zero again.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream).  Kernels are
 *     enqueued asynchronously; calls on one workspace must not overlap in time.
 *   - No torch (or other framework) types cross this boundary.
 */
#ifndef TSFA_H_
#define TSFA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TSFA_ABI_VERSION 1

#if defined(__GNUC__)
#define TSFA_API __attribute__((visibility("default")))
#else
#define TSFA_API
#endif

/* Block-type codes stored in blk_type (tree_sparse_flashattn.py:11-12).
 * ZERO tiles are not stored in the CSR. */
#define TSFA_FULL_BLOCK 0
#define TSFA_MIXED_BLOCK 1

/* Bytes at the start of every workspace reserved for arrival counters. */
#define TSFA_SYNC_BYTES 4096

/* Status codes (the Python layer maps them to the reference's exceptions). */
enum {
  TSFA_OK = 0,
  TSFA_ERR_VALUE = -1,         /* ValueError: bad mask shape / block size (tsfa.py:85-88),
                                  kv_len < q_len (bridge.py:91-93) */
  TSFA_ERR_ASSERT = -2,        /* AssertionError: shape mismatch (bridge.py:85-89) */
  TSFA_ERR_UNSUPPORTED = -3,   /* head_dim / dtype / stride layout this build does not handle */
  TSFA_ERR_WORKSPACE = -4,     /* workspace NULL or smaller than the *_workspace_bytes answer */
  TSFA_ERR_CUDA = -5,          /* a CUDA runtime call or kernel launch failed */
  TSFA_ERR_DEVICE_TIMEOUT = -6, /* a bounded device-side wait gave up (see tsfa_read_device_status) */
  TSFA_ERR_DEVICE_BOUNDS = -7   /* debug builds only: a metadata index failed its bounds check on the
                                   device (see tsfa_read_device_status_detail); the tile was skipped */
};

/* Element type of the tree mask.  A mask element is visible iff it is nonzero
 * (NaN is visible, -0.0 is not): the semantics of Tensor.to(torch.bool)
 * used by tsfa.py:90 and bridge.py:96. */
enum {
  TSFA_MASK_B8 = 0, /* bool / uint8 / int8 */
  TSFA_MASK_I16 = 1,
  TSFA_MASK_I32 = 2,
  TSFA_MASK_I64 = 3,
  TSFA_MASK_F16 = 4,
  TSFA_MASK_BF16 = 5,
  TSFA_MASK_F32 = 6,
  TSFA_MASK_F64 = 7
};

/* Element type of Q / K / V / O. */
enum { TSFA_DTYPE_BF16 = 0, TSFA_DTYPE_F16 = 1 };

/* Faults tsfa_debug_inject can ask the next launches for (tests only). */
#define TSFA_FAULT_NONE 0
#define TSFA_FAULT_WITHHOLD_TREE_LIST 1 /* the forward's tree-list warp never publishes its list */
#define TSFA_FAULT_REFUSE_COOPERATIVE 2 /* the host treats a cooperative forward launch as refused */

TSFA_API const char* tsfa_status_string(int status);
/* Text of the last failing CUDA runtime call made by this library on the
 * calling thread ("" if none), for messages accompanying TSFA_ERR_CUDA. */
TSFA_API const char* tsfa_last_error(void);
TSFA_API int tsfa_abi_version(void);

/* ------------------------------------------------------------------------- */
/* Metadata (replaces prepare_tree_sparse_metadata, tree_sparse_flashattn.py:67-160,
 * and _pack_block_mask_to_int32, tree_sparse_flashattn.py:44-64).             */
/* ------------------------------------------------------------------------- */

typedef struct TsfaMetaDims {
  int64_t n_q_blocks;       /* cdiv(q_len, block_m)               (tsfa.py:92) */
  int64_t n_tree_blocks;    /* cdiv(q_len, block_n)               (tsfa.py:93) */
  int64_t words_per_tile;   /* W = cdiv(block_m * block_n, 32)    (tsfa.py:53) */
  int64_t tile_capacity;    /* n_q_blocks * n_tree_blocks: upper bound of nnz */
  int64_t payload_capacity; /* tile_capacity * W: upper bound of the payload  */
} TsfaMetaDims;

/* Device buffers of one metadata set.  col_idx / blk_type / mixed_mask_offset
 * hold tile_capacity entries, mixed_mask_payload payload_capacity words; after
 * tsfa_meta_build the first nnz (resp. n_mixed * W) entries are the
 * reference's tensors, in the reference's order.  counts = {nnz, n_mixed}. */
typedef struct TsfaMeta {
  int32_t* row_ptr;            /* [n_q_blocks + 1] */
  int32_t* col_idx;            /* [tile_capacity] */
  int8_t* blk_type;            /* [tile_capacity] */
  int32_t* mixed_mask_payload; /* [payload_capacity] */
  int32_t* mixed_mask_offset;  /* [tile_capacity] */
  int32_t* counts;             /* [2] */
} TsfaMeta;

/* Shapes of the metadata for a [q_len, q_len] mask.  TSFA_ERR_VALUE if a block
 * size is not positive (tsfa.py:87-88) or q_len < 0. */
TSFA_API int tsfa_meta_dims(int32_t q_len, int32_t block_m, int32_t block_n, TsfaMetaDims* out);

/* Workspace bytes needed by tsfa_meta_build. */
TSFA_API int tsfa_meta_workspace_bytes(int32_t q_len, int32_t block_m, int32_t block_n, size_t* bytes);

/* Build the metadata on the device from a [q_len, q_len] mask with unit column
 * stride and `mask_row_stride` elements between rows.  One launch; no host
 * synchronisation.  Bit-exact with tsfa.py:67-160 (classification on the clipped
 * edge region, zero-padded bitsets, int32 words with bit 31 as the sign). */
TSFA_API int tsfa_meta_build(const void* tree_mask, int32_t mask_dtype, int64_t mask_row_stride,
                    int32_t q_len, int32_t block_m, int32_t block_n, const TsfaMeta* out,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Pack one [rows, cols] mask tile into cdiv(rows * cols, 32) int32 words,
 * row-major, bit i % 32 of word i / 32 = flat[i] (replaces
 * _pack_block_mask_to_int32, tree_sparse_flashattn.py:44-64). */
TSFA_API int tsfa_pack_block_mask(const void* tile, int32_t mask_dtype, int64_t row_stride, int32_t rows, int32_t cols,
                         int32_t* out_words, void* stream);

/* ------------------------------------------------------------------------- */
/* Forward (replaces block_sparse_tree_fwd_kernel, tree_sparse_flashattn.py:163-339,
 * launched as in eagle_tree_sparse_bridge.py:108-158).                        */
/* ------------------------------------------------------------------------- */

typedef struct TsfaFwdArgs {
  const void* q; /* [B, Hq,  q_len,  D] */
  const void* k; /* [B, Hkv, kv_len, D] */
  const void* v; /* [B, Hkv, kv_len, D] */
  void* o;       /* [B, Hq,  q_len,  D], written in `dtype` */
  int64_t q_stride[4]; /* element strides for (b, h, n, d); stride[3] must be 1 */
  int64_t k_stride[4];
  int64_t v_stride[4];
  int64_t o_stride[4];
  int32_t batch, num_heads, num_kv_heads, q_len, kv_len, prefix_len, head_dim;
  int32_t dtype;  /* TSFA_DTYPE_* */
  float sm_scale; /* 1/sqrt(head_dim) in the reference (bridge.py:116) */
  /* metadata, device pointers with the reference's layout */
  const int32_t* row_ptr;
  const int32_t* col_idx;
  const int8_t* blk_type;
  const int32_t* mixed_mask_payload;
  const int32_t* mixed_mask_offset;
  int32_t n_q_blocks, n_tree_blocks, block_m, block_n;
} TsfaFwdArgs;

/* Workspace bytes needed by tsfa_fwd for these shapes (split-KV partials,
 * arrival counters). */
TSFA_API int tsfa_fwd_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes);

/* Prefix sweep + CSR tree walk + normalise, for every (b, q-head, tree row). */
TSFA_API int tsfa_fwd(const TsfaFwdArgs* args, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* Whole op (replaces run_tree_sparse_kernel, eagle_tree_sparse_bridge.py:76-159):
 * metadata build from the mask + forward, on one stream, no host sync.        */
/* ------------------------------------------------------------------------- */

/* Workspace bytes for tsfa_run_tree_sparse: metadata buffers + both kernels'
 * work areas. */
TSFA_API int tsfa_run_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes);

/* args->row_ptr ... args->mixed_mask_offset and n_q_blocks / n_tree_blocks
 * are ignored and taken from the metadata built in the workspace;
 * args->block_m / block_n select the tile size (bridge.py:95-100). */
TSFA_API int tsfa_run_tree_sparse(const TsfaFwdArgs* args, const void* tree_mask, int32_t mask_dtype,
                         int64_t mask_row_stride, void* workspace, size_t workspace_bytes,
                         void* stream);

/* ------------------------------------------------------------------------- */
/* Whole op with one tree per batch element.  No reference counterpart: the
 * reference applies batch 0's tree to every batch element
 * (eagle_tree_sparse_bridge.py:57-58), while the draft trees of a batch of
 * EAGLE requests differ.                                                     */
/* ------------------------------------------------------------------------- */

/* Workspace bytes for tsfa_run_tree_sparse_batched: args->batch metadata
 * sets at fixed capacity + both kernels' work areas. */
TSFA_API int tsfa_run_batched_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes);

/* tsfa_run_tree_sparse with tree_masks[b] -- the [q_len, q_len] mask at
 * tree_masks + b * mask_batch_stride elements, rows mask_row_stride apart --
 * applied to batch element b.  Metadata build (one set per batch element)
 * + forward on one stream, no host sync.  mask_batch_stride may be 0 (one
 * mask read for every element); TSFA_ERR_VALUE if it is negative. */
TSFA_API int tsfa_run_tree_sparse_batched(const TsfaFwdArgs* args, const void* tree_masks, int32_t mask_dtype,
                                          int64_t mask_batch_stride, int64_t mask_row_stride, void* workspace,
                                          size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* Whole op over a paged K/V cache.  No reference counterpart: the reference
 * takes contiguous K/V and concatenates the cache into them every step
 * (eagle_tree_sparse_bridge.py:235-236, 365-366); serving systems keep the
 * cache in pages (FlashInfer's [pages][2][page_size][heads][dim], used by
 * benchmark.py:67-91, or separate K and V pools).                            */
/* ------------------------------------------------------------------------- */

/* K and V page pools and the page table.  Key n (0 <= n < kv_len) of batch
 * element b is token n % page_size of page
 * page_indices[page_indptr[b] + n / page_size]. */
typedef struct TsfaPagedKV {
  const void* k_pages;         /* [num_pages][page_size][num_kv_heads][head_dim] */
  const void* v_pages;         /* same shape as k_pages */
  int64_t k_stride[4];         /* element strides for (page, token, head, dim); stride[3] must be 1 */
  int64_t v_stride[4];
  int32_t num_pages;           /* pages in each pool (>= 1) */
  int32_t page_size;           /* a power of two >= 8 */
  const int32_t* page_indptr;  /* device [batch + 1], non-decreasing */
  const int32_t* page_indices; /* device page ids, batch element after batch element */
} TsfaPagedKV;

/* Workspace bytes for tsfa_run_tree_sparse_paged: tsfa_run_workspace_bytes
 * plus the tree keys' K and V gathered from the pages
 * (2 * batch * num_kv_heads * q_len * head_dim * 2 bytes). */
TSFA_API int tsfa_run_paged_workspace_bytes(const TsfaFwdArgs* args, size_t* bytes);

/* tsfa_run_tree_sparse with K/V read from `kv` instead of args->k / args->v
 * (ignored, as are their strides); args->kv_len keys per batch element.
 * Prefix tiles are read from the pages directly; the metadata kernel also
 * gathers the q_len tree keys into the workspace, because the tree starts
 * at key prefix_len, which need not be a page boundary.  Page slots past
 * kv_len may hold any values; a page list shorter than
 * cdiv(kv_len, page_size), or a page id outside the pool, reads zeros for
 * those keys. */
TSFA_API int tsfa_run_tree_sparse_paged(const TsfaFwdArgs* args, const TsfaPagedKV* kv, const void* tree_mask,
                                        int32_t mask_dtype, int64_t mask_row_stride, void* workspace,
                                        size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------- */
/* Whole op without any allocation.  No reference counterpart: the reference
 * allocates its metadata with torch on every call (tsfa.py:122-160).         */
/* ------------------------------------------------------------------------- */

/* Size of the library-owned workspace behind tsfa_run_tree_sparse_noalloc:
 * 8 MiB of static device memory per device -- the split-KV partial rows of
 * one launch (at most 148 x 128 rows of 2 head_dim + 16 bytes: 5.2 MB) plus
 * the metadata of q_len <= 2048 at block sizes >= 16
 * (tsfa_run_workspace_bytes gives the need of a given shape). */
#define TSFA_NOALLOC_WORKSPACE_BYTES (8u << 20)

/* tsfa_run_tree_sparse over a workspace that lives in a static __device__
 * array of this library, for callers that cannot allocate device memory (a
 * plain C / FFI host without a device allocator, or a step loop where a
 * cudaMalloc would synchronise the device).  Neither this call nor the
 * library allocates anything.
 *   - Every call looks up the array's address on the current device
 *     (cudaGetSymbolAddress; no allocation).  The first call that sees an
 *     address on a device -- the first call there, or the first after the
 *     module was loaded into a new context -- also clears its
 *     TSFA_SYNC_BYTES sync block on `stream` (a memset): make that first call
 *     before any stream capture.
 *   - TSFA_ERR_WORKSPACE if the shapes need more than
 *     TSFA_NOALLOC_WORKSPACE_BYTES; nothing is launched then.
 *   - All calls on one device share the array: calls that overlap in time
 *     (other streams, other threads) race.  Order them on one stream.
 *   - The device status word of this workspace is read (and cleared after an
 *     error) with tsfa_noalloc_read_device_status. */
TSFA_API int tsfa_run_tree_sparse_noalloc(const TsfaFwdArgs* args, const void* tree_mask, int32_t mask_dtype,
                                          int64_t mask_row_stride, void* stream);

/* Reads the device status word of a workspace written by tsfa_fwd /
 * tsfa_run_tree_sparse: TSFA_OK, or TSFA_ERR_DEVICE_TIMEOUT if a bounded wait
 * inside a kernel gave up (TSFA_ERR_DEVICE_BOUNDS: a debug build's metadata
 * check failed) -- in which case the whole TSFA_SYNC_BYTES block is cleared,
 * so the workspace can be used again.  Synchronises `stream`.  No reference
 * counterpart: the Triton kernel has no device-side error path. */
TSFA_API int tsfa_read_device_status(void* workspace, void* stream, int32_t* device_status);

/* tsfa_read_device_status with where the error arose: detail[0] = the status,
 * detail[1] = the wait site (1..14) or bounds check (101..105), detail[2] =
 * the key tile (or metadata index), detail[3] = the CTA's linear index. */
TSFA_API int tsfa_read_device_status_detail(void* workspace, void* stream, int32_t detail[4]);

/* tsfa_read_device_status_detail on the static workspace behind
 * tsfa_run_tree_sparse_noalloc (current device); clears it after an error. */
TSFA_API int tsfa_noalloc_read_device_status(void* stream, int32_t detail[4]);

/* Tests only: launches made afterwards by the calling thread use
 * `wait_limit_ns` as the limit of every bounded device wait (0 = the default,
 * 1 s) and inject `fault` (TSFA_FAULT_*).  With TSFA_FAULT_WITHHOLD_TREE_LIST
 * and a short limit the forward's waits on the tree list run out: the kernel
 * winds down, leaves TSFA_ERR_DEVICE_TIMEOUT in the workspace status block
 * and the context stays usable.  With TSFA_FAULT_REFUSE_COOPERATIVE the host
 * side treats every cooperative (global-merge) forward launch as refused by
 * the device, before launching anything, so the fallback to the cluster
 * merge runs.  TSFA_ERR_VALUE for an unknown fault.  No reference
 * counterpart. */
TSFA_API int tsfa_debug_inject(int32_t fault, uint64_t wait_limit_ns);

/* The plan of the calling thread's last forward launch: plan[0] = splits per
 * row tile, plan[1] = how the splits' partial rows were merged (0 none, 1
 * thread-block cluster, 2 global through L2; 3: one split, row-tile pairs),
 * plan[2] / plan[3] = grid x / y.
 * For tests and tuning; no reference counterpart. */
TSFA_API int tsfa_debug_last_plan(int32_t plan[4]);

/* For measurement and tests: mode 1 makes the calling thread's later forward
 * launches merge their splits through thread-block clusters (the per-batch
 * op's plan), also in tsfa_fwd and the whole op; mode 3 makes them run one
 * split with row-tile pairs (one CTA per two row tiles, sharing every K/V
 * tile: the plan of shapes whose pairs fill the GPU) wherever the shapes
 * have two row tiles and contiguous K/V; mode 0 restores the library's
 * choice.  TSFA_ERR_VALUE for other modes.  No reference counterpart. */
TSFA_API int tsfa_debug_force_merge(int32_t mode);

#ifdef __cplusplus
}
#endif
#endif /* TSFA_H_ */
