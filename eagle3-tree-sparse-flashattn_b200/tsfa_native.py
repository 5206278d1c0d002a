"""ctypes binding of libtsfa.so (the C ABI declared in include/tsfa.h), and
the loader of its PyTorch operators (libtsfa_torch.so: torch.ops.tsfa.*).

PyTorch supplies device memory and the current CUDA stream; every kernel is in
libtsfa.so.  There is no fallback: if a library is missing or no CUDA device
is visible, the calls raise.  The work buffer of every call is the operator
library's per-(device, stream) buffer (torch.ops.tsfa.workspace), so the
device status block read after a call through either binding is the one that
call wrote.
"""

from __future__ import annotations

import ctypes
import math
import os
import threading
import types

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("TSFA_LIB", os.path.join(_HERE, "libtsfa.so"))

TSFA_OK = 0
TSFA_ERR_VALUE = -1
TSFA_ERR_ASSERT = -2
TSFA_ERR_UNSUPPORTED = -3
TSFA_ERR_WORKSPACE = -4
TSFA_ERR_CUDA = -5
TSFA_ERR_DEVICE_TIMEOUT = -6
TSFA_ERR_DEVICE_BOUNDS = -7
SYNC_BYTES = 4096
FAULT_NONE = 0
FAULT_WITHHOLD_TREE_LIST = 1
FAULT_REFUSE_COOPERATIVE = 2  # TSFA_FAULT_REFUSE_COOPERATIVE
DEBUG_LIB_PATH = os.path.join(_HERE, "libtsfa_debug.so")
TORCH_OP_PATH = os.path.join(_HERE, "libtsfa_torch.so")

DTYPE_BF16 = 0
DTYPE_F16 = 1

MASK_DTYPES = {
    torch.bool: 0, torch.uint8: 0, torch.int8: 0,
    torch.int16: 1, torch.int32: 2, torch.int64: 3,
    torch.float16: 4, torch.bfloat16: 5, torch.float32: 6, torch.float64: 7,
}
QKV_DTYPES = {torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}

EXPORTS = (
    "tsfa_status_string", "tsfa_last_error", "tsfa_abi_version", "tsfa_meta_dims", "tsfa_meta_workspace_bytes",
    "tsfa_meta_build", "tsfa_pack_block_mask", "tsfa_fwd_workspace_bytes", "tsfa_fwd",
    "tsfa_run_workspace_bytes", "tsfa_run_tree_sparse", "tsfa_read_device_status",
    "tsfa_run_tree_sparse_noalloc", "tsfa_run_batched_workspace_bytes", "tsfa_run_tree_sparse_batched",
    "tsfa_run_tree_sparse_paged", "tsfa_run_paged_workspace_bytes", "tsfa_read_device_status_detail",
    "tsfa_noalloc_read_device_status", "tsfa_debug_inject", "tsfa_debug_last_plan", "tsfa_debug_force_merge",
)


class TsfaPagedKV(ctypes.Structure):
    _fields_ = [("k_pages", ctypes.c_void_p), ("v_pages", ctypes.c_void_p),
                ("k_stride", ctypes.c_int64 * 4), ("v_stride", ctypes.c_int64 * 4),
                ("num_pages", ctypes.c_int32), ("page_size", ctypes.c_int32),
                ("page_indptr", ctypes.c_void_p), ("page_indices", ctypes.c_void_p)]


class TsfaMetaDims(ctypes.Structure):
    _fields_ = [("n_q_blocks", ctypes.c_int64), ("n_tree_blocks", ctypes.c_int64),
                ("words_per_tile", ctypes.c_int64), ("tile_capacity", ctypes.c_int64),
                ("payload_capacity", ctypes.c_int64)]


class TsfaMeta(ctypes.Structure):
    _fields_ = [("row_ptr", ctypes.c_void_p), ("col_idx", ctypes.c_void_p), ("blk_type", ctypes.c_void_p),
                ("mixed_mask_payload", ctypes.c_void_p), ("mixed_mask_offset", ctypes.c_void_p),
                ("counts", ctypes.c_void_p)]


class TsfaFwdArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("o", ctypes.c_void_p),
        ("q_stride", ctypes.c_int64 * 4), ("k_stride", ctypes.c_int64 * 4),
        ("v_stride", ctypes.c_int64 * 4), ("o_stride", ctypes.c_int64 * 4),
        ("batch", ctypes.c_int32), ("num_heads", ctypes.c_int32), ("num_kv_heads", ctypes.c_int32),
        ("q_len", ctypes.c_int32), ("kv_len", ctypes.c_int32), ("prefix_len", ctypes.c_int32),
        ("head_dim", ctypes.c_int32), ("dtype", ctypes.c_int32), ("sm_scale", ctypes.c_float),
        ("row_ptr", ctypes.c_void_p), ("col_idx", ctypes.c_void_p), ("blk_type", ctypes.c_void_p),
        ("mixed_mask_payload", ctypes.c_void_p), ("mixed_mask_offset", ctypes.c_void_p),
        ("n_q_blocks", ctypes.c_int32), ("n_tree_blocks", ctypes.c_int32),
        ("block_m", ctypes.c_int32), ("block_n", ctypes.c_int32),
    ]


_lib = None
_lib_lock = threading.Lock()


def load_library(path: str | None = None) -> ctypes.CDLL:
    """Load libtsfa.so once (no GPU needed to load it)."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = path or LIB_PATH
        if not os.path.exists(p):
            raise RuntimeError(
                f"libtsfa.so not found at {p}: build it with "
                "`python eagle3-tree-sparse-flashattn_b200/csrc/build.py` (there is no CPU fallback)")
        lib = ctypes.CDLL(p)
        vp, i32, i64, sz = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t
        lib.tsfa_status_string.restype = ctypes.c_char_p
        lib.tsfa_status_string.argtypes = [ctypes.c_int]
        lib.tsfa_last_error.restype = ctypes.c_char_p
        lib.tsfa_last_error.argtypes = []
        lib.tsfa_abi_version.restype = ctypes.c_int
        lib.tsfa_meta_dims.argtypes = [i32, i32, i32, ctypes.POINTER(TsfaMetaDims)]
        lib.tsfa_meta_workspace_bytes.argtypes = [i32, i32, i32, ctypes.POINTER(sz)]
        lib.tsfa_meta_build.argtypes = [vp, i32, i64, i32, i32, i32, ctypes.POINTER(TsfaMeta), vp, sz, vp]
        lib.tsfa_pack_block_mask.argtypes = [vp, i32, i64, i32, i32, vp, vp]
        lib.tsfa_fwd_workspace_bytes.argtypes = [ctypes.POINTER(TsfaFwdArgs), ctypes.POINTER(sz)]
        lib.tsfa_fwd.argtypes = [ctypes.POINTER(TsfaFwdArgs), vp, sz, vp]
        lib.tsfa_run_workspace_bytes.argtypes = [ctypes.POINTER(TsfaFwdArgs), ctypes.POINTER(sz)]
        lib.tsfa_run_tree_sparse.argtypes = [ctypes.POINTER(TsfaFwdArgs), vp, i32, i64, vp, sz, vp]
        lib.tsfa_read_device_status.argtypes = [vp, vp, ctypes.POINTER(i32)]
        lib.tsfa_run_tree_sparse_noalloc.argtypes = [ctypes.POINTER(TsfaFwdArgs), vp, i32, i64, vp]
        lib.tsfa_run_batched_workspace_bytes.argtypes = [ctypes.POINTER(TsfaFwdArgs), ctypes.POINTER(sz)]
        lib.tsfa_run_tree_sparse_batched.argtypes = [ctypes.POINTER(TsfaFwdArgs), vp, i32, i64, i64, vp, sz, vp]
        lib.tsfa_run_paged_workspace_bytes.argtypes = [ctypes.POINTER(TsfaFwdArgs), ctypes.POINTER(sz)]
        lib.tsfa_run_tree_sparse_paged.argtypes = [ctypes.POINTER(TsfaFwdArgs), ctypes.POINTER(TsfaPagedKV), vp, i32,
                                                   i64, vp, sz, vp]
        lib.tsfa_read_device_status_detail.argtypes = [vp, vp, ctypes.POINTER(i32)]
        lib.tsfa_noalloc_read_device_status.argtypes = [vp, ctypes.POINTER(i32)]
        lib.tsfa_debug_inject.argtypes = [i32, ctypes.c_uint64]
        lib.tsfa_debug_last_plan.argtypes = [ctypes.POINTER(i32)]
        lib.tsfa_debug_force_merge.argtypes = [i32]
        for name in EXPORTS:
            if name not in ("tsfa_status_string", "tsfa_last_error"):
                getattr(lib, name).restype = ctypes.c_int
        if lib.tsfa_abi_version() != 1:
            raise RuntimeError("libtsfa.so ABI version mismatch")
        if path is None:
            _lib = lib
        return lib


_op_loaded = False


def load_torch_op():
    """Register torch.ops.tsfa.* (libtsfa_torch.so) once; returns torch.ops.tsfa."""
    global _op_loaded
    if _op_loaded:  # lock-free once loaded: torch.compile traces through this call
        return torch.ops.tsfa
    with _lib_lock:
        if not _op_loaded:
            if not os.path.exists(TORCH_OP_PATH):
                raise RuntimeError(f"libtsfa_torch.so not found at {TORCH_OP_PATH}: build it with "
                                   "`python eagle3-tree-sparse-flashattn_b200/csrc/build.py` (there is no fallback)")
            torch.ops.load_library(TORCH_OP_PATH)
            _op_loaded = True
    return torch.ops.tsfa


def status_text(status: int) -> str:
    return load_library().tsfa_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Map a libtsfa status to the reference's exception types."""
    if status == TSFA_OK:
        return
    msg = f"{what}: {status_text(status)} (status {status})"
    if status == TSFA_ERR_CUDA:
        msg += f" [{load_library().tsfa_last_error().decode()}]"
    if status == TSFA_ERR_VALUE:
        raise ValueError(msg)
    if status == TSFA_ERR_ASSERT:
        raise AssertionError(msg)
    if status == TSFA_ERR_UNSUPPORTED:
        raise NotImplementedError(msg)
    raise RuntimeError(msg)


def require_cuda(device: torch.device | None = None) -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("tree-sparse attention runs on CUDA (sm_100a) only; no CUDA device is visible")
    load_library()
    if device is None or device.type != "cuda":
        return torch.device("cuda", torch.cuda.current_device())
    return device


def stream_ptr(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


# ----------------------------------------------------------------- workspaces
def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """The per-(device, current stream) work buffer, at least `nbytes` long;
    its first SYNC_BYTES were zeroed when it was allocated (the kernels leave
    their arrival counters at zero).  Shared with torch.ops.tsfa.*."""
    return load_torch_op().workspace(device, int(nbytes))


# ----------------------------------------------------------------- helpers
def mask_dtype_code(t: torch.Tensor) -> int:
    code = MASK_DTYPES.get(t.dtype)
    if code is None:
        raise TypeError(f"unsupported tree_mask dtype {t.dtype}")
    return code


def qkv_dtype_code(t: torch.Tensor) -> int:
    code = QKV_DTYPES.get(t.dtype)
    if code is None:
        raise TypeError(f"query/key/value must be bfloat16 or float16, got {t.dtype}")
    return code


def fwd_args(q, k, v, o, *, prefix_len: int, sm_scale: float | None = None, meta=None,
             block_m: int = 64, block_n: int = 64) -> TsfaFwdArgs:
    B, Hq, T, D = q.shape
    Hkv, kv_len = k.shape[1], k.shape[2]
    a = TsfaFwdArgs()
    a.q, a.k, a.v, a.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    a.q_stride[:] = q.stride()
    a.k_stride[:] = k.stride()
    a.v_stride[:] = v.stride()
    a.o_stride[:] = o.stride()
    a.batch, a.num_heads, a.num_kv_heads = B, Hq, Hkv
    a.q_len, a.kv_len, a.prefix_len, a.head_dim = T, kv_len, prefix_len, D
    a.dtype = qkv_dtype_code(q)
    a.sm_scale = (1.0 / math.sqrt(D)) if sm_scale is None else float(sm_scale)
    a.block_m, a.block_n = block_m, block_n
    if meta is not None:
        a.row_ptr = meta.row_ptr.data_ptr()
        a.col_idx = meta.col_idx.data_ptr()
        a.blk_type = meta.blk_type.data_ptr()
        a.mixed_mask_payload = meta.mixed_mask_payload.data_ptr() if meta.mixed_mask_payload.numel() else None
        a.mixed_mask_offset = meta.mixed_mask_offset.data_ptr() if meta.mixed_mask_offset.numel() else None
        a.n_q_blocks, a.n_tree_blocks = meta.n_q_blocks, meta.n_tree_blocks
        a.block_m, a.block_n = meta.block_m, meta.block_n
    return a


def meta_dims(q_len: int, block_m: int, block_n: int) -> TsfaMetaDims:
    d = TsfaMetaDims()
    check(load_library().tsfa_meta_dims(q_len, block_m, block_n, ctypes.byref(d)), "tsfa_meta_dims")
    return d


def build_metadata_device(mask: torch.Tensor, block_m: int, block_n: int):
    """K1 on `mask`'s device.  Returns capacity-sized buffers and (nnz, n_mixed)
    read back with one device->host copy."""
    lib = load_library()
    dev = mask.device
    T = mask.shape[0]
    d = meta_dims(T, block_m, block_n)
    cap, pcap = int(d.tile_capacity), int(d.payload_capacity)
    row_ptr = torch.empty(int(d.n_q_blocks) + 1, dtype=torch.int32, device=dev)
    col_idx = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    blk_type = torch.empty(max(cap, 1), dtype=torch.int8, device=dev)
    payload = torch.empty(max(pcap, 1), dtype=torch.int32, device=dev)
    offset = torch.empty(max(cap, 1), dtype=torch.int32, device=dev)
    counts = torch.empty(2, dtype=torch.int32, device=dev)
    m = TsfaMeta(row_ptr.data_ptr(), col_idx.data_ptr(), blk_type.data_ptr(), payload.data_ptr(),
                 offset.data_ptr(), counts.data_ptr())
    nbytes = ctypes.c_size_t()
    check(lib.tsfa_meta_workspace_bytes(T, block_m, block_n, ctypes.byref(nbytes)), "tsfa_meta_workspace_bytes")
    ws = workspace(nbytes.value, dev)
    if mask.numel() and mask.stride(1) != 1:
        mask = mask.contiguous()
    stride = mask.stride(0) if mask.numel() else T
    check(lib.tsfa_meta_build(mask.data_ptr() if mask.numel() else None, mask_dtype_code(mask), stride, T,
                              block_m, block_n, ctypes.byref(m), ws.data_ptr(), ws.numel(), stream_ptr(dev)),
          "tsfa_meta_build")
    nnz, n_mixed = (int(x) for x in counts.tolist())
    return d, row_ptr, col_idx, blk_type, payload, offset, nnz, n_mixed


def pack_tile_device(tile: torch.Tensor) -> torch.Tensor:
    lib = load_library()
    dev = tile.device
    if tile.dim() != 2:
        tile = tile.reshape(1, -1)
    rows, cols = tile.shape
    if tile.numel() and tile.stride(1) != 1:
        tile = tile.contiguous()
    words = (rows * cols + 31) // 32
    out = torch.empty(words, dtype=torch.int32, device=dev)
    if words:
        check(lib.tsfa_pack_block_mask(tile.data_ptr(), mask_dtype_code(tile), tile.stride(0), rows, cols,
                                       out.data_ptr(), stream_ptr(dev)), "tsfa_pack_block_mask")
    return out


def run_tree_sparse(q, k, v, mask, out, *, prefix_len: int, block_m: int, block_n: int,
                    sm_scale: float | None = None) -> torch.Tensor:
    """Metadata build + forward in one native call (tsfa_run_tree_sparse)."""
    lib = load_library()
    a = fwd_args(q, k, v, out, prefix_len=prefix_len, sm_scale=sm_scale, block_m=block_m, block_n=block_n)
    nbytes = ctypes.c_size_t()
    check(lib.tsfa_run_workspace_bytes(ctypes.byref(a), ctypes.byref(nbytes)), "tsfa_run_workspace_bytes")
    ws = workspace(nbytes.value, q.device)
    if mask.numel() and mask.stride(1) != 1:
        mask = mask.contiguous()
    T = q.shape[2]
    stride = mask.stride(0) if mask.numel() else T
    check(lib.tsfa_run_tree_sparse(ctypes.byref(a), mask.data_ptr() if mask.numel() else None,
                                   mask_dtype_code(mask), stride, ws.data_ptr(), ws.numel(),
                                   stream_ptr(q.device)), "tsfa_run_tree_sparse")
    return out


def run_tree_sparse_batched(q, k, v, masks, out, *, prefix_len: int, block_m: int, block_n: int,
                            sm_scale: float | None = None) -> torch.Tensor:
    """Metadata build + forward with masks[b] ([B, T, T]) applied to batch
    element b, in one native call (tsfa_run_tree_sparse_batched)."""
    lib = load_library()
    a = fwd_args(q, k, v, out, prefix_len=prefix_len, sm_scale=sm_scale, block_m=block_m, block_n=block_n)
    nbytes = ctypes.c_size_t()
    check(lib.tsfa_run_batched_workspace_bytes(ctypes.byref(a), ctypes.byref(nbytes)),
          "tsfa_run_batched_workspace_bytes")
    ws = workspace(nbytes.value, q.device)
    if masks.numel() and masks.stride(2) != 1:
        masks = masks.contiguous()
    T = q.shape[2]
    bstride, rstride = (masks.stride(0), masks.stride(1)) if masks.numel() else (T * T, T)
    check(lib.tsfa_run_tree_sparse_batched(ctypes.byref(a), masks.data_ptr() if masks.numel() else None,
                                           mask_dtype_code(masks), bstride, rstride, ws.data_ptr(), ws.numel(),
                                           stream_ptr(q.device)), "tsfa_run_tree_sparse_batched")
    return out


def paged_kv(k_pages, v_pages, page_indptr, page_indices) -> TsfaPagedKV:
    kv = TsfaPagedKV()
    kv.k_pages, kv.v_pages = k_pages.data_ptr(), v_pages.data_ptr()
    kv.k_stride[:] = k_pages.stride()
    kv.v_stride[:] = v_pages.stride()
    kv.num_pages, kv.page_size = k_pages.shape[0], k_pages.shape[1]
    kv.page_indptr, kv.page_indices = page_indptr.data_ptr(), page_indices.data_ptr()
    return kv


def run_tree_sparse_paged(q, k_pages, v_pages, page_indptr, page_indices, mask, out, *, kv_len: int,
                          prefix_len: int, block_m: int, block_n: int, sm_scale: float | None = None) -> torch.Tensor:
    """Metadata build + forward over a paged K/V cache (tsfa_run_tree_sparse_paged):
    pools [num_pages, page_size, Hkv, D], page table page_indptr [B + 1] /
    page_indices (int32, on the device)."""
    lib = load_library()
    B, _, _, D = q.shape
    Hkv = k_pages.shape[2]
    # the dense K/V arguments only carry the shapes: K/V come from the pools
    shape_kv = types.SimpleNamespace(shape=(B, Hkv, kv_len, D), stride=lambda: (0, 0, 0, 1), data_ptr=lambda: 0)
    a = fwd_args(q, shape_kv, shape_kv, out, prefix_len=prefix_len, sm_scale=sm_scale, block_m=block_m,
                 block_n=block_n)
    kv = paged_kv(k_pages, v_pages, page_indptr, page_indices)
    nbytes = ctypes.c_size_t()
    check(lib.tsfa_run_paged_workspace_bytes(ctypes.byref(a), ctypes.byref(nbytes)), "tsfa_run_paged_workspace_bytes")
    ws = workspace(nbytes.value, q.device)
    if mask.numel() and mask.stride(1) != 1:
        mask = mask.contiguous()
    T = q.shape[2]
    stride = mask.stride(0) if mask.numel() else T
    check(lib.tsfa_run_tree_sparse_paged(ctypes.byref(a), ctypes.byref(kv), mask.data_ptr() if mask.numel() else None,
                                         mask_dtype_code(mask), stride, ws.data_ptr(), ws.numel(),
                                         stream_ptr(q.device)), "tsfa_run_tree_sparse_paged")
    return out


NOALLOC_WORKSPACE_BYTES = 8 << 20  # TSFA_NOALLOC_WORKSPACE_BYTES


def run_tree_sparse_noalloc(q, k, v, mask, out, *, prefix_len: int, block_m: int, block_n: int,
                            sm_scale: float | None = None) -> torch.Tensor:
    """tsfa_run_tree_sparse_noalloc: the whole op over the library's static
    workspace (no allocation).  Calls that overlap in time race; the first
    call on a device does set-up and should come before any stream capture."""
    lib = load_library()
    a = fwd_args(q, k, v, out, prefix_len=prefix_len, sm_scale=sm_scale, block_m=block_m, block_n=block_n)
    if mask.numel() and mask.stride(1) != 1:
        mask = mask.contiguous()
    T = q.shape[2]
    stride = mask.stride(0) if mask.numel() else T
    st = lib.tsfa_run_tree_sparse_noalloc(ctypes.byref(a), mask.data_ptr() if mask.numel() else None,
                                          mask_dtype_code(mask), stride, stream_ptr(q.device))
    if st == TSFA_ERR_WORKSPACE:
        raise ValueError(f"tsfa_run_tree_sparse_noalloc: q_len {T} with {block_m}x{block_n} blocks needs more "
                         f"workspace than the static workspace holds ({NOALLOC_WORKSPACE_BYTES} bytes); "
                         "use run_tree_sparse")
    check(st, "tsfa_run_tree_sparse_noalloc")
    return out


def launch_fwd_args(a: TsfaFwdArgs, device: torch.device) -> None:
    """tsfa_fwd on a filled argument block, with this stream's workspace."""
    lib = load_library()
    nbytes = ctypes.c_size_t()
    check(lib.tsfa_fwd_workspace_bytes(ctypes.byref(a), ctypes.byref(nbytes)), "tsfa_fwd_workspace_bytes")
    ws = workspace(nbytes.value, device)
    check(lib.tsfa_fwd(ctypes.byref(a), ws.data_ptr(), ws.numel(), stream_ptr(device)), "tsfa_fwd")


def fwd_with_metadata(q, k, v, out, meta, *, prefix_len: int, sm_scale: float | None = None) -> torch.Tensor:
    """Forward over prebuilt device metadata (tsfa_fwd)."""
    launch_fwd_args(fwd_args(q, k, v, out, prefix_len=prefix_len, sm_scale=sm_scale, meta=meta), q.device)
    return out


def read_device_status(device: torch.device) -> int:
    """Device status word of this stream's workspace (synchronises)."""
    return read_device_status_detail(device)[0]


def read_device_status_detail(device: torch.device) -> tuple:
    """(status, site or bounds check, key tile or index, CTA) of this stream's
    workspace (synchronises; clears the sync block after an error)."""
    lib = load_library()
    ws = workspace(SYNC_BYTES, device)
    d = (ctypes.c_int32 * 4)()
    check(lib.tsfa_read_device_status_detail(ws.data_ptr(), stream_ptr(device), d),
          "tsfa_read_device_status_detail")
    return tuple(int(x) for x in d)


def noalloc_read_device_status(device: torch.device) -> tuple:
    """tsfa_noalloc_read_device_status: the same detail for the static
    workspace of run_tree_sparse_noalloc (synchronises)."""
    lib = load_library()
    d = (ctypes.c_int32 * 4)()
    check(lib.tsfa_noalloc_read_device_status(stream_ptr(device), d), "tsfa_noalloc_read_device_status")
    return tuple(int(x) for x in d)


def last_plan() -> dict:
    """The calling thread's last forward launch (tsfa_debug_last_plan)."""
    d = (ctypes.c_int32 * 4)()
    check(load_library().tsfa_debug_last_plan(d), "tsfa_debug_last_plan")
    return {"splits": d[0], "merge": ("none", "cluster", "global", "pair")[d[1]], "grid": (d[2], d[3])}


def force_cluster_merge(on: bool) -> None:
    """For measurement: this thread's later forwards merge through clusters
    (the per-batch op's plan), also the whole op and tsfa_fwd over prebuilt
    metadata (tsfa_debug_force_merge)."""
    check(load_library().tsfa_debug_force_merge(1 if on else 0), "tsfa_debug_force_merge")


def force_row_pairs(on: bool) -> None:
    """For tests: this thread's later forwards run one split with row-tile
    pairs wherever the shapes allow it (tsfa_debug_force_merge mode 3)."""
    check(load_library().tsfa_debug_force_merge(3 if on else 0), "tsfa_debug_force_merge")


def debug_inject(fault: int = FAULT_NONE, wait_limit_ns: int = 0) -> None:
    """Tests only: the wait limit and injected fault of this thread's later
    launches (tsfa_debug_inject); debug_inject() restores the defaults."""
    check(load_library().tsfa_debug_inject(int(fault), int(wait_limit_ns)), "tsfa_debug_inject")
