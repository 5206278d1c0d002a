"""The C ABI: libtsfa.so loads without a GPU, exports every symbol the header
declares, and rejects bad arguments on the host before any CUDA call."""

import ctypes
import os
import re

import pytest

from conftest import REPO

import tsfa_native as nat

HEADER = os.path.join(REPO, "include", "tsfa.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"TSFA_API\s+(?:const\s+)?\w+\s*\*?\s*(tsfa_\w+)\s*\(", text)))


def test_header_declares_the_api():
    syms = declared_symbols()
    assert set(syms) == set(nat.EXPORTS), syms


def test_library_exports_every_declared_symbol():
    lib = nat.load_library()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    nm = os.popen(f"nm -D --defined-only {nat.LIB_PATH}").read()
    exported = set(re.findall(r" T (tsfa_\w+)", nm))
    assert exported == set(declared_symbols()), exported ^ set(declared_symbols())


def test_status_strings_and_version():
    lib = nat.load_library()
    assert lib.tsfa_abi_version() == 1
    for code in range(-7, 1):
        assert nat.status_text(code) != "unknown status"
    assert nat.status_text(-99) == "unknown status"


def test_debug_inject_checks_its_fault_code():
    """The test-only fault switch is host state: no GPU is needed to set it."""
    lib = nat.load_library()
    assert lib.tsfa_debug_inject(7, 1000) == nat.TSFA_ERR_VALUE
    assert lib.tsfa_debug_inject(nat.FAULT_WITHHOLD_TREE_LIST, 1000) == nat.TSFA_OK
    assert lib.tsfa_debug_inject(nat.FAULT_NONE, 0) == nat.TSFA_OK


def test_debug_library_exports_the_same_symbols():
    """libtsfa_debug.so (device-side bounds checks) is a drop-in for libtsfa.so."""
    if not os.path.exists(nat.DEBUG_LIB_PATH):
        pytest.skip("debug library not built")
    nm = os.popen(f"nm -D --defined-only {nat.DEBUG_LIB_PATH}").read()
    assert set(re.findall(r" T (tsfa_\w+)", nm)) == set(declared_symbols())


@pytest.mark.parametrize("T,bm,bn", [(64, 64, 64), (100, 16, 32), (0, 16, 16), (1024, 16, 16), (13, 3, 5)])
def test_meta_dims(T, bm, bn):
    d = nat.meta_dims(T, bm, bn)
    assert d.n_q_blocks == -(-T // bm) and d.n_tree_blocks == -(-T // bn)
    assert d.words_per_tile == -(-(bm * bn) // 32)
    assert d.tile_capacity == d.n_q_blocks * d.n_tree_blocks
    assert d.payload_capacity == d.tile_capacity * d.words_per_tile


@pytest.mark.parametrize("bm,bn", [(0, 16), (16, 0), (-1, 4)])
def test_meta_dims_rejects_bad_blocks(bm, bn):
    with pytest.raises(ValueError):
        nat.meta_dims(64, bm, bn)


def _args(**kw):
    a = nat.TsfaFwdArgs()
    a.q = a.k = a.v = a.o = 4096  # never dereferenced: the checks run first
    B, Hq, Hkv, T, P, D = kw.get("B", 1), kw.get("Hq", 32), kw.get("Hkv", 8), kw.get("T", 64), kw.get("P", 4096), kw.get("D", 128)
    kv = P + T
    a.q_stride[:] = (Hq * T * D, T * D, D, 1)
    a.k_stride[:] = (Hkv * kv * D, kv * D, D, 1)
    a.v_stride[:] = a.k_stride[:]
    a.o_stride[:] = a.q_stride[:]
    a.batch, a.num_heads, a.num_kv_heads, a.q_len, a.kv_len, a.prefix_len, a.head_dim = B, Hq, Hkv, T, kv, P, D
    a.dtype = kw.get("dtype", 0)
    a.sm_scale = 0.088
    a.block_m = a.block_n = 64
    a.n_q_blocks = a.n_tree_blocks = -(-T // 64)
    for f, v in kw.items():
        if hasattr(a, f) and f not in ("B", "Hq", "Hkv", "T", "P", "D"):
            setattr(a, f, v)
    return a


def _ws_bytes(a):
    n = ctypes.c_size_t()
    st = nat.load_library().tsfa_fwd_workspace_bytes(ctypes.byref(a), ctypes.byref(n))
    return st, n.value


def test_workspace_bytes_config2():
    st, n = _ws_bytes(_args())
    assert st == 0 and n >= nat.SYNC_BYTES
    st2, n2 = (lambda a: (nat.load_library().tsfa_run_workspace_bytes(ctypes.byref(a), ctypes.byref(ctypes.c_size_t())), 0))(_args())
    assert st2 == 0


@pytest.mark.parametrize("kw,code", [
    (dict(D=96), nat.TSFA_ERR_UNSUPPORTED),
    (dict(dtype=7), nat.TSFA_ERR_UNSUPPORTED),
    (dict(Hq=30, Hkv=8), nat.TSFA_ERR_ASSERT),
    (dict(prefix_len=-1), nat.TSFA_ERR_VALUE),
    (dict(block_m=0), nat.TSFA_ERR_VALUE),
])
def test_fwd_rejects_bad_args_on_host(kw, code):
    a = _args(**kw)
    assert _ws_bytes(a)[0] == code
    ws = ctypes.create_string_buffer(64)
    assert nat.load_library().tsfa_fwd(ctypes.byref(a), ws, 64, None) == code


def test_fwd_rejects_small_workspace_on_host():
    a = _args()
    a.row_ptr = a.col_idx = a.blk_type = 4096
    assert nat.load_library().tsfa_fwd(ctypes.byref(a), None, 0, None) == nat.TSFA_ERR_WORKSPACE


def test_misaligned_pointer_is_unsupported():
    a = _args()
    a.q = 4096 + 2
    assert _ws_bytes(a)[0] == nat.TSFA_ERR_UNSUPPORTED


def test_status_mapping():
    with pytest.raises(ValueError):
        nat.check(nat.TSFA_ERR_VALUE, "x")
    with pytest.raises(AssertionError):
        nat.check(nat.TSFA_ERR_ASSERT, "x")
    with pytest.raises(NotImplementedError):
        nat.check(nat.TSFA_ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        nat.check(nat.TSFA_ERR_DEVICE_TIMEOUT, "x")
    nat.check(nat.TSFA_OK, "x")


# ---------------------------------------------------------------- per-batch trees, paged K/V (host-side checks)
def test_batched_and_paged_workspace_sizes_cover_the_op():
    lib = nat.load_library()
    a = _args(B=3)
    run, bat, pag = (ctypes.c_size_t() for _ in range(3))
    assert lib.tsfa_run_workspace_bytes(ctypes.byref(a), ctypes.byref(run)) == 0
    assert lib.tsfa_run_batched_workspace_bytes(ctypes.byref(a), ctypes.byref(bat)) == 0
    assert lib.tsfa_run_paged_workspace_bytes(ctypes.byref(a), ctypes.byref(pag)) == 0
    meta = ctypes.c_size_t()
    assert lib.tsfa_meta_workspace_bytes(a.q_len, a.block_m, a.block_n, ctypes.byref(meta)) == 0
    assert bat.value > meta.value  # three metadata sets (its forward merges through clusters)
    # the whole op holds one metadata set and the global merge's partial rows:
    # 24 (batch, kv-head) units of 2 row tiles, 3 splits each, 128 rows of 272 bytes
    assert run.value >= meta.value + 24 * 2 * 3 * 128 * 272
    # the paged op adds the tree keys' K and V gathered from the pages
    assert pag.value >= run.value + 2 * 3 * 8 * 64 * 128 * 2


def test_batched_rejects_a_negative_mask_stride_on_host():
    lib = nat.load_library()
    a = _args(B=2)
    ws = ctypes.create_string_buffer(64)
    st = lib.tsfa_run_tree_sparse_batched(ctypes.byref(a), 4096, 0, -64 * 64, 64, ws, 64, None)
    assert st == nat.TSFA_ERR_VALUE


def _kv(page_size=16, num_pages=8, align=0):
    kv = nat.TsfaPagedKV()
    kv.k_pages = kv.v_pages = 4096 + align
    kv.k_stride[:] = (page_size * 8 * 128, 8 * 128, 128, 1)
    kv.v_stride[:] = kv.k_stride[:]
    kv.num_pages, kv.page_size = num_pages, page_size
    kv.page_indptr = kv.page_indices = 8192
    return kv


@pytest.mark.parametrize("kw,code", [
    (dict(page_size=12), nat.TSFA_ERR_UNSUPPORTED),   # not a power of two
    (dict(page_size=4), nat.TSFA_ERR_UNSUPPORTED),    # below 8 rows (SW128 atoms)
    (dict(num_pages=0), nat.TSFA_ERR_VALUE),
    (dict(align=8), nat.TSFA_ERR_UNSUPPORTED),        # pools must be 16-byte aligned
])
def test_paged_rejects_bad_pools_on_host(kw, code):
    lib = nat.load_library()
    a = _args()
    ws = ctypes.create_string_buffer(64)
    st = lib.tsfa_run_tree_sparse_paged(ctypes.byref(a), ctypes.byref(_kv(**kw)), 4096, 0, 64, ws, 64, None)
    assert st == code


def test_paged_rejects_a_small_workspace_on_host():
    lib = nat.load_library()
    a = _args()
    st = lib.tsfa_run_tree_sparse_paged(ctypes.byref(a), ctypes.byref(_kv()), 4096, 0, 64, None, 0, None)
    assert st == nat.TSFA_ERR_WORKSPACE
