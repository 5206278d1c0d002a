"""The debug build (libtsfa_debug.so, -DTSFA_DEBUG): device-side bounds checks
on every metadata index the forward reads (row_ptr order and range, col_idx,
blk_type, mixed_mask_offset and the payload word; csrc/tsfa_common.cuh).

compute-sanitizer is closed on this pool, so these checks stand in for it:
the golden cases run through the debug build must give the release build's
parity with status 0 (no check fires on metadata the reference's builder
produces), and metadata corrupted in value -- never in a way that would make
the release build read outside its buffers -- must be reported as
TSFA_ERR_DEVICE_BOUNDS with the failing check, the tile skipped.
The validation the reference does on the host (tree_sparse_flashattn.py:85-88)
is tested through the status codes elsewhere."""

import os

import numpy as np
import pytest
import torch

import tsfa_native as nat
from conftest import load_npz
from gpu_helpers import assert_close, make_inputs

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def debug_lib():
    if not os.path.exists(nat.DEBUG_LIB_PATH):
        pytest.fail("libtsfa_debug.so is not built (python eagle3-tree-sparse-flashattn_b200/csrc/build.py --debug)")
    dbg = nat.load_library(nat.DEBUG_LIB_PATH)
    saved = nat.load_library()
    nat._lib = dbg
    try:
        yield dbg
    finally:
        nat._lib = saved


def _ids():
    return [str(x) for x in load_npz("attn_golden.npz")["__ids__"]]


@pytest.mark.parametrize("cid", _ids())
@pytest.mark.parametrize("blocks", [(64, 64), (16, 16), (32, 16)])
def test_golden_cases_debug_build(debug_lib, attn_golden, cid, blocks):
    B, Hq, Hkv, D, P, T = (int(x) for x in attn_golden[f"{cid}.shape"])
    q, k, v = (x.cuda() for x in make_inputs(int(attn_golden[f"{cid}.seed"]), B, Hq, Hkv, D, P, T))
    out = torch.empty_like(q)
    # the ctypes binding calls the library swapped in by the fixture
    nat.run_tree_sparse(q, k, v, torch.as_tensor(attn_golden[f"{cid}.mask"]).cuda(), out, prefix_len=P,
                        block_m=blocks[0], block_n=blocks[1])
    torch.cuda.synchronize()
    assert nat.read_device_status_detail(out.device) == (0, 0, 0, 0)
    assert_close(out, attn_golden[f"{cid}.out"])


def test_golden_metadata_debug_build(debug_lib, meta_golden):
    for cid in [str(x) for x in meta_golden["__ids__"]]:
        mask = torch.from_numpy(np.ascontiguousarray(meta_golden[f"{cid}.mask"])).cuda()
        bm, bn, P = (int(x) for x in meta_golden[f"{cid}.params"][:3])
        d, row_ptr, col_idx, blk_type, payload, offset, nnz, n_mixed = nat.build_metadata_device(mask, bm, bn)
        W = int(d.words_per_tile)
        got = {"row_ptr": row_ptr, "col_idx": col_idx[:nnz], "blk_type": blk_type[:nnz],
               "mixed_mask_payload": payload[:n_mixed * W], "mixed_mask_offset": offset[:nnz if n_mixed else 0]}
        for f, t in got.items():
            assert np.array_equal(t.cpu().numpy(), meta_golden[f"{cid}.{f}"]), (cid, f)


@pytest.mark.parametrize("field,check", [("blk_type", 103), ("col_idx", 102)])
def test_corrupted_metadata_is_reported(debug_lib, field, check):
    """Value corruption that stays inside the buffers: a block type that is
    neither FULL nor MIXED, a tree column past n_tree_blocks."""
    import tree_sparse_flashattn as tsfa
    import tsfa_trees as trees

    B, Hq, Hkv, D, P, T = 1, 8, 2, 128, 256, 64
    q, k, v = (x.cuda() for x in make_inputs(31, B, Hq, Hkv, D, P, T))
    mask = torch.from_numpy(trees.random_tree(T, 6, 4, seed=31)).cuda()
    meta = tsfa.prepare_tree_sparse_metadata(mask, P, 16, 16)
    bad = getattr(meta, field).clone()
    bad[0] = 7 if field == "blk_type" else meta.n_tree_blocks + 5  # entry 0: row 0's root tile
    setattr(meta, field, bad)
    out = torch.empty_like(q)
    nat.fwd_with_metadata(q, k, v, out, meta, prefix_len=P)
    torch.cuda.synchronize()
    status, got_check, index, _ = nat.read_device_status_detail(out.device)
    assert status == nat.TSFA_ERR_DEVICE_BOUNDS and got_check == check and index == 0, (status, got_check, index)
    assert nat.read_device_status(out.device) == 0  # cleared by the read
