"""K1 (GPU metadata builder) is bit-exact with the reference's
prepare_tree_sparse_metadata on every golden case (values, dtypes, shapes)."""

import numpy as np
import pytest
import torch

from conftest import load_npz

pytestmark = pytest.mark.gpu

FIELDS = ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset")


def _ids():
    return [str(x) for x in load_npz("meta_golden.npz")["__ids__"]]


@pytest.mark.parametrize("on_gpu", [True, False])
@pytest.mark.parametrize("cid", _ids())
def test_gpu_metadata_bit_exact(meta_golden, cid, on_gpu):
    import tree_sparse_flashattn as tsfa

    mask = torch.from_numpy(np.ascontiguousarray(meta_golden[f"{cid}.mask"]))
    if on_gpu:
        mask = mask.cuda()
    bm, bn, P, nqb, ntb = (int(x) for x in meta_golden[f"{cid}.params"])
    md = tsfa.prepare_tree_sparse_metadata(mask, P, bm, bn)
    assert (md.n_q_blocks, md.n_tree_blocks, md.block_m, md.block_n, md.prefix_len) == (nqb, ntb, bm, bn, P)
    for f in FIELDS:
        got = getattr(md, f)
        assert got.device.type == ("cuda" if on_gpu else "cpu"), f
        want = meta_golden[f"{cid}.{f}"]
        got = got.cpu().numpy()
        assert got.dtype == want.dtype and got.shape == want.shape, (f, got.dtype, got.shape, want.shape)
        assert np.array_equal(got, want), f


def test_gpu_metadata_strided_mask(meta_golden):
    import tree_sparse_flashattn as tsfa

    cid = "cfg3_tree_16x16"
    m = torch.from_numpy(meta_golden[f"{cid}.mask"]).cuda()
    big = torch.zeros((m.shape[0], m.shape[1] + 37), dtype=torch.bool, device="cuda")
    big[:, 5:5 + m.shape[1]] = m
    view = big[:, 5:5 + m.shape[1]]  # row stride != q_len
    md = tsfa.prepare_tree_sparse_metadata(view, 8192, 16, 16)
    assert np.array_equal(md.mixed_mask_payload.cpu().numpy(), meta_golden[f"{cid}.mixed_mask_payload"])
    assert np.array_equal(md.col_idx.cpu().numpy(), meta_golden[f"{cid}.col_idx"])


def test_gpu_pack_bits():
    import tree_sparse_flashattn as tsfa

    g = load_npz("pack_golden.npz")
    n = len([k for k in g.files if k.endswith(".tile")])
    for i in range(n):
        tile = torch.from_numpy(g[f"t{i}.tile"])
        for t in (tile, tile.cuda()):
            got = tsfa._pack_block_mask_to_int32(t)
            assert got.dtype == torch.int32 and got.device == t.device
            assert np.array_equal(got.cpu().numpy(), g[f"t{i}.words"]), i


def test_gpu_metadata_repeat_calls_stable(meta_golden):
    """The large path's arrival counter is left at zero: repeated builds agree."""
    import tree_sparse_flashattn as tsfa

    cid = "tree1024_16x16"
    m = torch.from_numpy(meta_golden[f"{cid}.mask"]).cuda()
    for _ in range(3):
        md = tsfa.prepare_tree_sparse_metadata(m, 1024, 16, 16)
        assert np.array_equal(md.mixed_mask_payload.cpu().numpy(), meta_golden[f"{cid}.mixed_mask_payload"])
        assert np.array_equal(md.row_ptr.cpu().numpy(), meta_golden[f"{cid}.row_ptr"])
