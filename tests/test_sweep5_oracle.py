"""The sparsity / tiling sweep (fifth benchmark configuration) on the CPU:
the seeded tree generator still produces the masks the fixtures were made
from, and the oracle's metadata (tsfa.py:67-160 restated) equals the
reference's at every (tree size, tree, BLOCK_M, BLOCK_N) point -- 192 points,
BM != BN included, star / chain / wide / deep trees spanning ~0.2 % to ~50 %
visible pairs.  The fixture (tests/golden/sweep5_golden.npz) holds digests
made by running the reference's builder (tests/golden/gen_golden.py)."""

import pytest

import tsfa_oracle as orc
import tsfa_trees as trees
from conftest import load_npz, mask_digest, metadata_digest


@pytest.fixture(scope="module")
def sweep5():
    return load_npz("sweep5_golden.npz")


def test_every_sweep_point_has_a_fixture(sweep5):
    s = trees.SWEEP5
    ids = {str(x) for x in sweep5["__ids__"]}
    want = {f"T{T}_{k}_{bm}x{bn}" for T in s["T"] for k in trees.SWEEP5_TREES for bm in s["BLOCKS"]
            for bn in s["BLOCKS"]}
    assert ids == want and len(ids) == 192


@pytest.mark.parametrize("T", trees.SWEEP5["T"])
@pytest.mark.parametrize("kind", trees.SWEEP5_TREES)
def test_generator_and_oracle_metadata_match_the_reference(sweep5, T, kind):
    mask = trees.sweep5_tree(kind, T)
    assert bytes(sweep5[f"T{T}_{kind}.mask_sha256"]) == mask_digest(mask)
    assert abs(float(sweep5[f"T{T}_{kind}.visible_fraction"]) - float(mask.mean())) < 1e-12
    for bm in trees.SWEEP5["BLOCKS"]:
        for bn in trees.SWEEP5["BLOCKS"]:
            md = orc.prepare_tree_sparse_metadata(mask, 0, bm, bn)
            cid = f"T{T}_{kind}_{bm}x{bn}"
            assert metadata_digest(md) == bytes(sweep5[f"{cid}.sha256"]), cid
            nnz, n_mixed, nqb, ntb = (int(x) for x in sweep5[f"{cid}.counts"])
            assert (md.col_idx.size, int((md.blk_type == 1).sum()), md.n_q_blocks, md.n_tree_blocks) == \
                (nnz, n_mixed, nqb, ntb)


def test_sweep_spans_the_density_range(sweep5):
    fr = [float(sweep5[f"T{T}_{k}.visible_fraction"]) for T in trees.SWEEP5["T"] for k in trees.SWEEP5_TREES]
    assert min(fr) < 0.01 and max(fr) > 0.49
