"""Pin the numpy oracle to fixtures produced by the reference implementation."""

import numpy as np
import pytest

import tsfa_oracle as orc
from conftest import bf16_inputs, load_npz

FIELDS = ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset")


def _ids():
    return [str(x) for x in load_npz("meta_golden.npz")["__ids__"]]


@pytest.mark.parametrize("cid", _ids())
def test_metadata_bit_exact(meta_golden, cid):
    mask = meta_golden[f"{cid}.mask"]
    bm, bn, P, nqb, ntb = (int(x) for x in meta_golden[f"{cid}.params"])
    md = orc.prepare_tree_sparse_metadata(mask, P, bm, bn)
    assert (md.n_q_blocks, md.n_tree_blocks, md.block_m, md.block_n, md.prefix_len) == (nqb, ntb, bm, bn, P)
    for f in FIELDS:
        want = meta_golden[f"{cid}.{f}"]
        got = getattr(md, f)
        assert got.dtype == want.dtype, (f, got.dtype, want.dtype)
        assert got.shape == want.shape, (f, got.shape, want.shape)
        assert np.array_equal(got, want), f
    # CSR + bitsets expand back to the bool mask (round trip).
    assert np.array_equal(orc.metadata_to_dense(md, mask.shape[0]), mask != 0)


def test_pack_bits():
    g = load_npz("pack_golden.npz")
    n = len([k for k in g.files if k.endswith(".tile")])
    for i in range(n):
        got = orc.pack_block_mask_to_int32(g[f"t{i}.tile"])
        want = g[f"t{i}.words"]
        assert got.dtype == np.int32 and np.array_equal(got, want), i


def test_pack_bit31_is_negative():
    tile = np.zeros((1, 32), np.bool_)
    tile[0, 31] = True
    assert orc.pack_block_mask_to_int32(tile).tolist() == [-2147483648]


def test_metadata_errors():
    with pytest.raises(ValueError):
        orc.prepare_tree_sparse_metadata(np.ones((3, 4), np.bool_), 0, 16, 16)
    with pytest.raises(ValueError):
        orc.prepare_tree_sparse_metadata(np.ones((3,), np.bool_), 0, 16, 16)
    with pytest.raises(ValueError):
        orc.prepare_tree_sparse_metadata(np.ones((3, 3), np.bool_), 0, 0, 16)
    with pytest.raises(ValueError):
        orc.prepare_tree_sparse_metadata(np.ones((3, 3), np.bool_), 0, 16, -1)


def _attn_case(g, cid):
    B, Hq, Hkv, D, P, T = (int(x) for x in g[f"{cid}.shape"])
    q, k, v = bf16_inputs(int(g[f"{cid}.seed"]), B, Hq, Hkv, D, P, T)
    return q.float().numpy(), k.float().numpy(), v.float().numpy(), g[f"{cid}.mask"], P


@pytest.mark.parametrize("cid", [str(x) for x in load_npz("attn_golden.npz")["__ids__"]])
def test_dense_attention_matches_reference(attn_golden, cid):
    q, k, v, mask, P = _attn_case(attn_golden, cid)
    want = attn_golden[f"{cid}.out"]
    got = orc.dense_tree_attention(q, k, v, mask, P)
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.max(np.abs(got[ok] - want[ok])) < 1e-5


@pytest.mark.parametrize("cid", [str(x) for x in load_npz("attn_golden.npz")["__ids__"]])
@pytest.mark.parametrize("blocks", [(16, 16), (8, 32), (64, 64)])
def test_blocked_kernel_semantics_match_dense(attn_golden, cid, blocks):
    """The CSR/bitset walk (tsfa.py:163-339) equals dense+mask (benchmark.py:8-35)."""
    q, k, v, mask, P = _attn_case(attn_golden, cid)
    md = orc.prepare_tree_sparse_metadata(mask, P, *blocks)
    got = orc.blocked_tree_attention(q, k, v, md, mask.shape[0], k.shape[2])
    want = attn_golden[f"{cid}.out"]
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.max(np.abs(got[ok] - want[ok])) < 1e-5


def test_config1_matches_reference():
    import tsfa_trees as trees

    g = load_npz("cfg1_golden.npz")
    c = trees.CONFIGS["cfg1_cpu"]
    mask = trees.config_tree(c, seed=0)
    assert np.array_equal(mask, g["mask"])  # generator is stable across hosts
    q, k, v = bf16_inputs(int(g["seed"]), c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    assert abs(q.double().sum().item() - float(g["q_sum"])) < 1e-6
    got = orc.dense_tree_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(), mask, c["P"])
    assert np.max(np.abs(got.reshape(-1)[::17] - g["out_sample"])) < 1e-5


def test_extract_tree_mask():
    g = load_npz("extract_golden.npz")
    names = sorted({k.split(".")[0] for k in g.files})
    for n in names:
        got = orc.extract_tree_mask(g[f"{n}.in"], int(g[f"{n}.q_len"]), int(g[f"{n}.kv_len"]))
        if bool(g[f"{n}.none"]):
            assert got is None, n
        else:
            assert np.array_equal(got, g[f"{n}.out"]), n


def test_planted_mistake_is_caught(meta_golden):
    """A one-bit error planted in the oracle's output must fail the comparison."""
    cid = "cfg2_tree_64x64"
    mask = meta_golden[f"{cid}.mask"]
    md = orc.prepare_tree_sparse_metadata(mask, 4096, 64, 64)
    bad = md.mixed_mask_payload.copy()
    bad[3] ^= 1 << 7
    assert not np.array_equal(bad, meta_golden[f"{cid}.mixed_mask_payload"])
