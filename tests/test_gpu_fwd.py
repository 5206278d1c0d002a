"""GPU parity of the forward (run_tree_sparse_kernel and the kernel launcher)
against the dense+mask fp32 oracle (benchmark.py:8-35 restated)."""

import numpy as np
import pytest
import torch

import tsfa_trees as trees
from conftest import load_npz
from gpu_helpers import ATOL, assert_close, make_inputs, oracle, p_rounding_bound

pytestmark = pytest.mark.gpu


def _run(q, k, v, mask, bm=64, bn=64):
    import eagle_tree_sparse_bridge as br
    import tsfa_native as nat

    out = br.run_tree_sparse_kernel(q.cuda(), k.cuda(), v.cuda(), torch.as_tensor(mask), block_m=bm, block_n=bn)
    torch.cuda.synchronize()
    assert nat.read_device_status(out.device) == 0  # no bounded wait gave up
    return out


@pytest.mark.parametrize("cid", [str(x) for x in load_npz("attn_golden.npz")["__ids__"]])
@pytest.mark.parametrize("blocks", [(64, 64), (16, 16), (32, 16)])
def test_golden_cases(attn_golden, cid, blocks):
    B, Hq, Hkv, D, P, T = (int(x) for x in attn_golden[f"{cid}.shape"])
    q, k, v = make_inputs(int(attn_golden[f"{cid}.seed"]), B, Hq, Hkv, D, P, T)
    out = _run(q, k, v, attn_golden[f"{cid}.mask"], *blocks)
    assert out.dtype == torch.bfloat16 and out.shape == q.shape
    assert_close(out, attn_golden[f"{cid}.out"])


@pytest.mark.parametrize("name", ["cfg1_cpu", "cfg2_llama3_8b"])
@pytest.mark.parametrize("blocks", [(64, 64), (16, 16), (128, 128), (16, 64)])
def test_benchmark_configs(name, blocks):
    c = trees.CONFIGS[name]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(1, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    out = _run(q, k, v, mask, *blocks)
    err = assert_close(out, oracle(q, k, v, mask, c["P"]))
    assert err <= ATOL  # |O| is small here: the plain 2e-3 bound holds


@pytest.mark.parametrize("name,units", [
    ("cfg3_serving_70b", [(0, 0), (7, 3), (15, 7)]),
    ("cfg4_long_ctx", [(0, 0), (3, 7)]),
])
def test_large_configs_sliced(name, units):
    c = trees.CONFIGS[name]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(2, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    out = _run(q, k, v, mask)
    want = oracle(q, k, v, mask, c["P"], units=units)
    G = c["Hq"] // c["Hkv"]
    for (b, kh), w in want.items():
        assert_close(out[b, kh * G:(kh + 1) * G], w)


SWEEP = [
    # (B, Hq, Hkv, D, P, T, tree, BM, BN)
    (2, 32, 8, 64, 1024, 64, "tree", 16, 16),
    (2, 32, 8, 128, 0, 64, "tree", 32, 32),
    (1, 32, 8, 128, 0, 512, "chain", 64, 64),
    (1, 32, 8, 64, 0, 512, "star", 128, 128),
    (1, 8, 8, 128, 1024, 1024, "tree", 64, 64),
    (1, 32, 8, 64, 16384, 64, "star", 16, 32),
    (3, 12, 4, 128, 700, 100, "tree", 16, 16),
    (1, 4, 4, 64, 300, 1, "tree", 64, 64),
    (1, 64, 8, 128, 2048, 256, "tree", 64, 64),
    (1, 16, 2, 128, 33, 200, "chain", 128, 16),
]


@pytest.mark.parametrize("case", SWEEP)
def test_sweep_points(case):
    B, Hq, Hkv, D, P, T, kind, bm, bn = case
    mask = {"tree": lambda: trees.random_tree(T, 10, 6, seed=T + P),
            "chain": lambda: trees.chain_tree(T), "star": lambda: trees.star_tree(T)}[kind]()
    q, k, v = make_inputs(3, B, Hq, Hkv, D, P, T)
    out = _run(q, k, v, mask, bm, bn)
    assert_close(out, oracle(q, k, v, mask, P))


def test_fp16_inputs():
    c = trees.CONFIGS["cfg1_cpu"]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(4, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"], dtype=torch.float16)
    out = _run(q, k, v, mask)
    assert out.dtype == torch.float16
    assert_close(out, oracle(q, k, v, mask, c["P"]), dtype=torch.float16)


def test_empty_mask_row_gives_nan():
    """P = 0 and a tree row that sees nothing: 0 / 0 like tsfa.py:329."""
    mask = trees.chain_tree(40)
    mask[17, :] = False
    q, k, v = make_inputs(5, 1, 4, 2, 64, 0, 40)
    out = _run(q, k, v, mask, 16, 16)
    assert torch.isnan(out[0, :, 17]).all()
    assert not torch.isnan(out[0, :, :17]).any() and not torch.isnan(out[0, :, 18:]).any()
    assert_close(out, oracle(q, k, v, mask, 0))


def test_known_answers():
    # one visible key -> that key's V row; all-equal K -> mean of visible V rows
    T, D = 8, 64
    q, k, v = make_inputs(6, 1, 2, 1, D, 0, T)
    mask = np.eye(T, dtype=bool)
    out = _run(q, k, v, mask, 8, 8)
    ref = v[0, 0].float().repeat(2, 1, 1)
    assert torch.allclose(out[0].float().cpu(), ref, atol=0, rtol=2.0 ** -8)
    k2 = torch.ones_like(k)
    mask2 = np.ones((T, T), dtype=bool)
    out2 = _run(q, k2, v, mask2, 8, 8)
    mean = v[0, 0].float().mean(0)
    assert torch.allclose(out2[0].float().cpu(), mean.expand(2, T, D), atol=2e-3)


def test_strided_inputs():
    """[B, T, H, D] projections viewed as [B, H, T, D] (no copy)."""
    B, Hq, Hkv, D, P, T = 2, 16, 4, 128, 256, 48
    q, k, v = make_inputs(7, B, Hq, Hkv, D, P, T)
    mask = trees.random_tree(T, 5, 4, seed=7)
    qs = q.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    ks = k.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    vs = v.transpose(1, 2).contiguous().cuda().transpose(1, 2)
    import eagle_tree_sparse_bridge as br

    out = br.run_tree_sparse_kernel(qs, ks, vs, torch.from_numpy(mask).cuda(), block_m=16, block_n=16)
    assert_close(out, oracle(q, k, v, mask, P))


def test_kernel_launcher_matches_bridge():
    """benchmark.py-style launch with prebuilt device metadata == one-call op."""
    import eagle_tree_sparse_bridge as br
    import tree_sparse_flashattn as tsfa

    B, Hq, Hkv, D, P, T, BM, BN = 2, 32, 8, 128, 1024, 64, 16, 16
    q, k, v = (x.cuda() for x in make_inputs(8, B, Hq, Hkv, D, P, T))
    mask = torch.from_numpy(trees.random_causal_sparse(T, seed=42)).cuda()
    meta = tsfa.prepare_tree_sparse_metadata(mask, P, BM, BN)
    o = torch.empty_like(q)
    grid = (meta.n_q_blocks, B * Hq)
    tsfa.block_sparse_tree_fwd_kernel[grid](
        q, k, v, o, meta.row_ptr, meta.col_idx, meta.blk_type, meta.mixed_mask_payload, meta.mixed_mask_offset,
        *q.stride(), *k.stride(), *v.stride(), *o.stride(),
        1.0 / D ** 0.5, B, Hq, Hkv, T, P + T, P, meta.n_q_blocks, meta.n_tree_blocks, Hq // Hkv,
        BLOCK_M=BM, BLOCK_N=BN, BLOCK_D=D, num_warps=4, num_stages=2)
    ref = br.run_tree_sparse_kernel(q, k, v, mask, block_m=BM, block_n=BN)
    torch.cuda.synchronize()
    assert torch.equal(o, ref)


def test_cuda_graph_replay():
    import eagle_tree_sparse_bridge as br

    c = trees.CONFIGS["cfg2_llama3_8b"]
    mask = torch.from_numpy(trees.config_tree(c, seed=0)).cuda()
    q, k, v = (x.cuda() for x in make_inputs(9, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"]))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        eager = br.run_tree_sparse_kernel(q, k, v, mask, block_m=64, block_n=64)  # warm-up (workspace)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            out = br.run_tree_sparse_kernel(q, k, v, mask, block_m=64, block_n=64)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_errors_match_reference_exceptions():
    import eagle_tree_sparse_bridge as br

    q = torch.zeros(1, 4, 8, 64, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(1, 2, 6, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError):
        br.run_tree_sparse_kernel(q, k, k, torch.ones(8, 8, dtype=torch.bool), block_m=4, block_n=4)  # kv < q
    k = torch.zeros(1, 2, 16, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError):
        br.run_tree_sparse_kernel(q, k, k[:, :, :, :32], torch.ones(8, 8, dtype=torch.bool), block_m=4, block_n=4)
    with pytest.raises(AssertionError):
        br.run_tree_sparse_kernel(q.cpu(), k, k, torch.ones(8, 8, dtype=torch.bool), block_m=4, block_n=4)
    with pytest.raises(ValueError):
        br.run_tree_sparse_kernel(q, k, k, torch.ones(8, 8, dtype=torch.bool), block_m=0, block_n=4)
    with pytest.raises(TypeError):
        br.run_tree_sparse_kernel(q.float(), k.float(), k.float(), torch.ones(8, 8, dtype=torch.bool),
                                  block_m=4, block_n=4)


def test_rescale_in_some_rows_only():
    """Rows whose running max jumps by > 2^8 rescale O in TMEM while their warp
    neighbours do not (the lazy-rescale branch must stay warp-collective)."""
    B, Hq, Hkv, D, P, T = 1, 8, 2, 128, 512, 32
    q, k, v = make_inputs(11, B, Hq, Hkv, D, P, T)
    k = k.clone()
    k[:, :, 256:384] *= 8.0       # third prefix tile: much larger scores ...
    q = q.clone()
    q[:, :, 1::2] *= 0.01         # ... except for the odd tree rows
    mask = trees.random_tree(T, 5, 3, seed=11)
    out = _run(q, k, v, mask, 16, 16)
    # very peaked softmax rows: allow the bf16 rounding of p that the
    # reference kernel performs as well
    assert_close(out, oracle(q, k, v, mask, P), extra=p_rounding_bound(q, k, v, mask, P))


@pytest.mark.parametrize("name,P,D,blocks", [
    ("cfg2_llama3_8b", None, 128, (64, 64)),  # 16 row tiles: 9 splits per tile, merged through global memory
    ("cfg2_llama3_8b", 700, 64, (32, 32)),
    ("cfg1_cpu", None, 128, (16, 16)),
])
def test_fwd_with_prebuilt_metadata(name, P, D, blocks):
    """tsfa_fwd over device metadata (the kernel-launcher path): where one CTA
    per SM gives more splits than cluster co-scheduling, the splits merge
    through global memory in a cooperative launch."""
    import tree_sparse_flashattn as tsfa
    import tsfa_native as nat

    c = dict(trees.CONFIGS[name])
    P = c["P"] if P is None else P
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(5, c["B"], c["Hq"], c["Hkv"], D, P, c["T"])
    qd, kd, vd = (x.cuda() for x in (q, k, v))
    meta = tsfa.prepare_tree_sparse_metadata(torch.from_numpy(mask).cuda(), P, *blocks)
    out = torch.full_like(qd, float("nan"))
    for _ in range(2):  # the merge counters must be back at zero for the second call
        nat.fwd_with_metadata(qd, kd, vd, out, meta, prefix_len=P)
        torch.cuda.synchronize()
        assert nat.read_device_status(out.device) == 0
        err = assert_close(out, oracle(q, k, v, mask, P))
        assert err <= ATOL


@pytest.mark.parametrize("name,P,D,blocks,dtype", [
    ("cfg2_llama3_8b", None, 128, (64, 64), torch.bfloat16),
    ("cfg2_llama3_8b", 700, 64, (32, 32), torch.bfloat16),
    ("cfg2_llama3_8b", 1500, 128, (16, 16), torch.float16),
])
def test_whole_op_both_merges(name, P, D, blocks, dtype):
    """The whole op merges its splits through global memory (cooperative
    launch behind the metadata kernel) where that gives more splits; forced
    onto the thread-block-cluster merge (the per-batch op's), it must agree
    with the oracle too."""
    import tsfa_native as nat

    c = dict(trees.CONFIGS[name])
    P = c["P"] if P is None else P
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(6, c["B"], c["Hq"], c["Hkv"], D, P, c["T"], dtype=dtype)
    want = oracle(q, k, v, mask, P)
    got = {}
    for forced in (False, True):
        nat.force_cluster_merge(forced)
        try:
            got[forced] = _run(q, k, v, mask, *blocks)
        finally:
            nat.force_cluster_merge(False)
        assert nat.last_plan()["merge"] == ("cluster" if forced else "global"), nat.last_plan()
        assert_close(got[forced], want)


PAIR_CASES = [
    # (id, B, Hq, Hkv, D, P, tree, dtype): two or more row tiles per (batch, kv-head)
    ("d128-p1500-random", 2, 16, 4, 128, 1500, lambda: trees.random_tree(64, 6, 4, seed=3), torch.bfloat16),
    ("d64-p700-odd-tiles", 1, 8, 2, 64, 700, lambda: trees.random_tree(96, 5, 3, seed=7), torch.bfloat16),
    ("d64-p0-chain", 2, 8, 4, 64, 0, lambda: trees.chain_tree(70), torch.bfloat16),
    ("d128-p0-star", 1, 32, 8, 128, 0, lambda: trees.star_tree(64), torch.bfloat16),
    ("d128-p4096-fp16", 1, 32, 8, 128, 4096, lambda: trees.random_tree(64, 6, 4, seed=0), torch.float16),
    ("d128-p1024-T300", 1, 16, 2, 128, 1024, lambda: trees.random_tree(300, 8, 4, seed=9), torch.bfloat16),
]


@pytest.mark.parametrize("cid,B,Hq,Hkv,D,P,tree,dtype", PAIR_CASES, ids=[c[0] for c in PAIR_CASES])
def test_row_tile_pairs(cid, B, Hq, Hkv, D, P, tree, dtype):
    """One CTA per two row tiles (the plan of shapes whose pairs fill the
    GPU, e.g. config 3), forced onto smaller shapes: odd row-tile counts, both
    head dims, P = 0 and P > 0, fp16.  With head_dim 128 the pairs round P
    once on tree tiles, as the reference (tsfa.py:278) -- the oracle bound
    then adds that rounding (the library picks pairs there only where every
    row sees >= 1024 prefix keys)."""
    import tsfa_native as nat

    mask = tree()
    T = mask.shape[0]
    q, k, v = make_inputs(8, B, Hq, Hkv, D, P, T, dtype=dtype)
    nat.force_row_pairs(True)
    try:
        out = _run(q, k, v, mask, 32, 32)
    finally:
        nat.force_row_pairs(False)
    assert nat.last_plan()["merge"] == "pair", nat.last_plan()
    extra = p_rounding_bound(q, k, v, mask, P) if D == 128 else None
    assert_close(out, oracle(q, k, v, mask, P), dtype=dtype, extra=extra)


def test_config3_runs_row_tile_pairs():
    """Config 3 (1024 row-tile pairs) takes the pair plan by itself."""
    import tsfa_native as nat

    c = trees.CONFIGS["cfg3_serving_70b"]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(3, 2, c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])  # two batch rows: 128 pairs
    q, k, v = (torch.cat([x] * 8) for x in (q, k, v))                      # 16 batch rows: 1024 pairs
    out = _run(q, k, v, mask)
    assert nat.last_plan()["merge"] == "pair", nat.last_plan()
    want = oracle(q[:2], k[:2], v[:2], mask, c["P"], units=[(0, 0), (1, 5)])
    G = c["Hq"] // c["Hkv"]
    for (b, kh), w in want.items():
        assert_close(out[b, kh * G:(kh + 1) * G], w)
        assert torch.equal(out[b + 8], out[b])  # the same problem again in batch row b + 8
