"""The sparsity / tiling sweep (fifth benchmark configuration) on the GPU, at
every point: batch 32, 32 q-heads / 8 kv-heads, head_dim {64, 128},
prefix_len {0, 1024, 16384}, tree sizes {64, 512, 1024}, every BLOCK_M x
BLOCK_N pair of {16, 32, 64, 128}, star / chain / wide / deep trees (~0.2 % to
~50 % visible pairs).

* Metadata: K1 on the device is bit-exact with the reference's builder
  (tree_sparse_flashattn.py:67-160) at all 192 (tree size, tree, BM, BN)
  points -- compared by digest with fixtures made by running the reference
  (tests/golden/gen_golden.py --parts sweep5).
* Outputs: run_tree_sparse_kernel at the full batch of 32 for all 1152
  points; for each point three sampled (batch, kv-head) units -- the first,
  the last and one in the middle, each the G = 4 query heads of its kv-head
  -- are checked against the dense+mask fp32 oracle (benchmark.py:8-35
  restated), computed once per (head_dim, prefix, tree) because the block
  sizes change only the metadata, not the answer.

Inputs are N(0, 1) bf16 drawn on the device from a seeded generator (2.3 GB
of K/V at the largest point); the sampled units are copied to the host for
the oracle, so the oracle sees exactly the values the kernel saw.
"""

import pytest
import torch

import tsfa_oracle as orc
import tsfa_trees as trees
from conftest import load_npz, metadata_digest
from gpu_helpers import assert_close

pytestmark = pytest.mark.gpu

S = trees.SWEEP5
UNITS = [(0, 0), (17, 3), (S["B"] - 1, S["Hkv"] - 1)]


@pytest.fixture(scope="module")
def sweep5():
    return load_npz("sweep5_golden.npz")


@pytest.mark.parametrize("T", S["T"])
@pytest.mark.parametrize("kind", trees.SWEEP5_TREES)
def test_sweep5_metadata_bit_exact(sweep5, T, kind):
    import tree_sparse_flashattn as tsfa

    mask = torch.from_numpy(trees.sweep5_tree(kind, T)).cuda()
    for bm in S["BLOCKS"]:
        for bn in S["BLOCKS"]:
            md = tsfa.prepare_tree_sparse_metadata(mask, 0, bm, bn)
            assert md.row_ptr.device.type == "cuda"
            cid = f"T{T}_{kind}_{bm}x{bn}"
            assert metadata_digest(md) == bytes(sweep5[f"{cid}.sha256"]), cid


@pytest.mark.parametrize("T", S["T"])
@pytest.mark.parametrize("P", S["P"])
@pytest.mark.parametrize("D", S["D"])
def test_sweep5_outputs(D, P, T):
    import eagle_tree_sparse_bridge as br
    import tsfa_native as nat

    B, Hq, Hkv = S["B"], S["Hq"], S["Hkv"]
    G = Hq // Hkv
    gen = torch.Generator(device="cuda").manual_seed(5000 + 7 * D + 13 * P + T)
    q = torch.randn((B, Hq, T, D), generator=gen, device="cuda").to(torch.bfloat16)
    k = torch.randn((B, Hkv, P + T, D), generator=gen, device="cuda").to(torch.bfloat16)
    v = torch.randn((B, Hkv, P + T, D), generator=gen, device="cuda").to(torch.bfloat16)
    host = {u: tuple(x.float().cpu().numpy()[None] for x in (q[u[0], u[1] * G:(u[1] + 1) * G], k[u[0], u[1]:u[1] + 1],
                                                              v[u[0], u[1]:u[1] + 1])) for u in UNITS}
    for kind in trees.SWEEP5_TREES:
        mask = trees.sweep5_tree(kind, T)
        want = {u: orc.dense_tree_attention(qu, ku, vu, mask, P)[0] for u, (qu, ku, vu) in host.items()}
        mask_d = torch.from_numpy(mask).cuda()
        for bm in S["BLOCKS"]:
            for bn in S["BLOCKS"]:
                out = br.run_tree_sparse_kernel(q, k, v, mask_d, block_m=bm, block_n=bn)
                assert nat.read_device_status(out.device) == 0
                for (b, kh), w in want.items():
                    assert_close(out[b, kh * G:(kh + 1) * G], w,
                                 what=f"D={D} P={P} T={T} {kind} {bm}x{bn} unit ({b},{kh}):")
