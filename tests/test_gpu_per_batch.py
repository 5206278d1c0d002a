"""Per-batch draft trees: tsfa_run_tree_sparse_batched and the bridge's
run_tree_sparse_kernel_per_batch / extract_tree_masks_per_batch, against the
fp32 oracle applied to each batch element with its own tree.  (The reference
has no per-batch path: it applies batch 0's tree to every element.)"""

import ctypes

import numpy as np
import pytest
import torch

import eagle_tree_sparse_bridge as br
import tsfa_native as nat
import tsfa_trees as trees
from gpu_helpers import ATOL, assert_close, make_inputs, oracle

pytestmark = pytest.mark.gpu


def _per_batch_oracle(q, k, v, masks, P):
    return np.concatenate([oracle(q[b:b + 1], k[b:b + 1], v[b:b + 1], masks[b], P) for b in range(q.shape[0])])


def _masks(B, T, seed):
    kinds = [trees.random_tree(T, 6, 4, seed=seed + b) for b in range(B)]
    if B > 1:
        kinds[1] = trees.chain_tree(T)
    if B > 2:
        kinds[2] = trees.star_tree(T)
    return np.stack(kinds)


@pytest.mark.parametrize("B,Hq,Hkv,D,P,T,BM,BN", [
    (3, 8, 2, 128, 100, 40, 16, 16),
    (3, 32, 8, 128, 512, 64, 64, 64),
    (4, 4, 4, 64, 0, 48, 32, 16),
    (2, 4, 2, 64, 64, 600, 16, 16),  # 1444 tiles per mask: the metadata kernel's grid path, one mask at a time
])
def test_per_batch_trees_match_oracle(B, Hq, Hkv, D, P, T, BM, BN):
    q, k, v = make_inputs(31, B, Hq, Hkv, D, P, T)
    masks = _masks(B, T, seed=5)
    out = br.run_tree_sparse_kernel_per_batch(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(masks).cuda(),
                                              block_m=BM, block_n=BN)
    torch.cuda.synchronize()
    assert nat.read_device_status(out.device) == 0
    assert_close(out, _per_batch_oracle(q, k, v, masks, P), atol=ATOL)


def test_same_tree_everywhere_equals_the_shared_tree_op():
    B, Hq, Hkv, D, P, T = 3, 16, 4, 128, 300, 50
    q, k, v = (x.cuda() for x in make_inputs(32, B, Hq, Hkv, D, P, T))
    mask = torch.from_numpy(trees.random_tree(T, 5, 3, seed=9)).cuda()
    shared = br.run_tree_sparse_kernel(q, k, v, mask, block_m=16, block_n=32)
    per_batch = br.run_tree_sparse_kernel_per_batch(q, k, v, mask.expand(B, T, T), block_m=16, block_n=32)
    torch.cuda.synchronize()
    assert torch.equal(shared, per_batch)


def test_patched_dispatch_reads_every_batch_elements_tree():
    """The 4-D additive mask of a batch of verify steps -> per-batch trees."""
    B, Hq, Hkv, D, P, T = 2, 8, 2, 128, 70, 24
    q, k, v = make_inputs(33, B, Hq, Hkv, D, P, T)
    masks = _masks(B, T, seed=11)
    add = torch.zeros((B, 1, T, P + T))
    add[:, 0, :, P:] = torch.where(torch.from_numpy(masks), 0.0, float("-inf"))
    tm = br.extract_tree_masks_per_batch(add.cuda(), T, P + T)
    assert torch.equal(tm.cpu(), torch.from_numpy(masks))
    out = br._tree_dispatch(q.cuda(), k.cuda(), v.cuda(), add.cuda(), T, 16, 16, per_batch_trees=True)
    torch.cuda.synchronize()
    assert_close(out, _per_batch_oracle(q, k, v, masks, P), atol=ATOL)


def test_per_batch_rejects_bad_shapes_and_negative_mask_stride():
    B, Hq, Hkv, D, P, T = 2, 4, 2, 64, 16, 20
    q, k, v = (x.cuda() for x in make_inputs(34, B, Hq, Hkv, D, P, T))
    masks = torch.from_numpy(_masks(B, T, seed=1)).cuda()
    with pytest.raises(ValueError):
        br.run_tree_sparse_kernel_per_batch(q, k, v, masks[:1], block_m=16, block_n=16)  # batch mismatch
    with pytest.raises(ValueError):
        br.run_tree_sparse_kernel_per_batch(q, k, v, masks[0], block_m=16, block_n=16)  # 2-D
    out = torch.empty_like(q)
    a = nat.fwd_args(q, k, v, out, prefix_len=P, block_m=16, block_n=16)
    lib = nat.load_library()
    nbytes = ctypes.c_size_t()
    assert lib.tsfa_run_batched_workspace_bytes(ctypes.byref(a), ctypes.byref(nbytes)) == 0
    ws = torch.zeros(nbytes.value, dtype=torch.uint8, device="cuda")
    # a negative batch stride is refused before any launch
    st = lib.tsfa_run_tree_sparse_batched(ctypes.byref(a), masks[1].data_ptr(), nat.mask_dtype_code(masks), -T * T,
                                          T, ws.data_ptr(), ws.numel(), nat.stream_ptr(q.device))
    assert st == -1  # TSFA_ERR_VALUE


def test_per_batch_trees_with_row_tile_pairs():
    """The per-batch op on row-tile pairs (forced onto a small shape): each
    pair's two row tiles walk their own batch element's tree."""
    B, Hq, Hkv, D, P, T = 3, 32, 8, 128, 1500, 64
    q, k, v = make_inputs(33, B, Hq, Hkv, D, P, T)
    masks = _masks(B, T, seed=7)
    nat.force_row_pairs(True)
    try:
        out = br.run_tree_sparse_kernel_per_batch(q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(masks).cuda(),
                                                  block_m=32, block_n=32)
        torch.cuda.synchronize()
    finally:
        nat.force_row_pairs(False)
    assert nat.last_plan()["merge"] == "pair", nat.last_plan()
    assert nat.read_device_status(out.device) == 0
    from gpu_helpers import p_rounding_bound
    extra = np.concatenate([p_rounding_bound(q[b:b + 1], k[b:b + 1], v[b:b + 1], masks[b], P) for b in range(B)])
    assert_close(out, _per_batch_oracle(q, k, v, masks, P), extra=extra)
