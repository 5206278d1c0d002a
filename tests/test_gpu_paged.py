"""Paged K/V cache: tsfa_run_tree_sparse_paged through the bridge's
run_tree_sparse_kernel_paged must give exactly what the contiguous-K/V op
gives on the same keys (the kernel reads the same rows into the same tiles),
for page sizes below, at and above the 128-key tile, shuffled page order,
a last page only partly used and stale NaN in every unused slot and page,
FlashInfer's interleaved [pages, 2, page_size, Hkv, D] layout and separate
pools.  No reference counterpart (the reference takes contiguous K/V)."""

import numpy as np
import pytest
import torch

import eagle_tree_sparse_bridge as br
import tsfa_native as nat
import tsfa_trees as trees
from gpu_helpers import ATOL, assert_close, make_inputs, oracle

pytestmark = pytest.mark.gpu


def _paged(k, v, page_size, interleaved, seed):
    """Pages of k / v ([B, Hkv, KV, D]) in shuffled order, NaN elsewhere."""
    B, Hkv, KV, D = k.shape
    per = -(-KV // page_size)
    n_pages = B * per + 3  # spare pages nobody uses
    order = torch.randperm(n_pages, generator=torch.Generator().manual_seed(seed))[:B * per]
    if interleaved:
        cache = torch.full((n_pages, 2, page_size, Hkv, D), float("nan"), dtype=k.dtype, device=k.device)
        kp, vp = cache[:, 0], cache[:, 1]
    else:
        kp = torch.full((n_pages, page_size, Hkv, D), float("nan"), dtype=k.dtype, device=k.device)
        vp = torch.full_like(kp, float("nan"))
    for b in range(B):
        for i in range(per):
            pg = int(order[b * per + i])
            lo, hi = i * page_size, min(KV, (i + 1) * page_size)
            kp[pg, :hi - lo] = k[b, :, lo:hi].transpose(0, 1)
            vp[pg, :hi - lo] = v[b, :, lo:hi].transpose(0, 1)
    indptr = torch.arange(0, B * per + 1, per, dtype=torch.int32, device=k.device)
    return kp, vp, indptr, order.to(torch.int32).to(k.device)


@pytest.mark.parametrize("page_size,interleaved", [(16, True), (8, False), (64, False), (128, True), (256, False)])
@pytest.mark.parametrize("B,Hq,Hkv,D,P,T", [(2, 8, 2, 128, 100, 40), (1, 32, 8, 128, 4096, 64), (3, 4, 4, 64, 0, 24)])
def test_paged_equals_contiguous(page_size, interleaved, B, Hq, Hkv, D, P, T):
    q, k, v = (x.cuda() for x in make_inputs(41, B, Hq, Hkv, D, P, T))
    mask = torch.from_numpy(trees.random_tree(T, 5, 3, seed=4)).cuda()
    kp, vp, indptr, idx = _paged(k, v, page_size, interleaved, seed=page_size + B)
    want = br.run_tree_sparse_kernel(q, k, v, mask, block_m=16, block_n=16)
    got = br.run_tree_sparse_kernel_paged(q, kp, vp, indptr, idx, mask, kv_len=P + T, block_m=16, block_n=16)
    torch.cuda.synchronize()
    assert nat.read_device_status(q.device) == 0
    assert torch.equal(got.isnan(), want.isnan())
    ok = ~want.isnan()
    assert torch.equal(got[ok], want[ok])


def test_paged_matches_oracle_with_a_short_page_list():
    """A page list one page short of kv_len: the missing keys read as zeros,
    as if K and V rows were zero there."""
    B, Hq, Hkv, D, P, T, ps = 1, 8, 2, 128, 200, 40, 16
    q, k, v = make_inputs(42, B, Hq, Hkv, D, P, T)
    mask = trees.random_tree(T, 5, 3, seed=6)
    kp, vp, indptr, idx = _paged(k.cuda(), v.cuda(), ps, False, seed=1)
    per = int(indptr[1])
    indptr_short = torch.tensor([0, per - 1], dtype=torch.int32, device="cuda")
    got = br.run_tree_sparse_kernel_paged(q.cuda(), kp, vp, indptr_short, idx, torch.from_numpy(mask).cuda(),
                                          kv_len=P + T, block_m=16, block_n=16)
    torch.cuda.synchronize()
    k0, v0 = k.clone(), v.clone()
    k0[:, :, (per - 1) * ps:] = 0
    v0[:, :, (per - 1) * ps:] = 0
    assert_close(got, oracle(q, k0, v0, mask, P), atol=ATOL)


def test_paged_rejects_bad_page_sizes():
    B, Hq, Hkv, D, P, T = 1, 4, 2, 64, 32, 16
    q, k, v = (x.cuda() for x in make_inputs(43, B, Hq, Hkv, D, P, T))
    mask = torch.from_numpy(trees.random_tree(T, 4, 3, seed=2)).cuda()
    kp, vp, indptr, idx = _paged(k, v, 16, False, seed=3)
    with pytest.raises(NotImplementedError):  # 12 is not a power of two
        br.run_tree_sparse_kernel_paged(q, kp[:, :12], vp[:, :12], indptr, idx, mask, kv_len=P + T, block_m=16,
                                        block_n=16)
    with pytest.raises(ValueError):
        br.run_tree_sparse_kernel_paged(q, kp, vp, indptr, idx, mask, kv_len=T - 1, block_m=16, block_n=16)
