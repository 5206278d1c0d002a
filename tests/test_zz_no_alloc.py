"""tsfa_run_tree_sparse_noalloc: the whole op over the library's static
workspace must give what tsfa_run_tree_sparse gives over a caller workspace
(within the parity tolerance), on consecutive calls (the sync block must be
left clean for the next call), and must refuse shapes that do not fit before
launching anything.

Named to be collected last, so it also runs after every other GPU test has
used the library on this device."""

import pytest
import torch

import tsfa_native as nat
import tsfa_trees as trees
from gpu_helpers import ATOL, make_inputs

pytestmark = pytest.mark.gpu

CASES = [
    # (seed, B, Hq, Hkv, D, P, tree builder, block_m, block_n)
    (11, 1, 32, 8, 128, 4096, lambda: trees.random_tree(64, 6, 4, seed=3), 64, 64),
    (12, 2, 16, 4, 64, 700, lambda: trees.random_tree(200, 8, 6, seed=5), 32, 32),
]


def _inputs(seed, B, Hq, Hkv, D, P, tree):
    mask = torch.as_tensor(tree())
    T = mask.shape[0]
    q, k, v = (x.cuda() for x in make_inputs(seed, B, Hq, Hkv, D, P, T))
    return q, k, v, mask.cuda()


def test_noalloc_matches_workspace_entry_on_consecutive_calls():
    runs = [_inputs(*c[:6], c[6]) + c[7:] for c in CASES]
    want = []
    for q, k, v, mask, bm, bn in runs:
        out = torch.empty_like(q)
        nat.run_tree_sparse(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2], block_m=bm, block_n=bn)
        want.append(out)
    torch.cuda.synchronize()
    for rep in range(2):  # two calls in a row on each shape, alternating shapes
        for (q, k, v, mask, bm, bn), ref in zip(runs, want):
            out = torch.full_like(q, float("nan"))
            nat.run_tree_sparse_noalloc(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2],
                                        block_m=bm, block_n=bn)
            torch.cuda.synchronize()
            # Same op over another workspace: equal within the parity tolerance.
            assert torch.equal(out.isnan(), ref.isnan())
            ok = ~ref.isnan()
            err = (out[ok].float() - ref[ok].float()).abs()
            tol = ATOL + 2.0 ** -8 * ref[ok].float().abs()
            assert bool((err <= tol).all()), f"call {rep}: max |diff| {float(err.max()):.3e} from tsfa_run_tree_sparse"


def test_noalloc_rejects_oversized_shapes_before_launch():
    T, P = 4096, 128  # needs ~4.2 MB of workspace at 64x64 tiles, more than the 2 MiB array
    q = torch.zeros((1, 8, T, 64), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((1, 8, P + T, 64), dtype=torch.bfloat16, device="cuda")
    mask = torch.ones((T, T), dtype=torch.bool, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(ValueError, match="static workspace holds"):
        nat.run_tree_sparse_noalloc(q, k, k, mask, out, prefix_len=P, block_m=64, block_n=64)
    # the C entry point itself answers TSFA_ERR_WORKSPACE for the same shapes
    import ctypes
    a = nat.fwd_args(q, k, k, out, prefix_len=P, block_m=64, block_n=64)
    st = nat.load_library().tsfa_run_tree_sparse_noalloc(ctypes.byref(a), mask.data_ptr(), nat.mask_dtype_code(mask),
                                                        T, nat.stream_ptr(q.device))
    assert st == nat.TSFA_ERR_WORKSPACE
