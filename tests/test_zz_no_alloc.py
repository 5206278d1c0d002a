"""tsfa_run_tree_sparse_noalloc: the whole op over the library's own static
workspace, for callers that cannot allocate device memory (a plain C or FFI
host with no device allocator of its own, or a serving step loop where a
cudaMalloc would synchronise the device).

Called through the C ABI, it must give exactly what tsfa_run_tree_sparse gives
over a caller workspace -- the same kernels on the same inputs, so the outputs
are bit-identical (which is inside the parity tolerance of the other GPU
tests) -- on two calls in a row of each shape (the static sync block must be
left clean for the next call), match the fp32 oracle within that tolerance,
report its device status through tsfa_noalloc_read_device_status, and refuse
shapes that do not fit before launching anything.

Named to be collected last, so that a run stopping at its first failure has
run every other test first; it passes alone in a fresh process too (the first
call on the device does the static workspace's set-up)."""

import ctypes

import numpy as np
import pytest
import torch

import tsfa_native as nat
import tsfa_trees as trees
from gpu_helpers import assert_close, make_inputs, oracle

pytestmark = pytest.mark.gpu

CASES = [
    # (seed, B, Hq, Hkv, D, P, tree builder, block_m, block_n)
    (11, 1, 32, 8, 128, 4096, lambda: trees.random_tree(64, 6, 4, seed=3), 64, 64),
    (12, 2, 16, 4, 64, 700, lambda: trees.random_tree(200, 8, 6, seed=5), 32, 32),
]


def _inputs(seed, B, Hq, Hkv, D, P, tree):
    mask = tree()
    T = mask.shape[0]
    q, k, v = make_inputs(seed, B, Hq, Hkv, D, P, T)
    return (q, k, v, mask), tuple(x.cuda() for x in (q, k, v, torch.from_numpy(mask)))


def _noalloc(q, k, v, mask, out, bm, bn):
    """The entry point itself, through ctypes (no Python wrapper logic)."""
    a = nat.fwd_args(q, k, v, out, prefix_len=k.shape[2] - q.shape[2], block_m=bm, block_n=bn)
    return nat.load_library().tsfa_run_tree_sparse_noalloc(ctypes.byref(a), mask.data_ptr(), nat.mask_dtype_code(mask),
                                                          mask.stride(0), nat.stream_ptr(q.device))


def test_noalloc_matches_workspace_entry_on_consecutive_calls():
    runs = [_inputs(*c[:6], c[6]) + (c[7], c[8]) for c in CASES]
    want = []
    for _, (q, k, v, mask), bm, bn in runs:
        out = torch.empty_like(q)
        nat.run_tree_sparse(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2], block_m=bm, block_n=bn)
        want.append(out)
    torch.cuda.synchronize()
    for rep in range(2):  # two calls in a row on each shape, alternating shapes
        for (_, (q, k, v, mask), bm, bn), ref in zip(runs, want):
            out = torch.full_like(q, float("nan"))
            assert _noalloc(q, k, v, mask, out, bm, bn) == nat.TSFA_OK
            torch.cuda.synchronize()
            status = nat.noalloc_read_device_status(q.device)
            assert status[0] == nat.TSFA_OK, status
            assert torch.equal(out, ref), f"call {rep}: differs from tsfa_run_tree_sparse"
    # and the shared result against the fp32 oracle
    (q, k, v, mask), _, _, _ = runs[0]
    assert_close(want[0], oracle(q, k, v, np.asarray(mask), k.shape[2] - q.shape[2]))


def test_noalloc_device_status_is_readable_and_cleared():
    """A bounded wait that runs out (test fault, 1 ms limit) is reported by
    tsfa_noalloc_read_device_status, which clears the static sync block: the
    next call is correct."""
    _, (q, k, v, mask) = _inputs(*CASES[0][:6], CASES[0][6])
    ref = torch.empty_like(q)
    nat.run_tree_sparse(q, k, v, mask, ref, prefix_len=k.shape[2] - q.shape[2], block_m=64, block_n=64)
    out = torch.empty_like(q)
    try:
        nat.debug_inject(nat.FAULT_WITHHOLD_TREE_LIST, 1_000_000)
        assert _noalloc(q, k, v, mask, out, 64, 64) == nat.TSFA_OK
        torch.cuda.synchronize()
    finally:
        nat.debug_inject(nat.FAULT_NONE, 0)
    status = nat.noalloc_read_device_status(q.device)
    assert status[0] == nat.TSFA_ERR_DEVICE_TIMEOUT, status
    assert nat.noalloc_read_device_status(q.device)[0] == nat.TSFA_OK  # cleared
    assert _noalloc(q, k, v, mask, out, 64, 64) == nat.TSFA_OK
    torch.cuda.synchronize()
    assert nat.noalloc_read_device_status(q.device)[0] == nat.TSFA_OK
    assert torch.equal(out, ref)


def test_noalloc_rejects_oversized_shapes_before_launch():
    T, P = 8192, 128  # needs ~16 MiB of workspace at 64x64 tiles, more than the 8 MiB array
    q = torch.zeros((1, 8, T, 64), dtype=torch.bfloat16, device="cuda")
    k = torch.zeros((1, 8, P + T, 64), dtype=torch.bfloat16, device="cuda")
    mask = torch.ones((T, T), dtype=torch.bool, device="cuda")
    out = torch.empty_like(q)
    with pytest.raises(ValueError, match="static workspace holds"):
        nat.run_tree_sparse_noalloc(q, k, k, mask, out, prefix_len=P, block_m=64, block_n=64)
    # the C entry point itself answers TSFA_ERR_WORKSPACE for the same shapes
    assert _noalloc(q, k, k, mask, out, 64, 64) == nat.TSFA_ERR_WORKSPACE
