"""Failure detection on the GPU without a fault: a bounded device wait runs out.

The forward's waits are bounded in wall time.  tsfa_debug_inject shortens the
limit to 1 ms for this thread's launches and makes the tree-list warp withhold
its list (a flag that nothing then sets), so the producer's, the MMA issuer's
and the softmax threads' waits on it run out.  The kernel must wind down (its
own copies land, issued MMAs complete, TMEM is freed), leave
TSFA_ERR_DEVICE_TIMEOUT with the site of a list wait in the workspace status
block, and leave the context and the workspace usable: the next normal call on
the same stream and workspace gives the oracle's answer with status 0.

Each split-merge variant of the forward is covered: one split (no merge), the
global merge through L2 (the whole op, the paged op and tsfa_fwd over
prebuilt metadata) and the thread-block-cluster merge (the whole op and the
paged op, forced onto it).  The reference has no device-side error path;
its host-side checks (tree_sparse_flashattn.py:85-88,
eagle_tree_sparse_bridge.py:85-93) map to the status codes tested elsewhere.
"""

import pytest
import torch

import tsfa_native as nat
import tsfa_trees as trees
from gpu_helpers import assert_close, make_inputs, oracle

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms instead of 1 s
# wait sites (csrc/tsfa_fwd_tc.cu WaitSite): the producer's, the MMA issuer's
# and the softmax threads' waits on the tree list; a CTA of the global merge
# may instead first give up waiting for a split that aborted
LIST_SITES = {1, 4, 12}
MERGE_SITE = 13


@pytest.fixture(autouse=True)
def _restore_defaults():
    yield
    nat.debug_inject(nat.FAULT_NONE, 0)


def _cfg(name, P=None, B=None):
    c = dict(trees.CONFIGS[name])
    if P is not None:
        c["P"] = P
    if B is not None:
        c["B"] = B
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(21, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    return c, mask, q, k, v


def _whole_op(q, k, v, mask, bm, bn):
    out = torch.empty_like(q)
    nat.run_tree_sparse(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2], block_m=bm, block_n=bn)
    return out


def _paged_op(q, k, v, mask, bm, bn):
    """The whole op over a paged copy of K/V (pages of 64 keys, in order):
    the paged op merges its splits through thread-block clusters."""
    B, Hkv, KV, D = k.shape
    per = -(-KV // 64)
    kp = torch.zeros((B * per, 64, Hkv, D), dtype=k.dtype, device=k.device)
    vp = torch.zeros_like(kp)
    for b in range(B):
        for i in range(per):
            lo, hi = i * 64, min(KV, (i + 1) * 64)
            kp[b * per + i, :hi - lo] = k[b, :, lo:hi].transpose(0, 1)
            vp[b * per + i, :hi - lo] = v[b, :, lo:hi].transpose(0, 1)
    indptr = torch.arange(0, B * per + 1, per, dtype=torch.int32, device=k.device)
    indices = torch.arange(B * per, dtype=torch.int32, device=k.device)
    out = torch.empty_like(q)
    nat.run_tree_sparse_paged(q, kp, vp, indptr, indices, mask, out, kv_len=KV, prefix_len=KV - q.shape[2],
                              block_m=bm, block_n=bn)
    return out


def _clustered(call):
    """The same call with its forward forced onto the thread-block-cluster merge."""
    def run(*a):
        nat.force_cluster_merge(True)
        try:
            return call(*a)
        finally:
            nat.force_cluster_merge(False)
    return run


def _prebuilt(q, k, v, mask, bm, bn):
    import tree_sparse_flashattn as tsfa

    meta = tsfa.prepare_tree_sparse_metadata(mask, k.shape[2] - q.shape[2], bm, bn)
    out = torch.empty_like(q)
    nat.fwd_with_metadata(q, k, v, out, meta, prefix_len=k.shape[2] - q.shape[2])
    return out


CASES = [
    # (id, config, prefix override, batch override, call, merge the launch must use):
    # a single-split launch (T = 64, P = 0: one key tile); config 2 through
    # the whole op, the paged op and tsfa_fwd over prebuilt metadata (global
    # merge through L2), and through the whole op and the paged op forced onto
    # the thread-block-cluster merge
    ("no-merge", "cfg2_llama3_8b", 0, 1, _whole_op, "none"),
    ("global-merge-op", "cfg2_llama3_8b", None, 1, _whole_op, "global"),
    ("global-merge-paged", "cfg2_llama3_8b", None, 1, _paged_op, "global"),
    ("global-merge-fwd", "cfg2_llama3_8b", None, 1, _prebuilt, "global"),
    ("cluster-merge-op", "cfg2_llama3_8b", None, 1, _clustered(_whole_op), "cluster"),
    ("cluster-merge-paged", "cfg2_llama3_8b", None, 1, _clustered(_paged_op), "cluster"),
]


@pytest.mark.parametrize("cid,name,P,B,call,merge", CASES, ids=[c[0] for c in CASES])
def test_wait_runs_out_then_next_call_is_correct(cid, name, P, B, call, merge):
    c, mask, q, k, v = _cfg(name, P, B)
    qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))
    dev = qd.device
    assert nat.read_device_status(dev) == 0

    nat.debug_inject(nat.FAULT_WITHHOLD_TREE_LIST, LIMIT_NS)
    call(qd, kd, vd, md, c["BM"], c["BN"])
    torch.cuda.synchronize()
    nat.debug_inject(nat.FAULT_NONE, 0)
    status, site, tile, cta = nat.read_device_status_detail(dev)  # reads, then clears the sync block
    assert status == nat.TSFA_ERR_DEVICE_TIMEOUT, (status, site, tile, cta)
    assert site in LIST_SITES | {MERGE_SITE}, site
    assert 0 <= cta < 148 * 16
    # the context and the stream are usable
    assert float(torch.ones(4, device=dev).sum()) == 4.0

    out = call(qd, kd, vd, md, c["BM"], c["BN"])
    torch.cuda.synchronize()
    assert nat.last_plan()["merge"] == merge, nat.last_plan()
    assert nat.read_device_status(dev) == 0
    assert_close(out, oracle(q, k, v, mask, c["P"]))


@pytest.mark.parametrize("call", [_whole_op, _prebuilt], ids=["op", "prebuilt"])
def test_refused_cooperative_launch_falls_back_to_clusters(call):
    """Where the device refuses the global merge's cooperative launch (another
    context holding SMs), the forward falls back to the cluster merge.  The
    refusal is injected on the host (nothing is launched for it): the call
    must still succeed, merge through clusters and match the oracle."""
    c, mask, q, k, v = _cfg("cfg2_llama3_8b")
    qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))
    nat.debug_inject(nat.FAULT_REFUSE_COOPERATIVE, 0)
    try:
        out = call(qd, kd, vd, md, c["BM"], c["BN"])
        torch.cuda.synchronize()
        plan = nat.last_plan()
    finally:
        nat.debug_inject(nat.FAULT_NONE, 0)
    assert plan["merge"] == "cluster", plan
    assert nat.read_device_status(qd.device) == 0
    assert_close(out, oracle(q, k, v, mask, c["P"]))
    # and without the fault the same call merges through L2 again
    call(qd, kd, vd, md, c["BM"], c["BN"])
    torch.cuda.synchronize()
    assert nat.last_plan()["merge"] == "global", nat.last_plan()
