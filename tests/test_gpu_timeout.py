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
whole op's thread-block-cluster merge, and the cooperative global merge of
tsfa_fwd over prebuilt metadata.  The reference has no device-side error path;
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


def _cfg(name, P=None):
    c = dict(trees.CONFIGS[name])
    if P is not None:
        c["P"] = P
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(21, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    return c, mask, q, k, v


def _whole_op(q, k, v, mask, bm, bn):
    out = torch.empty_like(q)
    nat.run_tree_sparse(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2], block_m=bm, block_n=bn)
    return out


def _prebuilt(q, k, v, mask, bm, bn):
    import tree_sparse_flashattn as tsfa

    meta = tsfa.prepare_tree_sparse_metadata(mask, k.shape[2] - q.shape[2], bm, bn)
    out = torch.empty_like(q)
    nat.fwd_with_metadata(q, k, v, out, meta, prefix_len=k.shape[2] - q.shape[2])
    return out


CASES = [
    # (id, config, prefix override, call): a single-split launch (T = 64,
    # P = 0: one key tile), the whole op (cluster merge at config 2) and
    # tsfa_fwd over prebuilt metadata (global merge)
    ("no-merge", "cfg2_llama3_8b", 0, _whole_op),
    ("cluster-merge", "cfg2_llama3_8b", None, _whole_op),
    ("global-merge", "cfg2_llama3_8b", None, _prebuilt),
]


@pytest.mark.parametrize("cid,name,P,call", CASES, ids=[c[0] for c in CASES])
def test_wait_runs_out_then_next_call_is_correct(cid, name, P, call):
    c, mask, q, k, v = _cfg(name, P)
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
    assert nat.read_device_status(dev) == 0
    assert_close(out, oracle(q, k, v, mask, c["P"]))
