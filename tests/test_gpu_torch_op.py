"""torch.ops.tsfa.* on the GPU: the dispatcher op behind run_tree_sparse_kernel
(bridge.py:76-159) gives exactly the C ABI's answer, passes torch's operator
checks (schema, fake tensor, AOT dispatch), compiles with torch.compile with
no graph break and gives the eager result, and the metadata op's first nnz
entries are the reference's metadata."""

import numpy as np
import pytest
import torch

import tsfa_native as nat
import tsfa_trees as trees
from conftest import load_npz
from gpu_helpers import assert_close, make_inputs, oracle

pytestmark = pytest.mark.gpu


def _cfg2():
    c = trees.CONFIGS["cfg2_llama3_8b"]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(41, c["B"], c["Hq"], c["Hkv"], c["D"], c["P"], c["T"])
    return c, mask, q, k, v


def test_op_equals_c_abi_and_oracle():
    ops = nat.load_torch_op()
    c, mask, q, k, v = _cfg2()
    qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))
    got = ops.run_tree_sparse(qd, kd, vd, md, c["P"], 64, 64, c["D"] ** -0.5)
    ref = torch.empty_like(qd)
    nat.run_tree_sparse(qd, kd, vd, md, ref, prefix_len=c["P"], block_m=64, block_n=64)
    torch.cuda.synchronize()
    assert nat.read_device_status(qd.device) == 0
    assert torch.equal(got, ref)
    assert_close(got, oracle(q, k, v, mask, c["P"]))


def test_opcheck():
    ops = nat.load_torch_op()
    c, mask, q, k, v = _cfg2()
    args = (q.cuda(), k.cuda(), v.cuda(), torch.from_numpy(mask).cuda(), c["P"], 64, 64, c["D"] ** -0.5)
    torch.library.opcheck(ops.run_tree_sparse.default, args,
                          test_utils=("test_schema", "test_faketensor", "test_aot_dispatch_static"))
    torch.library.opcheck(ops.build_metadata.default, (args[3], 16, 16),
                          test_utils=("test_schema", "test_faketensor"))


def test_torch_compile_fullgraph_no_graph_break():
    import eagle_tree_sparse_bridge as br

    c, mask, q, k, v = _cfg2()
    qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))

    def verify_step(q, k, v, m):
        return br.run_tree_sparse_kernel(q, k, v, m, block_m=64, block_n=64) * 1.0

    torch._dynamo.reset()
    explain = torch._dynamo.explain(verify_step)(qd, kd, vd, md)
    assert explain.graph_break_count == 0 and explain.graph_count == 1, explain.break_reasons
    compiled = torch.compile(verify_step, fullgraph=True)
    got = compiled(qd, kd, vd, md)
    eager = verify_step(qd, kd, vd, md)
    torch.cuda.synchronize()
    assert torch.equal(got, eager)


def test_metadata_op_matches_golden(meta_golden):
    ops = nat.load_torch_op()
    for cid in [str(x) for x in meta_golden["__ids__"]][:12]:
        mask = torch.from_numpy(np.ascontiguousarray(meta_golden[f"{cid}.mask"])).cuda()
        bm, bn, _ = (int(x) for x in meta_golden[f"{cid}.params"][:3])
        rp, col, typ, pay, off, cnt = ops.build_metadata(mask, bm, bn)
        nnz, n_mixed = (int(x) for x in cnt.tolist())
        W = -(-bm * bn // 32)
        got = {"row_ptr": rp, "col_idx": col[:nnz], "blk_type": typ[:nnz], "mixed_mask_payload": pay[:n_mixed * W],
               "mixed_mask_offset": off[:nnz if n_mixed else 0]}
        for f, t in got.items():
            assert np.array_equal(t.cpu().numpy(), meta_golden[f"{cid}.{f}"]), (cid, f)
