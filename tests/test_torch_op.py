"""The PyTorch operator binding (libtsfa_torch.so, torch.ops.tsfa.*) on the
CPU: it loads without a GPU, registers the schemas, and its Meta kernels give
the output shapes, so fake-tensor tracing (what torch.compile runs before
compiling) sees run_tree_sparse_kernel (bridge.py:76-159) as one op."""

import pytest
import torch

import tsfa_native as nat


@pytest.fixture(scope="module")
def ops():
    return nat.load_torch_op()


def test_schemas(ops):
    assert str(ops.run_tree_sparse.default._schema) == (
        "tsfa::run_tree_sparse(Tensor q, Tensor k, Tensor v, Tensor tree_mask, int prefix_len, int block_m, "
        "int block_n, float sm_scale) -> Tensor")
    assert str(ops.build_metadata.default._schema).startswith("tsfa::build_metadata(Tensor tree_mask, int block_m")


@pytest.mark.parametrize("T,bm,bn", [(64, 64, 64), (100, 16, 32), (1024, 16, 16)])
def test_fake_tensor_shapes(ops, T, bm, bn):
    from torch._subclasses.fake_tensor import FakeTensorMode

    with FakeTensorMode():
        q = torch.empty(2, 32, T, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(2, 8, 512 + T, 128, dtype=torch.bfloat16, device="cuda")
        m = torch.empty(T, T, dtype=torch.bool, device="cuda")
        o = ops.run_tree_sparse(q, k, k, m, 512, bm, bn, 128 ** -0.5)
        assert o.shape == q.shape and o.dtype == q.dtype and o.is_contiguous() and o.device.type == "cuda"
        rp, col, typ, pay, off, cnt = ops.build_metadata(m, bm, bn)
    d = nat.meta_dims(T, bm, bn)
    assert rp.shape == (d.n_q_blocks + 1,) and col.shape == (d.tile_capacity,) and typ.dtype == torch.int8
    assert pay.shape == (d.payload_capacity,) and off.shape == (d.tile_capacity,) and cnt.shape == (2,)


def test_bridge_traces_to_one_op(ops):
    """make_fx with fake tensors over the public entry point: the graph holds
    the one tsfa op (plus nothing that touches the inputs' data)."""
    from torch.fx.experimental.proxy_tensor import make_fx
    from torch._subclasses.fake_tensor import FakeTensorMode

    import eagle_tree_sparse_bridge as br

    def fn(q, k, v, m):
        return br.run_tree_sparse_kernel(q, k, v, m, block_m=64, block_n=64)

    with FakeTensorMode():
        q = torch.empty(1, 32, 64, 128, dtype=torch.bfloat16, device="cuda")
        k = torch.empty(1, 8, 4160, 128, dtype=torch.bfloat16, device="cuda")
        m = torch.empty(64, 64, dtype=torch.bool, device="cuda")
        gm = make_fx(fn, tracing_mode="fake")(q, k, k, m)
    targets = [n.target for n in gm.graph.nodes if n.op == "call_function"]
    assert targets.count(torch.ops.tsfa.run_tree_sparse.default) == 1, targets


def test_bridge_compiles_fullgraph(ops):
    """torch.compile(fullgraph=True) over the public entry point traces with
    no graph break (meta tensors stand in for CUDA ones: the CUDA-device
    assertion of the entry point is the only line that differs)."""
    import inspect

    import eagle_tree_sparse_bridge as br

    src = inspect.getsource(br.run_tree_sparse_kernel).replace(
        "assert query_states.is_cuda and key_states.is_cuda and value_states.is_cuda", "pass")
    ns = dict(br.__dict__)
    exec(src, ns)
    fn = ns["run_tree_sparse_kernel"]

    def verify_step(q, k, v, m):
        return fn(q, k, v, m, block_m=64, block_n=64) * 1.0

    q = torch.empty(1, 32, 64, 128, dtype=torch.bfloat16, device="meta")
    k = torch.empty(1, 8, 4160, 128, dtype=torch.bfloat16, device="meta")
    m = torch.empty(64, 64, dtype=torch.bool, device="meta")
    torch._dynamo.reset()
    out = torch.compile(verify_step, backend="eager", fullgraph=True)(q, k, k, m)
    assert out.shape == q.shape

