"""The (batch, kv-head) split on several GPUs: one process per GPU with an NCCL
process group, each rank running the native op on its units (tsfa_shard), then
the NCCL all-gather of the output shards.

Checked on every rank:
* its shard is bit-identical to the same shard call run on GPU 0 alone -- the
  same kernel on the same views (each rank saves its shard; the parent
  compares against single-GPU runs of every rank's plan);
* the gathered output is complete and within the parity tolerance of the
  fp32 oracle.

Configurations: config 2's eight kv-heads over 2 ranks (strong scaling of one
problem) and config 3's 128 (batch, kv-head) units over 2 ranks.  Skipped with
fewer than two GPUs.  The reference has no multi-GPU path; this is the split
the benchmark's multi-GPU runs measure.
"""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import tsfa_shard as shard
import tsfa_trees as trees

pytestmark = pytest.mark.gpu

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs(name, P=None):
    c = dict(trees.CONFIGS[name])
    if P is not None:
        c["P"] = P
    mask = trees.config_tree(c, seed=0)
    g = torch.Generator().manual_seed(77)
    q = torch.randn((c["B"], c["Hq"], c["T"], c["D"]), generator=g).to(torch.bfloat16)
    k = torch.randn((c["B"], c["Hkv"], c["P"] + c["T"], c["D"]), generator=g).to(torch.bfloat16)
    v = torch.randn((c["B"], c["Hkv"], c["P"] + c["T"], c["D"]), generator=g).to(torch.bfloat16)
    return c, mask, q, k, v


def _rank(rank, world, port, name, P, outdir):
    import datetime

    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        c, mask, q, k, v = _inputs(name, P)
        qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))
        plan = shard.plan(c["B"], c["Hkv"], world, rank)
        out = torch.full_like(qd, float("nan"))
        shard.run_shard(qd, kd, vd, md, out, plan, block_m=c["BM"], block_n=c["BN"])
        torch.cuda.synchronize()
        torch.save({"pieces": plan.pieces(), "out": out.cpu()}, os.path.join(outdir, f"rank{rank}.pt"))
        shard.gather(out, plan)
        torch.cuda.synchronize()
        torch.save(out.cpu(), os.path.join(outdir, f"gathered{rank}.pt"))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < WORLD, reason="needs two GPUs")
@pytest.mark.parametrize("name,P", [("cfg2_llama3_8b", None), ("cfg3_serving_70b", 1024)])
def test_two_gpu_shards_are_bit_identical_and_gather(tmp_path, name, P):
    from gpu_helpers import assert_close, oracle

    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, WORLD, port, name, P, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]

    c, mask, q, k, v = _inputs(name, P)
    G = c["Hq"] // c["Hkv"]
    qd, kd, vd, md = (x.cuda(0) for x in (q, k, v, torch.from_numpy(mask)))
    for r in range(WORLD):
        saved = torch.load(os.path.join(tmp_path, f"rank{r}.pt"))
        # the same shard call on GPU 0 alone
        plan = shard.plan(c["B"], c["Hkv"], WORLD, r)
        alone = torch.full_like(qd, float("nan"))
        shard.run_shard(qd, kd, vd, md, alone, plan, block_m=c["BM"], block_n=c["BN"])
        torch.cuda.synchronize()
        for b, h0, h1 in plan.pieces():
            got = saved["out"][b, h0 * G:h1 * G]
            assert torch.equal(got, alone[b, h0 * G:h1 * G].cpu()), (r, b, h0, h1)
        gathered = torch.load(os.path.join(tmp_path, f"gathered{r}.pt"))
        assert not torch.isnan(gathered).any()
        # the gathered output (batch 0) within the parity bound of the oracle
        assert_close(gathered[0:1], oracle(q[0:1], k[0:1], v[0:1], mask, c["P"]))
