"""Data-parallel sharding over (batch, kv-head) units: the plan, the strided
views each rank computes on, and the gather -- on CPU with the fp32 oracle
standing in for the kernel, including world-size-2 gloo process groups --
plus a GPU check that the sharded native op matches the oracle."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import tsfa_oracle as orc
import tsfa_shard as shard
import tsfa_trees as trees


def _oracle_compute(q, k, v, mask, out):
    """CPU stand-in for the kernel on one set of views (dense + mask, fp32)."""
    P = k.shape[2] - q.shape[2]
    want = orc.dense_tree_attention(q.float().numpy(), k.float().numpy(), v.float().numpy(),
                                    np.asarray(mask.numpy(), bool), P)
    out.copy_(torch.from_numpy(want).to(out.dtype))


def _inputs(B, Hq, Hkv, D, P, T, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn((B, Hq, T, D), generator=g)
    k = torch.randn((B, Hkv, P + T, D), generator=g)
    v = torch.randn((B, Hkv, P + T, D), generator=g)
    mask = torch.from_numpy(trees.random_tree(T, 4, 3, seed=seed))
    return q, k, v, mask


@pytest.mark.parametrize("B,Hkv,world", [(1, 8, 1), (1, 8, 2), (1, 8, 8), (3, 2, 4), (16, 8, 8), (2, 3, 4), (1, 2, 3),
                                         (0, 4, 2)])
def test_plan_covers_every_unit_once_balanced(B, Hkv, world):
    seen = []
    sizes = []
    for r in range(world):
        p = shard.plan(B, Hkv, world, r)
        sizes.append(p.units)
        for b, h0, h1 in p.pieces():
            assert 0 <= b < B and 0 <= h0 < h1 <= Hkv
            seen += [b * Hkv + h for h in range(h0, h1)]
        assert sum(h1 - h0 for _, h0, h1 in p.pieces()) == p.units
    assert sorted(seen) == list(range(B * Hkv))
    assert max(sizes) - min(sizes) <= 1
    assert max(sizes) <= shard.max_units(B, Hkv, world)


def test_plan_rejects_bad_ranks():
    with pytest.raises(ValueError):
        shard.plan(1, 8, 2, 2)
    with pytest.raises(ValueError):
        shard.plan(1, 8, 0, 0)


@pytest.mark.parametrize("B,Hq,Hkv,world", [(1, 8, 4, 2), (3, 4, 2, 4), (2, 6, 3, 4)])
def test_shards_reassemble_the_full_op(B, Hq, Hkv, world):
    q, k, v, mask = _inputs(B, Hq, Hkv, 16, 24, 10)
    want = torch.empty_like(q)
    _oracle_compute(q, k, v, mask, want)
    out = torch.full_like(q, float("nan"))
    for r in range(world):
        shard.run_shard(q, k, v, mask, out, shard.plan(B, Hkv, world, r), compute=_oracle_compute)
    torch.testing.assert_close(out, want, rtol=0, atol=0)


@pytest.mark.parametrize("B,Hq,Hkv,world", [(3, 4, 2, 4), (2, 8, 4, 3)])
def test_shards_with_one_tree_per_batch_element(B, Hq, Hkv, world):
    q, k, v, _ = _inputs(B, Hq, Hkv, 16, 24, 10)
    masks = torch.from_numpy(np.stack([trees.random_tree(10, 4, 3, seed=30 + b) for b in range(B)]))
    want = torch.cat([_oracle_result(q[b:b + 1], k[b:b + 1], v[b:b + 1], masks[b]) for b in range(B)])
    out = torch.full_like(q, float("nan"))
    for r in range(world):
        shard.run_shard(q, k, v, masks, out, shard.plan(B, Hkv, world, r), compute=_oracle_compute)
    torch.testing.assert_close(out, want, rtol=0, atol=0)
    with pytest.raises(ValueError):
        shard.run_shard(q, k, v, masks[:1], out, shard.plan(B, Hkv, world, 0), compute=_oracle_compute)


def _oracle_result(q, k, v, mask):
    o = torch.empty_like(q)
    _oracle_compute(q, k, v, mask, o)
    return o


def test_shard_plan_must_match_inputs():
    q, k, v, mask = _inputs(1, 4, 2, 16, 8, 6)
    with pytest.raises(ValueError):
        shard.run_shard(q, k, v, mask, torch.empty_like(q), shard.plan(2, 2, 1, 0), compute=_oracle_compute)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_rank(rank, world, port, B, Hq, Hkv, results, per_batch=False):
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        q, k, v, mask = _inputs(B, Hq, Hkv, 16, 20, 9, seed=7)
        if per_batch:  # one tree per batch element
            mask = torch.from_numpy(np.stack([trees.random_tree(9, 4, 3, seed=40 + b) for b in range(B)]))
            want = torch.cat([_oracle_result(q[b:b + 1], k[b:b + 1], v[b:b + 1], mask[b]) for b in range(B)])
        else:
            want = _oracle_result(q, k, v, mask)
        out = shard.run_tree_sparse_sharded(q, k, v, mask, compute=_oracle_compute)
        results[rank] = float((out - want).abs().max())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B,Hq,Hkv,per_batch", [(1, 8, 4, False), (3, 4, 2, False), (1, 6, 3, False), (3, 4, 2, True)])
def test_gloo_world2_gather(B, Hq, Hkv, per_batch):
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, port, B, Hq, Hkv, results, per_batch))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert sorted(results.keys()) == [0, 1]
    assert all(v == 0.0 for v in results.values()), dict(results)


@pytest.mark.gpu
@pytest.mark.parametrize("world", [2, 4, 8])
def test_gpu_sharded_units_match_oracle(world):
    from gpu_helpers import ATOL, assert_close, make_inputs, oracle

    c = trees.CONFIGS["cfg2_llama3_8b"]
    mask = trees.config_tree(c, seed=0)
    q, k, v = make_inputs(3, 1, c["Hq"], c["Hkv"], c["D"], 512, c["T"])
    qd, kd, vd, md = (x.cuda() for x in (q, k, v, torch.from_numpy(mask)))
    out = torch.full_like(qd, float("nan"))
    for r in range(world):  # every rank's shard, one after another on this GPU
        shard.run_shard(qd, kd, vd, md, out, shard.plan(1, c["Hkv"], world, r))
    torch.cuda.synchronize()
    assert_close(out, oracle(q, k, v, mask, 512), atol=ATOL)


@pytest.mark.parametrize("B,Hkv,world", [(16, 8, 1), (16, 8, 2), (3, 2, 4), (2, 3, 4), (1, 8, 8), (5, 4, 3)])
def test_calls_cover_the_pieces_with_whole_rows_merged(B, Hkv, world):
    for r in range(world):
        p = shard.plan(B, Hkv, world, r)
        units = []
        for b0, b1, h0, h1 in p.calls():
            assert b1 > b0 and (b1 - b0 == 1 or (h0, h1) == (0, Hkv))
            units += [b * Hkv + h for b in range(b0, b1) for h in range(h0, h1)]
        assert units == list(range(p.unit_begin, p.unit_end))
    assert shard.plan(16, 8, 1, 0).calls() == [(0, 16, 0, 8)]
