"""Data-parallel sharding of the verify-step attention over the GPUs of a node.

The independent unit of ``run_tree_sparse_kernel`` (bridge.py:76-159) is one
(batch b, kv-head h) pair: it owns query heads ``[h*G, (h+1)*G)``, its own K/V
slice and its own output slice, and shares only the tree mask (bridge.py:57-58
uses batch 0's tree for every batch).  The ``B * Hkv`` units are flattened
(``u = b * Hkv + h``) and dealt out in contiguous, balanced ranges, one per
rank.  Each rank runs the kernel on strided views of its units -- one call per
batch row its range touches -- so the forward needs no collective.  An
optional gather (``torch.distributed.all_gather`` on the process group: NCCL
over NVLink on GPUs, gloo on CPU) assembles the full output on every rank.

The reference has no multi-GPU path; this module is the data-parallel layer
around the single-GPU op.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Tuple

import torch


@dataclass(frozen=True)
class ShardPlan:
    """Units [unit_begin, unit_end) of ``world`` ranks' flattened (b, kv-head) grid."""

    batch: int
    num_kv_heads: int
    world: int
    rank: int
    unit_begin: int
    unit_end: int

    @property
    def units(self) -> int:
        return self.unit_end - self.unit_begin

    def pieces(self) -> List[Tuple[int, int, int]]:
        """(b, h0, h1): the kv-head ranges of each batch row this shard touches."""
        out = []
        u = self.unit_begin
        while u < self.unit_end:
            b, h0 = divmod(u, self.num_kv_heads)
            h1 = min(self.num_kv_heads, h0 + (self.unit_end - u))
            out.append((b, h0, h1))
            u += h1 - h0
        return out

    def calls(self) -> List[Tuple[int, int, int, int]]:
        """(b0, b1, h0, h1): the op calls this shard makes with one tree for
        every batch element -- a run of whole batch rows is one call over the
        batch slice [b0, b1), a partial row one call of its own."""
        out: List[Tuple[int, int, int, int]] = []
        H = self.num_kv_heads
        for b, h0, h1 in self.pieces():
            whole = h0 == 0 and h1 == H
            if whole and out and out[-1][2] == 0 and out[-1][3] == H and out[-1][1] == b:
                out[-1] = (out[-1][0], b + 1, 0, H)
            else:
                out.append((b, b + 1, h0, h1))
        return out


def plan(batch: int, num_kv_heads: int, world: int, rank: int) -> ShardPlan:
    """Balanced contiguous split of ``batch * num_kv_heads`` units over ``world`` ranks."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} out of range for world size {world}")
    if batch < 0 or num_kv_heads <= 0:
        raise ValueError("batch must be >= 0 and num_kv_heads > 0")
    n = batch * num_kv_heads
    begin = rank * n // world
    end = (rank + 1) * n // world
    return ShardPlan(batch, num_kv_heads, world, rank, begin, end)


def max_units(batch: int, num_kv_heads: int, world: int) -> int:
    n = batch * num_kv_heads
    return -(-n // world) if world else 0


Compute = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], None]


def _native_compute(block_m: int, block_n: int) -> Compute:
    import tsfa_native as native

    def run(q, k, v, mask, out):
        native.run_tree_sparse(q, k, v, mask, out, prefix_len=k.shape[2] - q.shape[2], block_m=block_m,
                               block_n=block_n)

    return run


def run_shard(query_states: torch.Tensor, key_states: torch.Tensor, value_states: torch.Tensor,
              tree_mask: torch.Tensor, out: torch.Tensor, shard: ShardPlan, *, block_m: int = 64,
              block_n: int = 64, compute: Optional[Compute] = None) -> torch.Tensor:
    """Fill ``out``'s slices for this shard's units (views, no copies of K/V).

    ``tree_mask`` is one [T, T] tree for every batch element (the reference's
    case: a run of whole batch rows is then one call) or [B, T, T], one tree
    per batch element: every piece is one batch row, so it gets that row's
    tree.  ``compute(q, k, v, mask, out)`` runs the
    op on one set of views; the default is the native kernel
    (``tsfa_run_tree_sparse``).  Tests pass a CPU stand-in to check the plan
    and the views on hosts without a GPU.
    """
    B, Hq, T, D = query_states.shape
    Hkv = key_states.shape[1]
    if Hq % Hkv != 0:
        raise AssertionError("num_heads must be a multiple of num_key_value_heads")
    if (shard.batch, shard.num_kv_heads) != (B, Hkv):
        raise ValueError("shard plan does not match the inputs' batch / kv-head shape")
    G = Hq // Hkv
    per_batch = tree_mask.dim() == 3
    if per_batch and tree_mask.shape[0] != B:
        raise ValueError(f"tree_mask has {tree_mask.shape[0]} trees for a batch of {B}")
    fn = compute or _native_compute(block_m, block_n)
    if per_batch:
        for b, h0, h1 in shard.pieces():
            fn(query_states[b:b + 1, h0 * G:h1 * G], key_states[b:b + 1, h0:h1], value_states[b:b + 1, h0:h1],
               tree_mask[b], out[b:b + 1, h0 * G:h1 * G])
        return out
    for b0, b1, h0, h1 in shard.calls():  # whole batch rows in one call
        fn(query_states[b0:b1, h0 * G:h1 * G], key_states[b0:b1, h0:h1], value_states[b0:b1, h0:h1], tree_mask,
           out[b0:b1, h0 * G:h1 * G])
    return out


def _pack(out: torch.Tensor, shard: ShardPlan, G: int, cap: int) -> torch.Tensor:
    """This shard's output rows as [cap, G, T, D] (unit-major, zero padded)."""
    _, _, T, D = out.shape
    buf = out.new_zeros((cap, G, T, D))
    i = 0
    for b, h0, h1 in shard.pieces():
        n = h1 - h0
        buf[i:i + n] = out[b, h0 * G:h1 * G].reshape(n, G, T, D)
        i += n
    return buf


def gather(out: torch.Tensor, shard: ShardPlan, group=None) -> torch.Tensor:
    """All-gather every rank's slices into a full ``out`` on every rank."""
    import torch.distributed as dist

    B, Hq, T, D = out.shape
    G = Hq // shard.num_kv_heads
    cap = max_units(shard.batch, shard.num_kv_heads, shard.world)
    mine = _pack(out, shard, G, cap)
    parts = [torch.empty_like(mine) for _ in range(shard.world)]
    dist.all_gather(parts, mine, group=group)
    flat = out.view(B * shard.num_kv_heads, G, T, D) if out.is_contiguous() else None
    for r, part in enumerate(parts):
        p = plan(shard.batch, shard.num_kv_heads, shard.world, r)
        if flat is not None:
            flat[p.unit_begin:p.unit_end] = part[:p.units]
        else:
            i = 0
            for b, h0, h1 in p.pieces():
                n = h1 - h0
                out[b, h0 * G:h1 * G] = part[i:i + n].reshape(n * G, T, D)
                i += n
    return out


def run_tree_sparse_sharded(query_states: torch.Tensor, key_states: torch.Tensor, value_states: torch.Tensor,
                            tree_mask: torch.Tensor, *, block_m: int = 64, block_n: int = 64,
                            rank: Optional[int] = None, world: Optional[int] = None, group=None,
                            gather_output: bool = True, compute: Optional[Compute] = None) -> torch.Tensor:
    """``run_tree_sparse_kernel`` with its (batch, kv-head) units split over the ranks.

    Every rank holds the full inputs (or at least its units' slices) and
    returns a full-size output: its own units computed locally, the others'
    filled in by the gather (or left unwritten when ``gather_output`` is
    False).  With world size 1 this is the single-GPU op.
    """
    import torch.distributed as dist

    if rank is None or world is None:
        if dist.is_available() and dist.is_initialized():
            rank, world = dist.get_rank(group), dist.get_world_size(group)
        else:
            rank, world = 0, 1
    B, Hkv = query_states.shape[0], key_states.shape[1]
    shard = plan(B, Hkv, world, rank)
    out = torch.empty_like(query_states)
    run_shard(query_states, key_states, value_states, tree_mask, out, shard, block_m=block_m, block_n=block_n,
              compute=compute)
    if gather_output and world > 1:
        gather(out, shard, group)
    return out
