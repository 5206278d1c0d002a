"""Seeded draft-tree masks for the verify step (workload generator).

The reference ships no tree generator: its benchmark draws a random
causal-sparse mask (``benchmark.py:164-168``), which is not an ancestor tree.
These generators produce real draft trees so that the tile classes (ZERO /
FULL / MIXED) and the block density look like EAGLE-3 verify traffic:

* ``random_tree``  -- node 0 is the root; every later node picks a depth
  uniformly among the feasible depths (a depth d is feasible if some node at
  d-1 still has fewer than ``branching`` children, and d <= max_depth), then a
  parent uniformly among the eligible nodes at d-1.  Parents always precede
  children, so the mask is lower triangular.
* ``chain_tree``   -- one branch: the fully causal ``tril`` mask.
* ``star_tree``    -- every node is a child of the root: column 0 + diagonal.
* ``random_causal_sparse`` -- the reference benchmark's mask family
  (``tril & ~(rand > 0.6)`` with the diagonal forced on).

``tree_mask[i, j] = 1`` iff ``j`` is an ancestor of ``i`` or ``j == i``.
All generators are pure numpy on a seeded ``default_rng`` and so give the same
mask on every host.
"""

from __future__ import annotations

import numpy as np


def parents_to_mask(parents: np.ndarray) -> np.ndarray:
    """Ancestor-or-self mask from a parent array (parent[0] == -1)."""
    T = int(parents.size)
    mask = np.zeros((T, T), dtype=np.bool_)
    for i in range(T):
        mask[i, i] = True
        p = int(parents[i])
        if p >= 0:
            mask[i] |= mask[p]
    return mask


def random_tree_parents(T: int, max_depth: int, branching: int, seed: int) -> np.ndarray:
    if T <= 0:
        return np.zeros(0, dtype=np.int64)
    rng = np.random.default_rng(seed)
    parents = np.full(T, -1, dtype=np.int64)
    depth = np.zeros(T, dtype=np.int64)
    children = np.zeros(T, dtype=np.int64)
    by_depth = {0: [0]}
    cur_max = 0
    for i in range(1, T):
        feasible = []
        for d in range(1, min(max_depth, cur_max + 1) + 1):
            if any(children[j] < branching for j in by_depth.get(d - 1, [])):
                feasible.append(d)
        if not feasible:
            raise ValueError(
                f"tree of {T} nodes does not fit max_depth={max_depth}, branching={branching}")
        d = feasible[int(rng.integers(len(feasible)))]
        eligible = [j for j in by_depth[d - 1] if children[j] < branching]
        p = eligible[int(rng.integers(len(eligible)))]
        parents[i] = p
        depth[i] = d
        children[p] += 1
        by_depth.setdefault(d, []).append(i)
        cur_max = max(cur_max, d)
    return parents


def random_tree(T: int, max_depth: int = 6, branching: int = 4, seed: int = 0) -> np.ndarray:
    return parents_to_mask(random_tree_parents(T, max_depth, branching, seed))


def chain_tree(T: int) -> np.ndarray:
    return np.tril(np.ones((T, T), dtype=np.bool_))


def star_tree(T: int) -> np.ndarray:
    mask = np.eye(T, dtype=np.bool_)
    if T:
        mask[:, 0] = True
    return mask


def random_causal_sparse(T: int, seed: int = 0, drop: float = 0.6) -> np.ndarray:
    rng = np.random.default_rng(seed)
    mask = np.tril(np.ones((T, T), dtype=np.bool_)) & ~(rng.random((T, T)) > drop)
    np.fill_diagonal(mask, True)
    return mask


def block_density(mask: np.ndarray, block_m: int, block_n: int) -> float:
    """Fraction of BM x BN tiles that are not ZERO."""
    T = mask.shape[0]
    if T == 0:
        return 0.0
    nqb = -(-T // block_m)
    ntb = -(-T // block_n)
    pad = np.zeros((nqb * block_m, ntb * block_n), dtype=np.bool_)
    pad[:T, :T] = mask
    tiles = pad.reshape(nqb, block_m, ntb, block_n).any(axis=(1, 3))
    return float(tiles.mean())


# The workloads named by the benchmark configs: (B, Hq, Hkv, D, P, T, BM, BN,
# tree kwargs).  Inputs Q/K/V ~ N(0, 1) in bf16, scale 1/sqrt(D).
CONFIGS = {
    "cfg1_cpu": dict(B=1, Hq=32, Hkv=8, D=128, P=512, T=64, BM=64, BN=64, max_depth=6, branching=4),
    "cfg2_llama3_8b": dict(B=1, Hq=32, Hkv=8, D=128, P=4096, T=64, BM=64, BN=64, max_depth=6, branching=4),
    "cfg3_serving_70b": dict(B=16, Hq=64, Hkv=8, D=128, P=8192, T=256, BM=64, BN=64, max_depth=8, branching=6),
    "cfg4_long_ctx": dict(B=4, Hq=32, Hkv=8, D=128, P=32768, T=128, BM=64, BN=64, max_depth=7, branching=4),
}


def config_tree(cfg: dict, seed: int = 0) -> np.ndarray:
    return random_tree(cfg["T"], cfg["max_depth"], cfg["branching"], seed)


# The sparsity / tiling sweep (the fifth benchmark configuration): batch 32,
# 32 q-heads / 8 kv-heads, head_dim in {64, 128}, prefix_len in {0, 1024,
# 16384}, tree sizes {64, 512, 1024}, BLOCK_M / BLOCK_N in {16, 32, 64, 128}
# (every pair, BM != BN included).  Per tree size, four trees whose visible
# fraction spans ~0.2 % (star) to ~50 % (chain, fully causal): a wide random
# tree (depth <= 6, branching <= 8) and a deep one (depth <= 64, branching
# <= 2) between them.
SWEEP5 = dict(B=32, Hq=32, Hkv=8, D=(64, 128), P=(0, 1024, 16384), T=(64, 512, 1024), BLOCKS=(16, 32, 64, 128))
SWEEP5_TREES = ("star", "chain", "wide", "deep")


def sweep5_tree(kind: str, T: int) -> np.ndarray:
    if kind == "star":
        return star_tree(T)
    if kind == "chain":
        return chain_tree(T)
    if kind == "wide":
        return random_tree(T, 6, 8, seed=T + 1)
    if kind == "deep":
        return random_tree(T, 64, 2, seed=T + 2)
    raise ValueError(kind)
