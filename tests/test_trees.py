"""The seeded draft-tree generator the benchmark and the tests draw from:
masks are ancestor-or-self sets of a real tree (lower triangular, each row =
the node itself + its parent's row), depth and branching stay within the
limits, and a seed always gives the same tree."""

import numpy as np
import pytest

import tsfa_trees as trees


def _depths_and_children(parents):
    T = parents.size
    depth = np.zeros(T, dtype=int)
    children = np.zeros(T, dtype=int)
    for i in range(1, T):
        depth[i] = depth[parents[i]] + 1
        children[parents[i]] += 1
    return depth, children


@pytest.mark.parametrize("T,max_depth,branching,seed", [(64, 6, 4, 0), (256, 8, 6, 3), (128, 7, 4, 11), (9, 4, 3, 2)])
def test_random_tree_is_an_ancestor_mask_within_limits(T, max_depth, branching, seed):
    parents = trees.random_tree_parents(T, max_depth, branching, seed)
    mask = trees.parents_to_mask(parents)
    assert parents[0] == -1 and all(0 <= parents[i] < i for i in range(1, T))  # parents precede children
    assert np.array_equal(mask, np.tril(mask)) and mask.diagonal().all()
    for i in range(1, T):
        want = mask[parents[i]].copy()
        want[i] = True
        assert np.array_equal(mask[i], want)
    depth, children = _depths_and_children(parents)
    assert depth.max() <= max_depth and children.max() <= branching
    assert np.array_equal(mask, trees.random_tree(T, max_depth, branching, seed))  # seeded
    assert np.array_equal(mask.sum(axis=1), depth + 1)  # a row sees its whole ancestor chain


def test_random_tree_refuses_trees_that_do_not_fit():
    with pytest.raises(ValueError):
        trees.random_tree(10, max_depth=1, branching=3)  # root + 3 children at most


def test_chain_star_and_causal_sparse_shapes():
    T = 12
    assert np.array_equal(trees.chain_tree(T), np.tril(np.ones((T, T), bool)))
    star = trees.star_tree(T)
    assert star[:, 0].all() and star.diagonal().all() and star.sum() == 2 * T - 1
    cs = trees.random_causal_sparse(T, seed=1)
    assert np.array_equal(cs, np.tril(cs)) and cs.diagonal().all()
    assert trees.random_tree(0).shape == (0, 0) and trees.star_tree(0).shape == (0, 0)


def test_block_density():
    T = 64
    assert trees.block_density(trees.chain_tree(T), 64, 64) == 1.0
    assert trees.block_density(trees.chain_tree(T), 16, 16) == pytest.approx(10 / 16)  # lower triangle of 4 x 4
    assert trees.block_density(trees.star_tree(T), 16, 16) == pytest.approx(7 / 16)  # column 0 + diagonal
    assert trees.block_density(np.zeros((0, 0), bool), 16, 16) == 0.0
