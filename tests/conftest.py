"""Shared test setup: the ``gpu`` marker, import paths and seeded inputs."""

import os
import sys

import numpy as np
import pytest

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(REPO, "eagle3-tree-sparse-flashattn_b200")
GOLDEN = os.path.join(REPO, "tests", "golden")
for p in (PKG, os.path.join(REPO, "oracle"), REPO):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def bf16_inputs(seed, B, Hq, Hkv, D, P, T):
    """Q/K/V ~ N(0,1) drawn in fp32 from a seeded CPU generator, rounded to bf16.

    Returns bf16 torch tensors (CPU).  Same draw order as the golden generator.
    """
    import torch

    gen = torch.Generator().manual_seed(int(seed))
    q = torch.randn((B, Hq, T, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    k = torch.randn((B, Hkv, P + T, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    v = torch.randn((B, Hkv, P + T, D), generator=gen, dtype=torch.float32).to(torch.bfloat16)
    return q, k, v


@pytest.fixture(scope="session")
def meta_golden():
    return load_npz("meta_golden.npz")


@pytest.fixture(scope="session")
def attn_golden():
    return load_npz("attn_golden.npz")
