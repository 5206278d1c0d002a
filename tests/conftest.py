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


def pytest_terminal_summary(terminalreporter):
    """Parity statistics of the GPU tests: per test file, the elements checked
    against the oracle, the plain max_abs_err and how many elements exceeded a
    plain 2e-3 (those stayed inside 2e-3 plus half an ulp of the stored
    output)."""
    mod = sys.modules.get("gpu_helpers")
    stats = getattr(mod, "STATS", None)
    if not stats:
        return
    files = {}
    for key, (n, emax, above) in stats.items():
        f = key.split("::")[0]
        n0, m0, a0, t0 = files.get(f, (0, 0.0, 0, 0))
        files[f] = (n0 + n, max(m0, emax), a0 + above, t0 + 1)
    tr = terminalreporter
    tr.write_sep("-", "parity vs the fp32 oracle (plain max_abs_err; elements above a plain 2e-3)")
    for f, (n, emax, above, cases) in sorted(files.items()):
        tr.write_line(f"{f}: {cases} cases, {n} elements, max_abs_err {emax:.3e}, above 2e-3: {above}")


def load_npz(name):
    return np.load(os.path.join(GOLDEN, name), allow_pickle=False)


def _golden_generator():
    import importlib.util

    spec = importlib.util.spec_from_file_location("tsfa_gen_golden", os.path.join(GOLDEN, "gen_golden.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def metadata_digest(md) -> bytes:
    """The fixtures' digest of a metadata set (gen_golden.metadata_digest):
    `md` has the five reference fields, as numpy arrays or tensors."""
    arrs = []
    for f in ("row_ptr", "col_idx", "blk_type", "mixed_mask_payload", "mixed_mask_offset"):
        a = getattr(md, f)
        arrs.append(a.cpu().numpy() if hasattr(a, "cpu") else np.asarray(a))
    return _golden_generator().metadata_digest(arrs)


def mask_digest(mask) -> bytes:
    return _golden_generator().mask_digest(mask)


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
