"""Helpers shared by the GPU parity tests."""

import os

import numpy as np
import torch

import tsfa_oracle as orc
from conftest import bf16_inputs

ATOL = 2e-3  # the path's error budget: bf16 in, fp32 accumulate
# The oracle is exact fp32; the kernel's output is stored in bf16/fp16, whose own
# rounding (half an ulp, relative 2^-9 / 2^-12) is added to the budget.
OUT_REL = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}


def make_inputs(seed, B, Hq, Hkv, D, P, T, dtype=torch.bfloat16):
    q, k, v = bf16_inputs(seed, B, Hq, Hkv, D, P, T)
    if dtype != torch.bfloat16:
        q, k, v = (x.float().to(dtype) for x in (q, k, v))
    return q, k, v


def oracle(q, k, v, mask, P, units=None):
    """Dense+mask fp32 oracle; `units` = list of (b, kvh) to evaluate only those."""
    qn, kn, vn = (x.float().cpu().numpy() for x in (q, k, v))
    mask = np.asarray(mask)
    if units is None:
        return orc.dense_tree_attention(qn, kn, vn, mask, P)
    G = q.shape[1] // k.shape[1]
    outs = {}
    for b, kh in units:
        outs[(b, kh)] = orc.dense_tree_attention(qn[b:b + 1, kh * G:(kh + 1) * G], kn[b:b + 1, kh:kh + 1],
                                                 vn[b:b + 1, kh:kh + 1], mask, P)[0]
    return outs


def p_rounding_bound(q, k, v, mask, P):
    """Bound of the error from rounding p to bf16 before P.V (the reference
    does the same, tsfa.py:278): |dO| <= 2^-9 sum_j p_j |v_j|; twice that."""
    return 2.0 ** -8 * oracle(q, k, v.abs(), mask, P)


# Per test: (checked elements, max |err|, elements above the plain 2e-3).
# conftest prints the table at the end of the run, so every parity test shows
# both the plain max_abs_err and how many elements needed the output-rounding
# allowance.
STATS: dict = {}


def assert_close(got: torch.Tensor, want: np.ndarray, dtype=torch.bfloat16, atol=ATOL, extra=None, what=""):
    """|got - want| <= atol + OUT_REL[dtype] * |want| (+ extra) elementwise,
    NaN exactly where the oracle has NaN.  The bound: the north star's 2e-3
    for bf16 in / fp32 accumulate, plus half an ulp of the stored output --
    the bf16 store alone exceeds 2e-3 once |O| > 0.5, and the reference's
    output is rounded as well (to fp16, tsfa.py:339)."""
    g = got.float().cpu().numpy()
    assert g.shape == want.shape, (g.shape, want.shape)
    gn, wn = np.isnan(g), np.isnan(want)
    assert np.array_equal(gn, wn), f"{what} NaN pattern differs: {gn.sum()} vs {wn.sum()}"
    ok = ~wn
    err = np.abs(g[ok] - want[ok])
    tol = atol + OUT_REL[dtype] * np.abs(want[ok])
    if extra is not None:
        tol = tol + extra[ok]
    bad = err > tol
    emax = float(err.max()) if err.size else 0.0
    key = os.environ.get("PYTEST_CURRENT_TEST", "?").split(" ")[0]
    n0, m0, a0 = STATS.get(key, (0, 0.0, 0))
    STATS[key] = (n0 + int(err.size), max(m0, emax), a0 + int((err > ATOL).sum()))
    assert not bad.any(), f"{what} max_abs_err={emax:.3e}, {bad.sum()} elements above tolerance"
    return emax
