"""
The oracle against the golden vectors the reference produced
(tests/golden/make_golden.py): forward1, backward1 and backward2 of the masked
edge attention, float64, at the reference test's shapes, at the
microbenchmark's distribution and in the model's key-bias layout. This pins
the oracle before any GPU result is compared with it.
"""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest

from oracle import edge_attn as oracle
from tests.conftest import GOLDEN

CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "edge_attn_*.npz")))
TOL = 1e-12


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    fin = np.isfinite(b)
    assert np.array_equal(np.isfinite(a), fin), "non-finite entries differ"
    num = np.linalg.norm((a - b)[fin])
    den = max(np.linalg.norm(b[fin]), 1e-300)
    return num / den


@pytest.fixture(params=CASES)
def case(request):
    with np.load(os.path.join(GOLDEN, request.param + ".npz")) as f:
        return {k: f[k] for k in f.files}


def test_golden_cases_exist():
    assert {"edge_attn_testshape_plain", "edge_attn_testshape_masked", "edge_attn_cfg2_small",
            "edge_attn_keybias"} <= set(CASES)


def test_forward1(case):
    out, lse = oracle.forward1(case["q"], case["k"], case["v"], case["bias"], float(case["scale"]))
    assert rel(out, case["out"]) < TOL
    assert rel(lse, case["lse"]) < TOL


def test_backward1(case):
    got = oracle.backward1(case["q"], case["k"], case["v"], case["bias"], case["grad_out"], float(case["scale"]))
    for name, g in zip(("dq", "dk", "dv", "dbias"), got):
        assert g.shape == case[f"b1_{name}"].shape, name
        assert rel(g, case[f"b1_{name}"]) < TOL, name


def test_backward2(case):
    got = oracle.backward2(
        case["q"], case["k"], case["v"], case["bias"], case["grad_out"], float(case["scale"]),
        case["hq"], case["hk"], case["hv"], case["hb"],
    )
    for name, g in zip(("dq", "dk", "dv", "dbias", "dgrad_out"), got):
        assert g.shape == case[f"b2_{name}"].shape, name
        assert rel(g, case[f"b2_{name}"]) < TOL, name


def test_key_counts_equal_minus_inf_bias():
    """The kernels' key_counts mask is the reference's -inf bias on those keys."""
    with np.load(os.path.join(GOLDEN, "edge_attn_cfg2_small.npz")) as f:
        c = {k: f[k] for k in f.files}
    finite_bias = np.where(np.isfinite(c["bias"]), c["bias"], 0.0)
    out, lse = oracle.forward1(c["q"], c["k"], c["v"], finite_bias, float(c["scale"]), c["key_counts"])
    assert rel(out, c["out"]) < TOL and rel(lse, c["lse"]) < TOL


def test_fully_masked_rows_give_zero():
    rng = np.random.default_rng(0)
    q, k, v = (rng.standard_normal((1, 2, 4, 3)) for _ in range(3))
    bias = np.zeros((1, 1, 1, 4))
    out, lse = oracle.forward1(q, k, v, bias, 0.5, key_counts=np.array([0]))
    assert np.all(out == 0) and np.all(lse == -np.inf)
    g = oracle.backward1(q, k, v, bias, rng.standard_normal(out.shape), 0.5, key_counts=np.array([0]))
    assert all(np.all(x == 0) for x in g)
