"""
Parity of the sm_100a edge-attention kernels (cg_edge_attn_fwd1/bwd1/bwd2,
through the C ABI) with the oracle and with the reference's golden vectors.

- float64 kernels against the golden vectors at 1e-10 (the reference test's
  own tolerance, tests/test_custom_ops.py:20 there);
- float32 kernels against the float64 oracle at 1e-5 relative (the stated
  float32 tolerance) in fp32 precision, and at the stated TF32 bound (2e-3
  relative, Frobenius; measured 4e-4 to 6e-4) in tf32 precision;
- ``cg.testing.check_op`` of the registered op against differentiable torch
  attention, as the reference tests its op;
- the microbenchmark shape (4096 x 8 heads x 32 tokens x 32 dims) on a sample
  of slices, the key-count mask, strided inputs and determinism.
"""

from __future__ import annotations

import glob
import os

import numpy as np
import pytest
import torch

import create_graph_b200 as cg
from create_graph_b200.edge_attn import (
    EdgeAttention,
    EdgeAttentionTF32,
    attn_backward1,
    attn_backward2,
    attn_forward1,
)
from oracle import edge_attn as oracle
from oracle.torch_ref import attention
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu
CASES = sorted(os.path.basename(p)[:-4] for p in glob.glob(os.path.join(GOLDEN, "edge_attn_*.npz")))
F32_TOL = 1e-5
# one tf32 product per tile: operands rounded to 2^-11 relative, fp32
# accumulation; the Frobenius-relative error of every output stays below this
TF32_TOL = 2e-3
TOL = {"fp32": F32_TOL, "tf32": TF32_TOL}
PRECISIONS = ["fp32", "tf32"]


def rel(a, b):
    a = a.detach().double().cpu().numpy() if isinstance(a, torch.Tensor) else np.asarray(a, np.float64)
    b = b.detach().double().cpu().numpy() if isinstance(b, torch.Tensor) else np.asarray(b, np.float64)
    fin = np.isfinite(b)
    assert np.array_equal(np.isfinite(a), fin), "non-finite entries differ"
    return np.linalg.norm((a - b)[fin]) / max(np.linalg.norm(b[fin]), 1e-300)


def load(name):
    with np.load(os.path.join(GOLDEN, name + ".npz")) as f:
        return {k: f[k] for k in f.files}


def dev(x, dtype=torch.float64):
    return torch.as_tensor(x, dtype=dtype, device="cuda")


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("dtype,precision", [(torch.float64, "fp32"), (torch.float32, "fp32"),
                                             (torch.float32, "tf32")])
def test_kernels_match_golden(name, dtype, precision):
    c = load(name)
    if dtype == torch.float64 and c["q"].shape[-1] > 16:
        pytest.skip("float64 kernels take head dims up to 16")
    tol = 1e-10 if dtype == torch.float64 else TOL[precision]
    q, k, v, bias, g = (dev(c[n], dtype) for n in ("q", "k", "v", "bias", "grad_out"))
    hq, hk, hv, hb = (dev(c[n], dtype) for n in ("hq", "hk", "hv", "hb"))
    scale = float(c["scale"])
    out, lse = attn_forward1(q, k, v, bias, scale, precision=precision)
    torch.cuda.synchronize()
    assert rel(out, c["out"]) < tol
    assert rel(lse, c["lse"]) < tol
    # backward kernels get the reference's lse so each is checked on its own
    lse_ref = dev(c["lse"], dtype)
    b1 = attn_backward1(q, k, v, bias, lse_ref, g, scale, precision=precision)
    for got, n in zip(b1, ("dq", "dk", "dv", "dbias")):
        assert got.shape == c[f"b1_{n}"].shape, n
        assert rel(got, c[f"b1_{n}"]) < tol, n
    got2 = attn_backward2(q, k, v, bias, lse_ref, g, scale, hq, hk, hv, hb, precision=precision)
    for got, n in zip(got2, ("dq", "dk", "dv", "dbias", "dgrad_out")):
        assert got.shape == c[f"b2_{n}"].shape, n
        assert rel(got, c[f"b2_{n}"]) < tol, n


def attn_args(seed=0, masked=False, dtype=torch.float64):
    """The reference test's arguments (tests/test_custom_ops.py:24-31 there), on the GPU."""
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(2, 3, 5, 4, generator=gen, dtype=dtype) for _ in range(3))
    bias = torch.randn(2, 1, 1, 5, generator=gen, dtype=dtype)
    if masked:
        bias[0, 0, 0, 1] = -torch.inf
        bias[1, 0, 0, 4] = -torch.inf
    return tuple(t.cuda() for t in (q, k, v, bias)) + (0.5,)


@pytest.mark.parametrize("op", [EdgeAttention, EdgeAttentionTF32])
@pytest.mark.parametrize("masked", [False, True])
def test_check_op_against_differentiable_attention(masked, op):
    """float64 inputs: both registered ops compute in float64."""
    errors = cg.testing.check_op(op, attention, attn_args(masked=masked))
    bad = {k: v for k, v in errors.items() if v > 1e-10}
    assert not bad, errors
    assert {"backward2.q", "backward2.bias", "backward2.grad_out"} <= set(errors)


def cfg2_inputs(n=4096, h=8, s=32, d=32, seed=0, device="cuda"):
    """The microbenchmark's inputs: q/k/v ~ N(0,1), bias ~ N(0, 0.1), keys
    j >= c_n masked with c_n ~ U{8..32}."""
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(n, h, s, d, generator=gen) for _ in range(3))
    bias = 0.1 * torch.randn(n, h, s, s, generator=gen)
    counts = torch.randint(8, s + 1, (n,), generator=gen, dtype=torch.int32)
    return [t.to(device) for t in (q, k, v, bias)], counts.to(device), 1.0 / d**0.5


@pytest.mark.parametrize("precision", PRECISIONS)
def test_microbench_shape_sampled_slices(precision):
    (q, k, v, bias), counts, scale = cfg2_inputs()
    gen = torch.Generator().manual_seed(1)
    g, hq, hk, hv = (torch.randn(q.shape, generator=gen).cuda() for _ in range(4))
    hb = 0.1 * torch.randn(bias.shape, generator=gen).cuda()
    tol = TOL[precision]
    out, lse = attn_forward1(q, k, v, bias, scale, counts, precision=precision)
    b1 = attn_backward1(q, k, v, bias, lse, g, scale, counts, precision=precision)
    b2 = attn_backward2(q, k, v, bias, lse, g, scale, hq, hk, hv, hb, counts, precision=precision)
    torch.cuda.synchronize()
    pick = torch.tensor([0, 1, 777, 2048, 4095])
    np_ = lambda t: t[pick].double().cpu().numpy()  # noqa: E731
    kc = counts[pick].cpu().numpy()
    args = [np_(t) for t in (q, k, v, bias)]
    want_out, want_lse = oracle.forward1(*args, scale, kc)
    assert rel(out[pick], want_out) < tol and rel(lse[pick], want_lse) < tol
    w1 = oracle.backward1(*args, np_(g), scale, kc)
    for got, want in zip(b1, w1):
        assert rel(got[pick], want) < tol
    w2 = oracle.backward2(*args, np_(g), scale, np_(hq), np_(hk), np_(hv), np_(hb), kc)
    for got, want in zip(b2, w2):
        assert rel(got[pick], want) < tol


@pytest.mark.parametrize("precision", PRECISIONS)
def test_deterministic(precision):
    (q, k, v, bias), counts, scale = cfg2_inputs(n=256)
    g = torch.randn_like(q)
    hq, hk, hv, hb = torch.randn_like(q), torch.randn_like(q), torch.randn_like(q), torch.randn_like(bias)
    out, lse = attn_forward1(q, k, v, bias, scale, counts, precision=precision)
    first = attn_backward2(q, k, v, bias, lse, g, scale, hq, hk, hv, hb, counts, precision=precision)
    second = attn_backward2(q, k, v, bias, lse, g, scale, hq, hk, hv, hb, counts, precision=precision)
    assert all(torch.equal(a, b) for a, b in zip(first, second))


def test_strided_token_layout_and_broadcast_bias():
    """q, k, v read in place from an (n, s, 3, h, d) token tensor; bias (n, h, 1, s)."""
    n, s, h, d = 20, 30, 4, 16
    gen = torch.Generator().manual_seed(3)
    tok = torch.randn(n, s, 3, h, d, generator=gen).cuda()
    q, k, v = (tok[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    bias = torch.randn(n, h, 1, s, generator=gen).cuda()
    g = torch.randn(n, h, s, d, generator=gen).cuda()
    out, lse = attn_forward1(q, k, v, bias, 0.25)
    dq, dk, dv, db = attn_backward1(q, k, v, bias, lse, g, 0.25)
    torch.cuda.synchronize()
    a = [t.double().cpu().numpy() for t in (q, k, v, bias)]
    wo, wl = oracle.forward1(*a, 0.25)
    assert rel(out, wo) < F32_TOL and rel(lse, wl) < F32_TOL
    w = oracle.backward1(*a, g.double().cpu().numpy(), 0.25)
    for got, want in zip((dq, dk, dv, db), w):
        assert got.shape == want.shape
        assert rel(got, want) < F32_TOL


def test_head_broadcast_bias_reduces_over_heads():
    """bias (n, 1, s, s): dbias is summed over heads through scratch, deterministically."""
    n, h, s, d = 9, 5, 16, 8
    gen = torch.Generator().manual_seed(4)
    q, k, v = (torch.randn(n, h, s, d, generator=gen, dtype=torch.float64).cuda() for _ in range(3))
    bias = torch.randn(n, 1, s, s, generator=gen, dtype=torch.float64).cuda()
    g = torch.randn(n, h, s, d, generator=gen, dtype=torch.float64).cuda()
    out, lse = attn_forward1(q, k, v, bias, 0.3)
    got = attn_backward1(q, k, v, bias, lse, g, 0.3)
    a = [t.cpu().numpy() for t in (q, k, v, bias)]
    want = oracle.backward1(*a, g.cpu().numpy(), 0.3)
    for x, y in zip(got, want):
        assert x.shape == y.shape and rel(x, y) < 1e-10


def test_bad_arguments_raise():
    q = torch.randn(2, 3, 40, 8, device="cuda")  # 40 tokens > 32
    with pytest.raises(cg.NativeError, match="k = 40"):
        attn_forward1(q, q, q, torch.zeros(1, device="cuda"), 1.0)
    with pytest.raises(cg.NativeError, match="CUDA tensors"):
        attn_forward1(q.cpu(), q, q, torch.zeros(1, device="cuda"), 1.0)
    with pytest.raises(ValueError, match="precision"):
        attn_forward1(q[:, :, :8], q[:, :, :8], q[:, :, :8], torch.zeros(1, device="cuda"), 1.0, precision="bf16")
