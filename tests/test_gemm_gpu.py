"""
The tcgen05 tf32 GEMM (cg_gemm_tf32) against float64 torch matmul.

tf32 keeps 10 explicit mantissa bits per operand and accumulates in fp32, so
the stated bound is a norm-wise relative error below 3e-3 (observed ~5e-4).
Covers the four operand layouts (x W^T, g W, g^T x, and both transposed),
partial tiles, every tile width, bias, the SiLU and SiLU-derivative epilogues,
accumulation, and that no bounded wait fired.
"""

from __future__ import annotations

import pytest
import torch

from create_graph_b200 import native
from create_graph_b200.gemm import ACT_ADD, ACT_SILU, ACT_SILU_GRAD, gemm

pytestmark = pytest.mark.gpu
TF32_TOL = 3e-3


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def operands(m, n, k, a_t, b_t, seed=0):
    gen = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=gen)
    b = torch.randn(n, k, generator=gen)
    a_dev = (a.t().contiguous() if a_t else a).cuda()
    b_dev = (b.t().contiguous() if b_t else b).cuda()
    return a, b, a_dev, b_dev


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize(
    "mnk",
    [(128, 64, 32), (300, 200, 100), (1000, 2304, 768), (768, 768, 4100), (77, 3072, 768), (12, 128, 20000),
     (128, 12, 20000), (5000, 12, 128), (5000, 128, 12), (40, 24, 300), (8280, 768, 768)],
)
def test_layouts_and_sizes(a_t, b_t, mnk):
    m, n, k = mnk
    a, b, a_dev, b_dev = operands(m, n, k, a_t, b_t)
    got = gemm(a_dev, b_dev, a_t=a_t, b_t=b_t)
    torch.cuda.synchronize()
    assert native.device_error() == 0
    assert rel(got.cpu(), a.double() @ b.double().T) < TF32_TOL


def test_bias_silu_and_saved_preactivation():
    m, n, k = 513, 384, 256
    a, b, a_dev, b_dev = operands(m, n, k, False, False, seed=1)
    bias = torch.randn(n)
    pre = torch.empty(m, n, device="cuda")
    got = gemm(a_dev, b_dev, bias=bias.cuda(), act=ACT_SILU, aux_out=pre)
    z = a.double() @ b.double().T + bias.double()
    assert rel(pre.cpu(), z) < TF32_TOL
    assert rel(got.cpu(), torch.nn.functional.silu(z)) < TF32_TOL


def test_silu_gradient_epilogue_and_accumulate():
    m, n, k = 256, 640, 96
    a, b, a_dev, b_dev = operands(m, n, k, False, True, seed=2)
    z = torch.randn(m, n)
    s = torch.sigmoid(z.double())
    dsilu = s * (1 + z.double() * (1 - s))
    got = gemm(a_dev, b_dev, b_t=True, act=ACT_SILU_GRAD, aux_in=z.cuda())
    assert rel(got.cpu(), (a.double() @ b.double().T) * dsilu) < TF32_TOL
    # the product before the derivative, written through aux_out
    u = torch.empty(m, n, device="cuda")
    again = gemm(a_dev, b_dev, b_t=True, act=ACT_SILU_GRAD, aux_in=z.cuda(), aux_out=u)
    assert torch.equal(again, got)
    assert rel(u.cpu(), a.double() @ b.double().T) < TF32_TOL
    base = torch.randn(m, n)
    acc = base.clone().cuda()
    gemm(a_dev, b_dev, b_t=True, out=acc, accumulate=True, alpha=0.5)
    assert rel(acc.cpu(), base.double() + 0.5 * a.double() @ b.double().T) < TF32_TOL


@pytest.mark.parametrize("mnk", [(513, 384, 256), (12, 128, 20000)])
def test_residual_add_epilogue(mnk):
    """C = A B^T + bias + R (R read through the aux operand), also on the split-K path."""
    m, n, k = mnk
    a, b, a_dev, b_dev = operands(m, n, k, False, False, seed=6)
    bias, r = torch.randn(n), torch.randn(m, n)
    got = gemm(a_dev, b_dev, bias=bias.cuda(), act=ACT_ADD, aux_in=r.cuda())
    torch.cuda.synchronize()
    assert native.device_error() == 0
    want = a.double() @ b.double().T + bias.double() + r.double()
    assert rel(got.cpu(), want) < TF32_TOL


@pytest.mark.parametrize("n,b_t,act", [(768, False, ACT_ADD), (768, True, ACT_SILU_GRAD), (3072, False, ACT_SILU),
                                       (3072, True, ACT_ADD)])
def test_wide_tile_epilogues_on_eight_warps(n, b_t, act):
    """Output-heavy shapes (8280 rows, 192- and 256-column tiles) whose epilogue
    streams a second (M, N) operand run on eight epilogue warps: every epilogue
    form against float64, ragged last row tile."""
    m, k = 8280, 256
    a, b, a_dev, b_dev = operands(m, n, k, False, b_t, seed=8)
    gen = torch.Generator().manual_seed(9)
    bias, aux = torch.randn(n, generator=gen), torch.randn(m, n, generator=gen)
    prod = a.double() @ b.double().T
    x = prod + bias.double()
    side = torch.full((m, n), float("nan"), device="cuda")
    if act == ACT_ADD:
        got = gemm(a_dev, b_dev, b_t=b_t, bias=bias.cuda(), act=act, aux_in=aux.cuda())
        want, want_side = x + aux.double(), None
    elif act == ACT_SILU:
        got = gemm(a_dev, b_dev, b_t=b_t, bias=bias.cuda(), act=act, aux_out=side)
        want, want_side = torch.nn.functional.silu(x), x
    else:
        s = torch.sigmoid(aux.double())
        got = gemm(a_dev, b_dev, b_t=b_t, bias=bias.cuda(), act=act, aux_in=aux.cuda(), aux_out=side)
        want, want_side = x * (s * (1 + aux.double() * (1 - s))), x
    torch.cuda.synchronize()
    assert native.device_error() == 0
    assert rel(got.cpu(), want) < TF32_TOL
    if want_side is not None:
        assert rel(side.cpu(), want_side) < TF32_TOL


def test_split_k_is_deterministic_and_uses_the_epilogue():
    """Weight-gradient shapes (small M x N, K = edges) split K across CTAs; the
    partial tiles are added in a fixed order."""
    m, n, k = 12, 128, 50000
    a, b, a_dev, b_dev = operands(m, n, k, True, True, seed=5)
    bias = torch.randn(n)
    first = gemm(a_dev, b_dev, a_t=True, b_t=True, bias=bias.cuda())
    second = gemm(a_dev, b_dev, a_t=True, b_t=True, bias=bias.cuda())
    assert torch.equal(first, second)
    assert rel(first.cpu(), a.double() @ b.double().T + bias.double()) < TF32_TOL


def test_strided_operands_in_place():
    """Column slices of wider tensors (a (M, 3C) activation, a sub-block of W)."""
    gen = torch.Generator().manual_seed(3)
    big = torch.randn(400, 3 * 96, generator=gen).cuda()
    w = torch.randn(64, 96, generator=gen).cuda()
    x = big[:, 96:192]
    got = gemm(x, w)
    assert rel(got.cpu(), x.double().cpu() @ w.double().cpu().T) < TF32_TOL


# ---------------------------------------------------------------------------
# fp32 precision: the three-term tf32 split (CG_GEMM_FP32)
# ---------------------------------------------------------------------------

FP32_TOL = 1e-5


@pytest.mark.parametrize("a_t", [False, True])
@pytest.mark.parametrize("b_t", [False, True])
@pytest.mark.parametrize(
    "mnk",
    [(128, 64, 32), (300, 200, 100), (1000, 2304, 768), (768, 768, 4100), (77, 3072, 768), (12, 128, 20000),
     (5000, 12, 128), (40, 24, 300), (4096, 512, 128)],
)
def test_fp32_precision_layouts_and_sizes(a_t, b_t, mnk):
    m, n, k = mnk
    a, b, a_dev, b_dev = operands(m, n, k, a_t, b_t, seed=3)
    got = gemm(a_dev, b_dev, a_t=a_t, b_t=b_t, precision="fp32")
    torch.cuda.synchronize()
    assert native.device_error() == 0
    err = rel(got.cpu(), a.double() @ b.double().T)
    assert err < FP32_TOL, err


def test_fp32_precision_epilogues():
    m, n, k = 513, 384, 256
    a, b, a_dev, b_dev = operands(m, n, k, False, False, seed=4)
    bias = torch.randn(n)
    pre = torch.empty(m, n, device="cuda")
    got = gemm(a_dev, b_dev, bias=bias.cuda(), act=ACT_SILU, aux_out=pre, precision="fp32")
    z = a.double() @ b.double().T + bias.double()
    assert rel(pre.cpu(), z) < FP32_TOL
    assert rel(got.cpu(), torch.nn.functional.silu(z)) < FP32_TOL
    r = torch.randn(m, n)
    got = gemm(a_dev, b_dev, act=ACT_ADD, aux_in=r.cuda(), precision="fp32")
    assert rel(got.cpu(), r.double() + a.double() @ b.double().T) < FP32_TOL


def test_fp32_precision_is_the_thread_default_inside_gemm_precision():
    from create_graph_b200.gemm import current_precision, gemm_precision

    a, b, a_dev, b_dev = operands(256, 256, 512, False, False, seed=5)
    want = a.double() @ b.double().T
    assert current_precision() == "tf32"
    with gemm_precision("fp32"):
        assert current_precision() == "fp32"
        inside = gemm(a_dev, b_dev)
    assert current_precision() == "tf32"
    outside = gemm(a_dev, b_dev)
    assert rel(inside.cpu(), want) < FP32_TOL
    assert FP32_TOL < rel(outside.cpu(), want) < TF32_TOL
    assert torch.equal(inside, gemm(a_dev, b_dev, precision="fp32"))

