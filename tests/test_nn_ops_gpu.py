"""
The fused ops of the energy network (create_graph_b200.nn) against float64
torch composites of the same functions, at all three levels create_graph
uses: forward, the force-pass gradient (create_graph=True) and the
parameter backward through it (tests/twice.py).

Tolerances: float32 kernels at 1e-5 relative (norm-wise); ops on the tf32
GEMM at the stated tf32 bound 3e-3.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

from create_graph_b200 import native
from create_graph_b200 import nn as cgnn
from tests.twice import twice_errors

pytestmark = pytest.mark.gpu
F32_TOL = 1e-5
TF32_TOL = 3e-3


def check(errors, tol):
    bad = {k: v for k, v in errors.items() if not v <= tol}
    assert not bad, f"above {tol}: {bad} (all {errors})"


def randn(*shape, seed=0, scale=1.0):
    g = torch.Generator().manual_seed(seed)
    return (scale * torch.randn(*shape, generator=g)).cuda()


def test_mm_and_linear():
    x, w, b = randn(300, 96, seed=1), randn(200, 96, seed=2), randn(200, seed=3)
    check(twice_errors(cgnn.mm, lambda a, c: a @ c.T, [x, w]), TF32_TOL)
    check(twice_errors(lambda *a: cgnn.LinearFn.apply(*a), F.linear, [x, w, b]), TF32_TOL)
    silu_lin = lambda *a: cgnn.LinearSiluFn.apply(*a)[0]  # noqa: E731
    check(twice_errors(silu_lin, lambda *a: F.silu(F.linear(*a)), [x, w, b]), TF32_TOL)


@pytest.mark.parametrize("cols", [192, 128, 768])
def test_layer_norm(cols):
    """192 columns take the strided row kernels, 128 and 768 the row-resident ones."""
    x = randn(257, cols, seed=4, scale=2.0) + 0.5
    gamma, beta = randn(cols, seed=5), randn(cols, seed=6)
    mine = lambda x, g, b: cgnn.ScaleShift.apply(cgnn.RowNorm.apply(x, 1e-5), g, b)  # noqa: E731
    ref = lambda x, g, b: F.layer_norm(x, (x.shape[-1],), g, b, 1e-5)  # noqa: E731
    check(twice_errors(mine, ref, [x, gamma, beta]), F32_TOL)


@pytest.mark.parametrize("cols", [192, 256, 768])
def test_residual_branch_and_linear_residual(cols):
    """x + Linear(LayerNorm(x)) with the branch point's two gradients summed in
    the normalisation backward kernel and the add in the GEMM epilogue."""
    x = randn(257, cols, seed=9, scale=2.0) + 0.5
    w, b = randn(cols, cols, seed=10, scale=1.0 / math.sqrt(cols)), randn(cols, seed=11)
    gamma, beta = randn(cols, seed=12), randn(cols, seed=13)

    def mine(x, w, b, g, be):
        r, xhat = cgnn.BranchNorm.apply(x, 1e-5)
        return cgnn.LinearResidualFn.apply(cgnn.ScaleShift.apply(xhat, g, be), w, b, r)

    def ref(x, w, b, g, be):
        return x + F.linear(F.layer_norm(x, (x.shape[-1],), g, be, 1e-5), w, b)

    check(twice_errors(mine, ref, [x, w, b, gamma, beta]), TF32_TOL)


def test_ffn_with_silu_gradient_in_the_epilogue():
    """r + W2 silu(W1 x + b1) + b2 through LinearSiluFn and SiluLinearResidualFn
    (the SiLU derivative applied in the second layer's input-gradient GEMM)."""
    x, r = randn(257, 128, seed=17), randn(257, 128, seed=18)
    w1, b1 = randn(512, 128, seed=19, scale=1.0 / math.sqrt(128)), randn(512, seed=20)
    w2, b2 = randn(128, 512, seed=21, scale=1.0 / math.sqrt(512)), randn(128, seed=22)

    def mine(x, w1, b1, w2, b2, r):
        y, z = cgnn.LinearSiluFn.apply(x, w1, b1)
        return cgnn.SiluLinearResidualFn.apply(y, z, w2, b2, r)

    def ref(x, w1, b1, w2, b2, r):
        return r + F.linear(F.silu(F.linear(x, w1, b1)), w2, b2)

    check(twice_errors(mine, ref, [x, w1, b1, w2, b2, r]), TF32_TOL)


def test_rownorm_backward_with_residual_matches_separate_add():
    x, g, r = randn(300, 768, seed=14), randn(300, 768, seed=15), randn(300, 768, seed=16)
    fused = cgnn.RowNormGrad.apply(g, x, 1e-5, r)
    plain = cgnn.RowNormGrad.apply(g, x, 1e-5, None) + r
    torch.cuda.synchronize()
    assert (fused - plain).abs().max().item() <= 1e-5 * plain.abs().max().item()


def test_column_ops():
    a, b = randn(1000, 40, seed=7), randn(1000, 40, seed=8)
    check(twice_errors(lambda a: cgnn.ColSum.apply(a), lambda a: a.sum(0), [a]), F32_TOL)
    check(twice_errors(lambda a, b: cgnn.ColDot.apply(a, b), lambda a, b: (a * b).sum(0), [a, b]), F32_TOL)


def test_gather_and_segment_sum():
    n, e = 50, 400
    g = torch.Generator().manual_seed(9)
    index = torch.randint(-1, n, (e,), generator=g).cuda()
    csr = cgnn.Csr.from_index(index, n)
    src = randn(n, 24, seed=10)
    rows = randn(e, 24, seed=11)

    def ref_gather(s):
        out = s[index.clamp_min(0).long()]
        return out * (index >= 0)[:, None].to(out.dtype)

    def ref_segsum(r):
        out = torch.zeros(n, r.shape[1], dtype=r.dtype, device=r.device)
        keep = index >= 0
        return out.index_add(0, index[keep].long(), r[keep])

    check(twice_errors(lambda s: cgnn.Gather.apply(s, csr), ref_gather, [src]), F32_TOL)
    check(twice_errors(lambda r: cgnn.SegmentSum.apply(r, csr), ref_segsum, [rows]), F32_TOL)
    # deterministic: bitwise equal on repeat
    a = cgnn.segment_sum_raw(rows, csr)
    assert torch.equal(a, cgnn.segment_sum_raw(rows, csr))


def test_pool_family():
    x, w = randn(37, 30, 64, seed=12), randn(37, 30, seed=13)
    check(twice_errors(lambda x, w: cgnn.Pool.apply(x, w), lambda x, w: (w[..., None] * x).sum(1), [x, w]), F32_TOL)


def neighbor_case(n=40, k=12, seed=14):
    g = torch.Generator().manual_seed(seed)
    pos = (3.0 * torch.rand(n, 3, generator=g)).cuda()
    counts = torch.randint(0, k + 1, (n,), generator=g, dtype=torch.int32)
    nbr = torch.full((n, k), -1, dtype=torch.int32)
    for i in range(n):
        others = torch.tensor([j for j in range(n) if j != i])
        pick = others[torch.randperm(n - 1, generator=g)[: int(counts[i])]]
        nbr[i, : int(counts[i])] = pick.to(torch.int32)
    nbr = nbr.cuda()
    graph = cgnn.NeighborGraph(nbr, counts.cuda(), cgnn.Csr.from_index(nbr.flatten(), n), k)
    return pos, graph


def ref_geometry(pos, nbr, n_rbf, cutoff, gamma):
    n, k = nbr.shape
    valid = (nbr >= 0).flatten()
    i = torch.arange(n, device=pos.device).repeat_interleave(k)
    # padded slots point at another atom so the masked terms stay finite
    j = torch.where(valid, nbr.flatten().long(), (i + 1) % n)
    vec = pos[j] - pos[i]
    d = vec.norm(dim=-1)
    mu = torch.arange(n_rbf, device=pos.device, dtype=pos.dtype) * (cutoff / (n_rbf - 1))
    rbf = torch.exp(-gamma * (d[:, None] - mu) ** 2) * valid[:, None]
    env = 0.5 * (torch.cos(math.pi * d / cutoff) + 1) * (d < cutoff) * valid
    return rbf, env


def test_edge_geometry():
    pos, graph = neighbor_case()
    args = (16, 2.5, 4.0)
    mine = lambda p: cgnn.EdgeGeometry.apply(p, graph, *args)  # noqa: E731
    ref = lambda p: ref_geometry(p, graph.nbr, *args)  # noqa: E731
    check(twice_errors(mine, ref, [pos]), F32_TOL)


def ref_token_attention(qkv, bias, index, counts, heads, scale):
    n = counts.shape[0]
    k = index.numel() // n
    d = qkv.shape[1] // (3 * heads)
    valid = (index >= 0)[:, None].to(qkv.dtype)
    tok = qkv[index.clamp_min(0).long()] * valid
    t = tok.view(n, k, 3, heads, d)
    q, kk, v = (t[:, :, i].permute(0, 2, 1, 3) for i in range(3))
    b = bias.view(n, k, heads).permute(0, 2, 1)[:, :, None, :]
    mask = torch.arange(k, device=tok.device)[None, :] >= counts[:, None].long()
    b = b.masked_fill(mask[:, None, None, :], -torch.inf)
    logits = q @ kk.transpose(-1, -2) * scale + b
    row_ok = (~mask).any(-1)[:, None, None, None]  # atoms without neighbours give zeros
    p = torch.softmax(torch.where(row_ok, logits, torch.zeros_like(logits)), -1) * row_ok
    return (p @ v).permute(0, 2, 1, 3).reshape(n, k, heads * d)


@pytest.mark.parametrize("precision,tol", [("fp32", F32_TOL), ("tf32", 5e-3)])
def test_token_attention(precision, tol):
    """Tokens gathered from per-atom qkv rows through the neighbour index (padded
    slots read zeros); per-token gradients reduced back to atoms. tf32: one
    tf32 product per tile, checked at the stated TF32 bound."""
    pos, graph = neighbor_case(n=40, k=12)
    heads, d = 4, 16
    g = torch.Generator().manual_seed(15)
    qkv = torch.randn(40, 3 * heads * d, generator=g).cuda()
    bias = torch.randn(40 * 12, heads, generator=g).cuda()
    mine = lambda q, b: cgnn.TokenAttention.apply(q, b, graph, heads, 0.25, precision)  # noqa: E731
    ref = lambda q, b: ref_token_attention(q, b, graph.tokens.index, graph.counts, heads, 0.25)  # noqa: E731
    check(twice_errors(mine, ref, [qkv, bias]), tol)


@pytest.mark.parametrize("precision,tol", [("fp32", F32_TOL), ("tf32", 5e-3)])
@pytest.mark.parametrize("heads,d", [(4, 16), (2, 64), (3, 20)])
def test_pooled_token_attention(precision, tol, heads, d):
    """Attention among each atom's tokens followed by the envelope-weighted sum
    over tokens, fused (cg_pooled_attn_*), against the torch composition of the
    two: output, first and second derivatives w.r.t. qkv, bias and env; atoms
    with no neighbour, padded token slots and a head dim below the padded
    width included."""
    n, k = 40, 12
    pos, graph = neighbor_case(n=n, k=k)
    g = torch.Generator().manual_seed(16)
    qkv = torch.randn(n, 3 * heads * d, generator=g).cuda()
    bias = torch.randn(n * k, heads, generator=g).cuda()
    env = torch.rand(n * k, generator=g).cuda()
    mine = lambda q, b, e: cgnn.PooledTokenAttention.apply(q, b, e, graph, heads, 0.25, precision)  # noqa: E731

    def ref(q, b, e):
        o = ref_token_attention(q, b, graph.tokens.index, graph.counts, heads, 0.25)
        return (e.view(n, k, 1) * o).sum(1)

    check(twice_errors(mine, ref, [qkv, bias, env]), tol)


def test_pooled_token_attention_deterministic():
    n, k, heads, d = 40, 12, 2, 64
    pos, graph = neighbor_case(n=n, k=k)
    g = torch.Generator().manual_seed(17)
    qkv = torch.randn(n, 3 * heads * d, generator=g).cuda().requires_grad_(True)
    bias = torch.randn(n * k, heads, generator=g).cuda().requires_grad_(True)
    env = torch.rand(n * k, generator=g).cuda().requires_grad_(True)

    def run():
        out = cgnn.PooledTokenAttention.apply(qkv, bias, env, graph, heads, 0.125, "tf32")
        gq, gb, ge = torch.autograd.grad(out.square().sum(), [qkv, bias, env], create_graph=True)
        return [out, gq, gb, ge, *torch.autograd.grad(gq.sum() + gb.square().sum() + ge.sum(), [qkv, bias, env])]

    first, second = run(), run()
    assert all(torch.equal(a, b) for a, b in zip(first, second))


def test_segment_sum_scaled():
    """out[a, h*d + c] = sum over tokens t of atom a of w[t, h] * src[t // k, h*d + c]."""
    n, k, heads, d = 30, 7, 3, 12
    pos, graph = neighbor_case(n=n, k=k)
    g = torch.Generator().manual_seed(18)
    w = torch.randn(n * k, heads, generator=g).cuda()
    src = torch.randn(n, heads * d, generator=g).cuda()
    csr = graph.tokens
    out = torch.full((n, heads * d + 5), 7.0, device="cuda")
    native.call("cg_segment_sum_scaled", w.data_ptr(), src.data_ptr(), src.stride(0), k, heads, d,
                csr.row_ptr.data_ptr(), csr.perm.data_ptr(), n, out.data_ptr(), out.stride(0), 0,
                native.stream_ptr())
    idx = csr.index.long().cpu()
    want = torch.zeros(n, heads, d, dtype=torch.float64)
    rows = (w.double().cpu()[:, :, None] * src.double().cpu().view(n, 1, heads, d).repeat_interleave(k, 0)[:, 0])
    for t in range(n * k):
        if idx[t] >= 0:
            want[idx[t]] += rows[t]
    assert torch.allclose(out[:, : heads * d].double().cpu(), want.view(n, -1), rtol=1e-5, atol=1e-5)
    assert torch.all(out[:, heads * d :] == 7.0)


@pytest.mark.parametrize("cols", [20, 132, 1536])
def test_segment_sum_long_segments(cols):
    """Segments longer than the 32 rows the kernel prefetches, and column
    counts that leave the last 128-column chunk partial."""
    n, e = 5, 400
    g = torch.Generator().manual_seed(19)
    index = torch.randint(-1, n, (e,), generator=g).cuda()
    csr = cgnn.Csr.from_index(index, n)
    rows = randn(e, cols, seed=20)
    keep = index >= 0
    want = torch.zeros(n, cols, dtype=torch.float64, device="cuda").index_add(0, index[keep].long(),
                                                                             rows[keep].double())
    got = cgnn.segment_sum_raw(rows, csr)
    assert torch.allclose(got.double(), want, rtol=1e-5, atol=1e-4)
    assert torch.equal(got, cgnn.segment_sum_raw(rows, csr))
    w = randn(e, 4, seed=21)
    src = randn(e // 8, 4 * 8, seed=22)
    out = torch.empty(n, 32, device="cuda")
    native.call("cg_segment_sum_scaled", w.data_ptr(), src.data_ptr(), src.stride(0), 8, 4, 8, csr.row_ptr.data_ptr(),
                csr.perm.data_ptr(), n, out.data_ptr(), out.stride(0), 0, native.stream_ptr())
    terms = (w.double()[:, :, None] * src.double().repeat_interleave(8, 0).view(e, 4, 8)).view(e, 32)
    want2 = torch.zeros(n, 32, dtype=torch.float64, device="cuda").index_add(0, index[keep].long(), terms[keep])
    assert torch.allclose(out.double(), want2, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("rows,cols", [(248400, 12), (8280, 768), (3001, 132), (777, 130), (5, 3072)])
def test_colsum_coldot_shapes(rows, cols):
    """Column sums and column dot products: packed narrow rows, full 128-column
    blocks, a partial block, the scalar path (columns not a multiple of 4) and
    fewer rows than warps; bitwise repeatable."""
    a, b = randn(rows, cols, seed=23), randn(rows, cols, seed=24)
    s1, s2 = cgnn.ColSum.apply(a), cgnn.ColSum.apply(a)
    d1, d2 = cgnn.ColDot.apply(a, b), cgnn.ColDot.apply(a, b)
    assert torch.equal(s1, s2) and torch.equal(d1, d2)
    want_s = a.double().sum(0)
    want_d = (a.double() * b.double()).sum(0)
    scale = rows ** 0.5
    assert (s1.double() - want_s).abs().max().item() < 1e-5 * scale
    assert (d1.double() - want_d).abs().max().item() < 1e-5 * scale


@pytest.mark.parametrize("precision,tol", [("fp32", F32_TOL), ("tf32", 5e-3)])
def test_pooled_token_attention_strided_bias(precision, tol):
    """The per-key bias as a column block of a wider matrix (the model's one
    GEMM for every block's bias), read in place through its row pitch, in the
    forward and both derivatives (the dbias cotangent arrives strided too)."""
    n, k, heads, d = 40, 12, 4, 16
    pos, graph = neighbor_case(n=n, k=k)
    g = torch.Generator().manual_seed(25)
    qkv = torch.randn(n, 3 * heads * d, generator=g).cuda()
    bias = torch.randn(n * k, heads, generator=g).cuda()
    env = torch.rand(n * k, generator=g).cuda()

    def widen(b):
        z = torch.zeros(b.shape[0], heads, dtype=b.dtype, device=b.device)
        return cgnn.SplitCols.apply(torch.cat([z, b, z], dim=1), heads)[1]

    def mine(q, b, e):
        view = widen(b)
        assert view.stride(0) == 3 * heads and view.stride(1) == 1
        return cgnn.PooledTokenAttention.apply(q, view, e, graph, heads, 0.25, precision)

    def ref(q, b, e):
        o = ref_token_attention(q, b, graph.tokens.index, graph.counts, heads, 0.25)
        return (e.view(n, k, 1) * o).sum(1)

    check(twice_errors(mine, ref, [qkv, bias, env]), tol)


def test_pooled_output_from_known_weights_equals_the_forward():
    """cg_pooled_attn_out (a checkpoint recompute's attention output from the
    first forward's weights) equals the forward kernel's output bit for bit."""
    from create_graph_b200.edge_attn import pooled_attention_forward, pooled_attention_out

    gen = torch.Generator().manual_seed(9)
    for n, h, k, d, prec in ((300, 12, 30, 64, "tf32"), (200, 4, 32, 32, "fp32"), (50, 2, 12, 16, "fp32")):
        qkv = torch.randn(n, 3 * h * d, generator=gen).cuda()
        bias = (0.1 * torch.randn(n * k, h, generator=gen)).cuda()
        env = torch.rand(n * k, generator=gen).cuda()
        counts = torch.randint(1, k + 1, (n,), generator=gen, dtype=torch.int32).cuda()
        index = torch.randint(0, n, (n, k), generator=gen, dtype=torch.int32).cuda()
        index[torch.arange(k, device="cuda")[None, :] >= counts[:, None]] = -1
        out, lse, w = pooled_attention_forward(qkv, bias, env, index.view(-1), counts, k, h, d ** -0.5, prec)
        again = pooled_attention_out(qkv, w, index.view(-1), counts, k, h)
        assert torch.equal(again, out)
