"""
The fused kernels as ``torch.library`` operators (namespace ``cg_b200``), each
with a fake (shape function), so FakeTensor, ``torch.fx`` and
``torch.compile`` can trace code that calls them.

The energy network itself calls the kernels through the autograd Functions of
``create_graph_b200.nn`` (no dispatcher on the hot path); these registrations
are the same kernels for callers that build their own models on the
dispatcher, as the reference registers its edge-attention op through
torch.library (src/create_graph/ops.py:146-169 there). Every operator's
autograd formula is written with registered operators, so derivatives trace
too and the chains that create_graph differentiates twice stay differentiable:

    mm(a, b) = a @ b.T                      backward: mm, mm
    linear(x, w, b) = x w^T + b             backward: mm, mm, colsum
    linear_silu(x, w, b) = (silu(z), z)     backward: silu_grad, then as linear
    silu_grad(g, z) = g silu'(z)            backward: silu_grad, silu_grad2
    colsum(x)                               backward: expand
    segment_sum_csr / gather_csr            each other's backward
    edge_geom -> edge_geom_bwd1 -> edge_geom_bwd2   (pos -> rbf, env)
    neighbor_list                           integer outputs, no gradient
    edge_attn, edge_attn_tf32               registered by create_graph_b200.edge_attn

CSR arguments are (index, row_ptr, perm, rows) as in ``nn.Csr``; neighbour
graphs are (nbr, rev_ptr, rev_idx) as ``neighbor_list`` returns them.
"""

from __future__ import annotations

import ctypes

import torch
from torch import Tensor

from create_graph_b200 import native
from create_graph_b200 import nn as cgnn
from create_graph_b200.gemm import ACT_SILU


def _stream() -> int:
    return native.stream_ptr()


def _empty(like: Tensor, *shape: int, dtype=None) -> Tensor:
    return torch.empty(*shape, dtype=dtype or like.dtype, device=like.device)


# ---------------------------------------------------------------------------
# GEMM family
# ---------------------------------------------------------------------------


@torch.library.custom_op("cg_b200::mm", mutates_args=())
def mm(a: Tensor, b: Tensor) -> Tensor:
    """a @ b.T on the tcgen05 GEMM (a (M, K), b (N, K); transposed views are
    read in place)."""
    return cgnn.mm_raw(a, b)


@mm.register_fake
def _mm_fake(a, b):
    return _empty(a, a.shape[0], b.shape[0])


def _mm_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _mm_backward(ctx, g):
    a, b = ctx.saved_tensors
    ga = mm(g, b.t()) if ctx.needs_input_grad[0] else None
    gb = mm(g.t(), a.t()) if ctx.needs_input_grad[1] else None
    return ga, gb


mm.register_autograd(_mm_backward, setup_context=_mm_setup)


@torch.library.custom_op("cg_b200::colsum", mutates_args=())
def colsum(x: Tensor) -> Tensor:
    """Column sums of a (rows, cols) matrix, in a fixed order."""
    return cgnn.colsum_raw(x)


@colsum.register_fake
def _colsum_fake(x):
    return _empty(x, x.shape[1])


def _colsum_setup(ctx, inputs, output):
    ctx.rows = inputs[0].shape[0]


colsum.register_autograd(lambda ctx, h: h.expand(ctx.rows, h.shape[0]), setup_context=_colsum_setup)


@torch.library.custom_op("cg_b200::silu_grad", mutates_args=())
def silu_grad(g: Tensor, z: Tensor) -> Tensor:
    """g * silu'(z)."""
    g, z = cgnn._f32(g, "silu_grad"), cgnn._f32(z, "silu_grad")
    out = torch.empty_like(g)
    native.call("cg_silu_grad", g.data_ptr(), z.data_ptr(), out.data_ptr(), g.numel(), _stream())
    return out


@torch.library.custom_op("cg_b200::silu_grad2", mutates_args=())
def silu_grad2(h: Tensor, g: Tensor, z: Tensor) -> Tensor:
    """h * g * silu''(z) (the z-derivative of <h, silu_grad(g, z)>)."""
    h, g, z = (cgnn._f32(t, "silu_grad2") for t in (h, g, z))
    out = torch.empty_like(h)
    native.call("cg_silu_grad2", h.data_ptr(), g.data_ptr(), z.data_ptr(), out.data_ptr(), h.numel(), _stream())
    return out


for _op in (silu_grad, silu_grad2):
    _op.register_fake(lambda *args: torch.empty_like(args[0], memory_format=torch.contiguous_format))


def _silu_grad_setup(ctx, inputs, output):
    ctx.save_for_backward(*inputs)


def _silu_grad_backward(ctx, h):
    g, z = ctx.saved_tensors
    dg = silu_grad(h, z) if ctx.needs_input_grad[0] else None
    dz = silu_grad2(h, g, z) if ctx.needs_input_grad[1] else None
    return dg, dz


silu_grad.register_autograd(_silu_grad_backward, setup_context=_silu_grad_setup)


@torch.library.custom_op("cg_b200::linear", mutates_args=())
def linear(x: Tensor, w: Tensor, b: Tensor | None) -> Tensor:
    """x @ w.T + b (b may be None)."""
    return cgnn.mm_raw(x, w, bias=b)


@linear.register_fake
def _linear_fake(x, w, b):
    return _empty(x, x.shape[0], w.shape[0])


def _linear_setup(ctx, inputs, output):
    x, w, b = inputs
    ctx.save_for_backward(x, w)
    ctx.has_bias = b is not None


def _linear_grads(ctx, g, x, w):
    gx = mm(g, w.t()) if ctx.needs_input_grad[0] else None
    gw = mm(g.t(), x.t()) if ctx.needs_input_grad[1] else None
    gb = colsum(g) if ctx.has_bias and ctx.needs_input_grad[2] else None
    return gx, gw, gb


def _linear_backward(ctx, g):
    x, w = ctx.saved_tensors
    return _linear_grads(ctx, g, x, w)


linear.register_autograd(_linear_backward, setup_context=_linear_setup)


@torch.library.custom_op("cg_b200::linear_silu", mutates_args=())
def linear_silu(x: Tensor, w: Tensor, b: Tensor | None) -> tuple[Tensor, Tensor]:
    """(silu(z), z) with z = x @ w.T + b, from one GEMM (SiLU in its epilogue)."""
    z = torch.empty(x.shape[0], w.shape[0], device=x.device)
    y = cgnn.mm_raw(x, w, bias=b, act=ACT_SILU, aux_out=z)
    return y, z


@linear_silu.register_fake
def _linear_silu_fake(x, w, b):
    return _empty(x, x.shape[0], w.shape[0]), _empty(x, x.shape[0], w.shape[0])


def _linear_silu_setup(ctx, inputs, output):
    x, w, b = inputs
    ctx.save_for_backward(x, w, output[1])
    ctx.has_bias = b is not None
    ctx.set_materialize_grads(False)


def _linear_silu_backward(ctx, gy, gz):
    x, w, z = ctx.saved_tensors
    g = silu_grad(gy, z) if gy is not None else None
    if gz is not None:
        g = gz if g is None else g + gz
    if g is None:
        return None, None, None
    return _linear_grads(ctx, g, x, w)


linear_silu.register_autograd(_linear_silu_backward, setup_context=_linear_silu_setup)


# ---------------------------------------------------------------------------
# segment sums over a sorted CSR and their transpose
# ---------------------------------------------------------------------------


@torch.library.custom_op("cg_b200::segment_sum_csr", mutates_args=())
def segment_sum_csr(src: Tensor, index: Tensor, row_ptr: Tensor, perm: Tensor, rows: int) -> Tensor:
    """out[r] = sum of src[e] over index[e] == r, in ascending e (fixed order)."""
    return cgnn.segment_sum_raw(src, cgnn.Csr(index, row_ptr, perm, rows))


@torch.library.custom_op("cg_b200::gather_csr", mutates_args=())
def gather_csr(src: Tensor, index: Tensor, row_ptr: Tensor, perm: Tensor, rows: int) -> Tensor:
    """out[e] = src[index[e]] (zeros where index[e] < 0): segment_sum_csr's transpose."""
    return cgnn.gather_raw(src, cgnn.Csr(index, row_ptr, perm, rows))


@segment_sum_csr.register_fake
def _segment_sum_fake(src, index, row_ptr, perm, rows):
    return _empty(src, rows, src.shape[1])


@gather_csr.register_fake
def _gather_fake(src, index, row_ptr, perm, rows):
    return _empty(src, index.shape[0], src.shape[1])


def _csr_setup(ctx, inputs, output):
    _, index, row_ptr, perm, rows = inputs
    ctx.save_for_backward(index, row_ptr, perm)
    ctx.rows = rows


def _segment_sum_backward(ctx, g):
    index, row_ptr, perm = ctx.saved_tensors
    return gather_csr(g, index, row_ptr, perm, ctx.rows), None, None, None, None


def _gather_backward(ctx, g):
    index, row_ptr, perm = ctx.saved_tensors
    return segment_sum_csr(g, index, row_ptr, perm, ctx.rows), None, None, None, None


segment_sum_csr.register_autograd(_segment_sum_backward, setup_context=_csr_setup)
gather_csr.register_autograd(_gather_backward, setup_context=_csr_setup)


# ---------------------------------------------------------------------------
# edge geometry and its first and second derivatives
# ---------------------------------------------------------------------------


def _geom(pos: Tensor, nbr: Tensor, rev_ptr: Tensor, rev_idx: Tensor, n_rbf: int, cutoff: float, gamma: float):
    a = native.GeomArgs()
    a.pos, a.nbr, a.rev_ptr, a.rev_idx = pos.data_ptr(), nbr.data_ptr(), rev_ptr.data_ptr(), rev_idx.data_ptr()
    a.n_atoms, a.k = nbr.shape[0], nbr.shape[1]
    a.n_rbf, a.cutoff, a.gamma = n_rbf, cutoff, gamma
    return a


@torch.library.custom_op("cg_b200::edge_geom", mutates_args=())
def edge_geom(pos: Tensor, nbr: Tensor, rev_ptr: Tensor, rev_idx: Tensor, n_rbf: int, cutoff: float,
              gamma: float) -> tuple[Tensor, Tensor]:
    """(rbf (n*k, n_rbf), env (n*k,)) of the neighbour edges: Gaussians
    exp(-gamma (d - mu_m)^2) on [0, cutoff] and the cosine envelope."""
    pos = cgnn._f32(pos, "edge_geom")
    e = nbr.numel()
    rbf, env = torch.empty(e, n_rbf, device=pos.device), torch.empty(e, device=pos.device)
    a = _geom(pos, nbr, rev_ptr, rev_idx, n_rbf, cutoff, gamma)
    native.invoke("cg_edge_geom_fwd", ctypes.byref(a), rbf.data_ptr(), env.data_ptr(), _stream())
    return rbf, env


@torch.library.custom_op("cg_b200::edge_geom_bwd1", mutates_args=())
def edge_geom_bwd1(pos: Tensor, nbr: Tensor, rev_ptr: Tensor, rev_idx: Tensor, g_rbf: Tensor, g_env: Tensor,
                   n_rbf: int, cutoff: float, gamma: float) -> Tensor:
    """g_pos for cotangents (g_rbf, g_env) of edge_geom's outputs."""
    pos, g_rbf, g_env = (cgnn._f32(t, "edge_geom_bwd1") for t in (pos, g_rbf, g_env))
    gvec = torch.empty(nbr.numel(), 3, device=pos.device)
    g_pos = torch.empty_like(pos)
    a = _geom(pos, nbr, rev_ptr, rev_idx, n_rbf, cutoff, gamma)
    native.invoke("cg_edge_geom_bwd1", ctypes.byref(a), g_rbf.data_ptr(), g_env.data_ptr(), gvec.data_ptr(),
                  g_pos.data_ptr(), _stream())
    return g_pos


@torch.library.custom_op("cg_b200::edge_geom_bwd2", mutates_args=())
def edge_geom_bwd2(pos: Tensor, nbr: Tensor, rev_ptr: Tensor, rev_idx: Tensor, g_rbf: Tensor, g_env: Tensor,
                   h_pos: Tensor, n_rbf: int, cutoff: float, gamma: float) -> tuple[Tensor, Tensor, Tensor]:
    """(d pos, d g_rbf, d g_env) of <h_pos, edge_geom_bwd1(...)>."""
    pos, g_rbf, g_env, h_pos = (cgnn._f32(t, "edge_geom_bwd2") for t in (pos, g_rbf, g_env, h_pos))
    e = nbr.numel()
    gvec = torch.empty(e, 3, device=pos.device)
    d_pos, d_g_rbf, d_g_env = torch.empty_like(pos), torch.empty(e, n_rbf, device=pos.device), torch.empty(
        e, device=pos.device)
    a = _geom(pos, nbr, rev_ptr, rev_idx, n_rbf, cutoff, gamma)
    native.invoke("cg_edge_geom_bwd2", ctypes.byref(a), g_rbf.data_ptr(), g_env.data_ptr(), h_pos.data_ptr(),
                  gvec.data_ptr(), d_pos.data_ptr(), d_g_rbf.data_ptr(), d_g_env.data_ptr(), _stream())
    return d_pos, d_g_rbf, d_g_env


@edge_geom.register_fake
def _edge_geom_fake(pos, nbr, rev_ptr, rev_idx, n_rbf, cutoff, gamma):
    e = nbr.numel()
    return _empty(pos, e, n_rbf), _empty(pos, e)


@edge_geom_bwd1.register_fake
def _edge_geom_bwd1_fake(pos, nbr, rev_ptr, rev_idx, g_rbf, g_env, n_rbf, cutoff, gamma):
    return torch.empty_like(pos, memory_format=torch.contiguous_format)


@edge_geom_bwd2.register_fake
def _edge_geom_bwd2_fake(pos, nbr, rev_ptr, rev_idx, g_rbf, g_env, h_pos, n_rbf, cutoff, gamma):
    e = nbr.numel()
    return torch.empty_like(pos, memory_format=torch.contiguous_format), _empty(pos, e, n_rbf), _empty(pos, e)


def _geom_setup(ctx, inputs, output):
    pos, nbr, rev_ptr, rev_idx, n_rbf, cutoff, gamma = inputs
    ctx.save_for_backward(pos, nbr, rev_ptr, rev_idx)
    ctx.meta = (n_rbf, cutoff, gamma)
    ctx.set_materialize_grads(True)


def _geom_backward(ctx, g_rbf, g_env):
    pos, nbr, rev_ptr, rev_idx = ctx.saved_tensors
    return (edge_geom_bwd1(pos, nbr, rev_ptr, rev_idx, g_rbf, g_env, *ctx.meta), None, None, None, None, None, None)


def _geom_bwd1_setup(ctx, inputs, output):
    pos, nbr, rev_ptr, rev_idx, g_rbf, g_env, n_rbf, cutoff, gamma = inputs
    ctx.save_for_backward(pos, nbr, rev_ptr, rev_idx, g_rbf, g_env)
    ctx.meta = (n_rbf, cutoff, gamma)


def _geom_bwd1_backward(ctx, h_pos):
    pos, nbr, rev_ptr, rev_idx, g_rbf, g_env = ctx.saved_tensors
    d_pos, d_g_rbf, d_g_env = edge_geom_bwd2(pos, nbr, rev_ptr, rev_idx, g_rbf, g_env, h_pos, *ctx.meta)
    return d_pos, None, None, None, d_g_rbf, d_g_env, None, None, None


edge_geom.register_autograd(_geom_backward, setup_context=_geom_setup)
edge_geom_bwd1.register_autograd(_geom_bwd1_backward, setup_context=_geom_bwd1_setup)


# ---------------------------------------------------------------------------
# neighbour lists
# ---------------------------------------------------------------------------


@torch.library.custom_op("cg_b200::neighbor_list", mutates_args=())
def neighbor_list(pos: Tensor, sys_ptr: Tensor, max_atoms: int, cutoff: float,
                  k: int) -> tuple[Tensor, Tensor, Tensor, Tensor]:
    """(nbr (n, k), counts (n,), rev_ptr (n + 1,), rev_idx (n*k,)) int32: the k
    nearest atoms within ``cutoff`` of each atom in its own system, ordered by
    (distance^2, index), and their reverse CSR (bit-exact, see graph.build_graph)."""
    from create_graph_b200.graph import build_graph

    g = build_graph(pos, sys_ptr, sys_ptr.shape[0] - 1, max_atoms, cutoff, k)
    return g.nbr, g.counts, g.tokens.row_ptr, g.tokens.perm


@neighbor_list.register_fake
def _neighbor_list_fake(pos, sys_ptr, max_atoms, cutoff, k):
    n = pos.shape[0]
    i32 = torch.int32
    return _empty(pos, n, k, dtype=i32), _empty(pos, n, dtype=i32), _empty(pos, n + 1, dtype=i32), _empty(
        pos, max(n * k, 1), dtype=i32)
