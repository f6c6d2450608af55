"""
Fused, twice-differentiable ops of the energy network and the modules built
from them.

Every op is an autograd Function whose forward and backward run sm_100a
kernels from libcg_b200.so. Under ``cg.create_graph`` the force pass is
autograd calling these backwards with ``create_graph=True``, and
``loss.backward()`` differentiates them once more:

- bilinear ops (``mm`` on the tcgen05 GEMM, gather / segment sum over a
  sorted CSR, envelope pooling, column scale / dot / sum) write their
  backward with ops of the same family, so their second derivative is again
  those kernels;
- nonlinear ops (edge attention, edge geometry, row normalisation, the SiLU
  derivative) have explicit backward2 kernels.

Backwards skip the gradients nobody asked for: during the force pass the
parameters' gradients are not computed (``engine_will_execute``), which
removes the weight-gradient GEMMs from it.

These Functions are the package's own fused kernels, not user
``torch.autograd.Function``s, so regions accept them on the differentiated
path (``_cg_fused``).
"""

from __future__ import annotations

import ctypes
import dataclasses
import functools
import math

import torch
from torch import Tensor, nn

from create_graph_b200 import native
from create_graph_b200.checkpoint import (
    active_recompute_cache,
    cut_forward_tensor,
    deferral_slot,
    deferred_cotangent,
    plus,
)
from create_graph_b200.compile_config import active_memory_budget, engine_will_execute, gradient_edge
from create_graph_b200.edge_attn import (
    pooled_attention_backward1,
    pooled_attention_backward2,
    pooled_attention_forward,
    token_attention_backward1,
    token_attention_backward2,
    token_attention_forward1,
)
from create_graph_b200.errors import NativeError
from create_graph_b200.gemm import ACT_ADD, ACT_SILU, ACT_SILU_GRAD, current_precision, gemm, gemm_precision

Function = torch.autograd.Function


def _stream() -> int:
    return native.stream_ptr()


class _Fused(Function):
    """Marker base: the package's fused ops (accepted on the differentiated path)."""

    _cg_fused = True


def _edges(*tensors):
    return [gradient_edge(t) if isinstance(t, Tensor) else None for t in tensors]


def _wanted(ctx, i: int) -> bool:
    """Whether input i's gradient is needed by the backward pass running now."""
    return ctx.needs_input_grad[i] and engine_will_execute(ctx.edges[i])


def _keep_precision(ctx) -> None:
    """Record the GEMM precision of a GEMM op's forward (see _at_forward_precision)."""
    ctx.precision = current_precision()


def _at_forward_precision(backward):
    """Run a GEMM op's backward, and so every op it records, at the GEMM
    precision of its forward: autograd calls backwards on its own threads,
    where the forward thread's setting is not visible."""

    @functools.wraps(backward)
    def run(ctx, *grads):
        with gemm_precision(ctx.precision):
            return backward(ctx, *grads)

    return run


def _f32(t: Tensor, name: str) -> Tensor:
    native.require_cuda(t)
    if t.dtype != torch.float32:
        raise NativeError(f"{name}: float32 expected, got {t.dtype}")
    return t if t.is_contiguous() else t.contiguous()


# ---------------------------------------------------------------------------
# GEMM family: mm(a, b) = a @ b.T on the tcgen05 kernel
# ---------------------------------------------------------------------------


def _mm_operand(t: Tensor) -> tuple[Tensor, bool]:
    """(tensor, mn_major) for a logical (rows, K) operand: row-contiguous tensors
    are K-major, transposed views of row-contiguous tensors are MN-major."""
    if t.stride(-1) == 1 and t.stride(0) >= t.shape[1]:
        return t, False
    if t.stride(0) == 1 and t.stride(1) >= t.shape[0]:
        return t.t(), True
    return t.contiguous(), False


def mm_raw(a: Tensor, b: Tensor, **kw) -> Tensor:
    A, at = _mm_operand(a)
    B, bt = _mm_operand(b)
    return gemm(A, B, a_t=at, b_t=bt, **kw)


# the deferred first-order backward inside checkpointed blocks: ops read the
# forward tensors their backward builds on through _cut, and add what
# _deferred hands them (create_graph_b200.checkpoint)
_op_slot, _cut, _deferred, _plus = deferral_slot, cut_forward_tensor, deferred_cotangent, plus


class MM(_Fused):
    """C = a @ b.T (+ add) (a (M, K), b (N, K)); backward: g @ b and g.T @ a.
    ``add`` (M, N) enters through the GEMM epilogue."""

    @staticmethod
    def forward(ctx, a, b, reuse=None, add=None):
        """reuse: (cache, key) inside a checkpointed block's VJP (_vjp_reuse)."""
        _keep_precision(ctx)
        ctx.save_for_backward(a, b)
        ctx.edges = _edges(a, b)
        if add is not None:
            return mm_raw(a, b, act=ACT_ADD, aux_in=_f32(add, "mm_add"))
        return _reused_in_rebuild(reuse, lambda: mm_raw(a, b))

    @staticmethod
    @_at_forward_precision
    def backward(ctx, g):
        a, b = ctx.saved_tensors
        ga = MM.apply(g, b.t()) if _wanted(ctx, 0) else None
        gb = MM.apply(g.t(), a.t()) if _wanted(ctx, 1) else None
        g_add = g if len(ctx.needs_input_grad) > 3 and ctx.needs_input_grad[3] else None
        return ga, gb, None, g_add


def mm(a: Tensor, b: Tensor) -> Tensor:
    return MM.apply(a, b)


def _block_slot():
    """(cache, slot) of the checkpointed block call whose forward is running
    (memory budget above 0.25), else (None, None). Ops take their slot in
    call order, the same in the call's first forward and its recomputes."""
    cache = active_recompute_cache() if active_memory_budget() > 0.25 else None
    return (cache, cache.slot()) if cache is not None else (None, None)


def _vjp_reuse(ctx, what: str):
    """(cache, key) when an op's backward runs inside its block call's VJP:
    the force pass, or the VJP's rebuild in the parameter backward, which sees
    the same inputs and cotangents. The force pass leaves its result there and
    the rebuild takes it (_reused_in_rebuild); None elsewhere."""
    cache, slot = getattr(ctx, "block", (None, None))
    if cache is None or not cache.in_vjp:
        return None
    return cache, (what, slot)


def _reused_in_rebuild(reuse, compute):
    """compute(), kept for the VJP's rebuild when ``reuse`` is set; in the
    rebuild, the force pass's result (an alias of its storage, a tensor of
    this node's own; bit for bit what compute() gives), which is then dropped."""
    if reuse is None:
        return compute()
    cache, key = reuse
    kept = cache.slots.pop(key, None)
    if kept is not None:
        return kept.detach()
    out = compute()
    cache.slots[key] = out.detach()
    return out


def colsum_raw(x: Tensor) -> Tensor:
    """out[c] = sum_r x[r, c] (deterministic two-pass reduction)."""
    x = _f32(x, "colsum")
    out = torch.empty(x.shape[1], device=x.device)
    nbytes = native.lib().cg_colsum_scratch_bytes(x.shape[0], x.shape[1])
    scratch = torch.empty(max(nbytes // 4, 1), device=x.device)
    native.call("cg_colsum", x.data_ptr(), x.stride(0), x.shape[0], x.shape[1], out.data_ptr(), 0,
                scratch.data_ptr(), _stream())
    return out


class ColSum(_Fused):
    """out[c] = sum_r x[r, c] (deterministic two-pass reduction)."""

    @staticmethod
    def forward(ctx, x):
        ctx.rows = x.shape[0]
        return colsum_raw(x)

    @staticmethod
    def backward(ctx, h):
        return h.expand(ctx.rows, h.shape[0])


class ColDot(_Fused):
    """out[c] = sum_r a[r, c] b[r, c]."""

    @staticmethod
    def forward(ctx, a, b):
        a, b = _f32(a, "coldot"), _f32(b, "coldot")
        ctx.save_for_backward(a, b)
        out = torch.empty(a.shape[1], device=a.device)
        nbytes = native.lib().cg_coldot_scratch_bytes(a.shape[0], a.shape[1])
        scratch = torch.empty(max(nbytes // 4, 1), device=a.device)
        native.call("cg_coldot", a.data_ptr(), b.data_ptr(), a.shape[0], a.shape[1], out.data_ptr(), 0,
                    scratch.data_ptr(), _stream())
        return out

    @staticmethod
    def backward(ctx, h):
        a, b = ctx.saved_tensors
        ga = ScaleShift.apply(b, h, None) if ctx.needs_input_grad[0] else None
        gb = ScaleShift.apply(a, h, None) if ctx.needs_input_grad[1] else None
        return ga, gb


class ScaleShift(_Fused):
    """y[r, c] = x[r, c] * gamma[c] + beta[c] (beta optional).

    When x is a row normalisation of ``src`` (LayerNorm) and the active memory
    budget is 0.25 or less, x is not kept: the gamma gradient rebuilds it from
    ``src`` (which the residual stream keeps alive anyway) with the same
    normalisation kernel, bit for bit."""

    @staticmethod
    def forward(ctx, x, gamma, beta, src=None, eps=None):
        x = _f32(x, "scale_shift")

        def compute():
            out = torch.empty_like(x)
            native.call("cg_scale_shift", x.data_ptr(), native.ptr(gamma), native.ptr(beta), out.data_ptr(),
                        x.shape[0], x.shape[1], _stream())
            return out

        # a LayerNorm's output inside checkpointed blocks at a budget of 0.5 or
        # more: the recomputes take the first forward's
        out = _kept_across_recomputes(compute, _block_slot() if src is not None else (None, None), min_budget=0.5)
        ctx.rebuild = src is not None and active_memory_budget() <= 0.25
        ctx.eps = eps
        ctx.save_for_backward(src if ctx.rebuild else x, gamma)
        ctx.edges = _edges(x, gamma, beta)
        ctx.has_beta = beta is not None
        ctx.op = _op_slot()
        return out

    @staticmethod
    def backward(ctx, g):
        kept, gamma = ctx.saved_tensors
        role = "src" if ctx.rebuild else "x"
        c = _deferred(ctx, role)
        gx = ScaleShift.apply(g, gamma, None) if _wanted(ctx, 0) else None
        gg = None
        if _wanted(ctx, 1):
            kept = _cut(ctx, role, kept)
            x = RowNorm.apply(kept, ctx.eps) if ctx.rebuild else kept
            gg = ColDot.apply(g, x)
        gb = ColSum.apply(g) if ctx.has_beta and _wanted(ctx, 2) else None
        if ctx.rebuild:
            return gx, gg, gb, c, None
        return _plus(gx, c), gg, gb, None, None


# ---------------------------------------------------------------------------
# Linear layers (bias and SiLU fused into the GEMM epilogue)
# ---------------------------------------------------------------------------


def _linear_backward(ctx, g, x, w, has_bias):
    """(gx, gw, gb); gx takes the deferred cotangent of x in its epilogue, gw
    reads x through _cut."""
    c = _deferred(ctx, "x")
    gx = MM.apply(g, w.t(), _vjp_reuse(ctx, "gx"), c) if _wanted(ctx, 0) else None
    gw = MM.apply(g.t(), _cut(ctx, "x", x).t()) if _wanted(ctx, 1) else None
    gb = ColSum.apply(g) if has_bias and _wanted(ctx, 2) else None
    return gx, gw, gb


class LinearFn(_Fused):
    """y = x @ w.T + b."""

    @staticmethod
    def forward(ctx, x, w, b):
        _keep_precision(ctx)
        ctx.save_for_backward(x, w)
        ctx.edges = _edges(x, w, b)
        ctx.has_bias = b is not None
        # inside checkpointed blocks at a budget of 0.5 or more, the recomputes
        # take the first forward's projection (the q/k/v rows: 3C floats per atom)
        ctx.block = _block_slot()
        ctx.op = _op_slot()
        return _kept_across_recomputes(lambda: mm_raw(x, w, bias=b), ctx.block, min_budget=0.5)

    @staticmethod
    @_at_forward_precision
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        return _linear_backward(ctx, g, x, w, ctx.has_bias)


def _kept_across_recomputes(compute, where, min_budget: float | None = None):
    """The op's output from ``compute()``; inside a checkpointed block call
    (``where`` = _block_slot()) whose memory budget is above 0.25 (and at
    least ``min_budget`` when given,
    for outputs that cost more memory per microsecond saved), a recompute on
    the same inputs takes what the call's first forward computed instead (bit
    for bit the same), as an alias of its storage: each recompute's node gets
    its own tensor, and nothing writes these outputs in place. For ops whose
    backward reads only their inputs, so the kept output is all a recompute
    needs."""
    cache, slot = where
    if cache is None or (min_budget is not None and active_memory_budget() < min_budget):
        return compute()
    kept = cache.slots.get(slot)
    if kept is not None:
        return tuple(t.detach() for t in kept) if isinstance(kept, tuple) else kept.detach()
    out = compute()
    cache.slots[slot] = tuple(t.detach() for t in out) if isinstance(out, tuple) else out.detach()
    return out


class LinearResidualFn(_Fused):
    """y = r + x @ w.T + b: the residual add in the GEMM epilogue (reads r once,
    no separate (rows, out) add); r's gradient is g itself."""

    @staticmethod
    def forward(ctx, x, w, b, r):
        _keep_precision(ctx)
        ctx.save_for_backward(x, w)
        ctx.edges = _edges(x, w, b, r)
        ctx.has_bias = b is not None
        ctx.block = _block_slot()
        ctx.op = _op_slot()
        return _kept_across_recomputes(
            lambda: mm_raw(x, w, bias=b, act=ACT_ADD, aux_in=_f32(r, "linear_residual")), ctx.block)

    @staticmethod
    @_at_forward_precision
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        return (*_linear_backward(ctx, g, x, w, ctx.has_bias), g if ctx.needs_input_grad[3] else None)


class SiluGrad(_Fused):
    """out = g * silu'(z)."""

    @staticmethod
    def forward(ctx, g, z):
        g, z = _f32(g, "silu_grad"), _f32(z, "silu_grad")
        out = torch.empty_like(g)
        native.call("cg_silu_grad", g.data_ptr(), z.data_ptr(), out.data_ptr(), g.numel(), _stream())
        ctx.save_for_backward(g, z)
        return out

    @staticmethod
    def backward(ctx, h):
        g, z = ctx.saved_tensors
        dg = SiluGrad.apply(h, z) if ctx.needs_input_grad[0] else None
        dz = None
        if ctx.needs_input_grad[1]:
            h = _f32(h, "silu_grad2")
            dz = torch.empty_like(h)
            native.call("cg_silu_grad2", h.data_ptr(), g.data_ptr(), z.data_ptr(), dz.data_ptr(), h.numel(),
                        _stream())
        return dg, dz


class Silu(_Fused):
    """y = silu(z), elementwise (rebuilds a SiLU activation that was not kept)."""

    @staticmethod
    def forward(ctx, z):
        z = _f32(z, "silu")
        out = torch.empty_like(z)
        native.call("cg_silu", z.data_ptr(), out.data_ptr(), z.numel(), _stream())
        ctx.save_for_backward(z)
        return out

    @staticmethod
    def backward(ctx, g):
        (z,) = ctx.saved_tensors
        return SiluGrad.apply(g, z)


class LinearSiluFn(_Fused):
    """(y, z) with z = x @ w.T + b and y = silu(z), from one GEMM."""

    @staticmethod
    def forward(ctx, x, w, b):
        _keep_precision(ctx)

        def compute():
            z = torch.empty(x.shape[0], w.shape[0], device=x.device)
            return mm_raw(x, w, bias=b, act=ACT_SILU, aux_out=z), z

        # inside checkpointed blocks: the recomputes take the first forward's
        # (y, z) at a budget of 0.5 or more, and its backward's input gradient
        # is kept for the VJP's rebuild
        ctx.block = _block_slot()
        y, z = _kept_across_recomputes(compute, ctx.block, min_budget=0.5)
        ctx.save_for_backward(x, w, z)
        ctx.edges = _edges(x, w, b)
        ctx.has_bias = b is not None
        ctx.op = _op_slot()
        # z is usually unused: its gradient arrives as None, not as a zero-filled
        # (rows, out) tensor added to the SiLU gradient
        ctx.set_materialize_grads(False)
        return y, z

    @staticmethod
    @_at_forward_precision
    def backward(ctx, gy, gz):
        x, w, z = ctx.saved_tensors
        gz = _plus(gz, _deferred(ctx, "z"))
        g = None
        if gy is not None:
            g = SiluGrad.apply(gy, _cut(ctx, "z", z))
        if gz is not None:
            g = gz if g is None else g + gz
        if g is None:
            return _deferred(ctx, "x"), None, None
        return _linear_backward(ctx, g, x, w, ctx.has_bias)


class MMSiluGrad(_Fused):
    """out = (g @ w) * silu'(z): the input gradient of a linear layer applied
    to silu(z), taken straight to z (the SiLU derivative in the GEMM epilogue)."""

    @staticmethod
    def forward(ctx, g, w, z, keep_u=False, reuse=None):
        """reuse: (cache, key) inside a checkpointed block's VJP (_vjp_reuse)."""
        _keep_precision(ctx)
        z = _f32(z, "mm_silu_grad")
        # u = g @ w, the second-order term's factor, comes out of the same
        # epilogue when the caller builds a graph through this node (keep_u);
        # a result taken from the force pass comes without it (the backward
        # then forms u with one GEMM)
        kept = reuse is not None and reuse[1] in reuse[0].slots
        u = torch.empty_like(z) if keep_u and not kept else None
        out = _reused_in_rebuild(reuse, lambda: mm_raw(g, w.t(), act=ACT_SILU_GRAD, aux_in=z, aux_out=u))
        ctx.save_for_backward(g, w, z, u)
        ctx.edges = _edges(g, w, z)
        return out

    @staticmethod
    @_at_forward_precision
    def backward(ctx, h):
        g, w, z, u = ctx.saved_tensors
        s = SiluGrad.apply(h, z) if (_wanted(ctx, 0) or _wanted(ctx, 1)) else None  # h * silu'(z)
        dg = MM.apply(s, w) if _wanted(ctx, 0) else None
        dw = MM.apply(g.t(), s.t()) if _wanted(ctx, 1) else None
        dz = None
        if _wanted(ctx, 2):
            h = _f32(h, "mm_silu_grad2")
            if u is None:
                u = mm_raw(g, w.t())  # g @ w
            dz = torch.empty_like(h)
            native.call("cg_silu_grad2", h.data_ptr(), u.data_ptr(), z.data_ptr(), dz.data_ptr(), h.numel(),
                        _stream())
        return dg, dw, dz, None, None


class SiluLinearResidualFn(_Fused):
    """out = r + silu(z) @ w.T + b, given y = silu(z) (written by the producing
    GEMM's epilogue). Backward sends the gradient to z through MMSiluGrad (one
    GEMM with the SiLU derivative in its epilogue) and none to y, so the
    producer's backward runs no separate SiLU-gradient pass. y must have no
    other consumer; its second-order terms still flow through the weight
    gradient, which reads y.

    Memory budget (the active region's CompileConfig.memory_budget): below 1
    the second-order factor u = g @ w is not kept by the force pass (the
    parameter backward recomputes it with one GEMM); at 0.5 or less y is not
    kept either (the weight gradient rebuilds it from z, bit for bit)."""

    @staticmethod
    def forward(ctx, y, z, w, b, r):
        _keep_precision(ctx)
        budget = active_memory_budget()
        ctx.keep_u = budget >= 1.0
        ctx.save_for_backward(y if budget > 0.5 else None, z, w)
        ctx.edges = _edges(y, z, w, b, r)
        ctx.has_bias = b is not None
        ctx.block = _block_slot()
        ctx.op = _op_slot()
        return _kept_across_recomputes(
            lambda: mm_raw(y, w, bias=b, act=ACT_ADD, aux_in=_f32(r, "silu_linear_residual")), ctx.block)

    @staticmethod
    @_at_forward_precision
    def backward(ctx, g):
        y, z, w = ctx.saved_tensors
        # grad mode is on here exactly when this backward is being recorded
        # (create_graph), i.e. when MMSiluGrad's own backward will run
        keep_u = ctx.keep_u and torch.is_grad_enabled()
        # below a memory budget of 1 (no u kept) the VJP's rebuild takes the
        # force pass's gz; at 1 the rebuild runs the GEMM again for its u
        reuse = None if ctx.keep_u else _vjp_reuse(ctx, "gz")
        # deferred cotangents: z's joins gz; y's is y's gradient (through the
        # producer's SiLU derivative)
        cy, cz = _deferred(ctx, "y"), _deferred(ctx, "z")
        gz = _plus(MMSiluGrad.apply(g, w, _cut(ctx, "z", z), keep_u, reuse), cz) if _wanted(ctx, 1) else None
        gw = None
        if _wanted(ctx, 2):
            gw = MM.apply(g.t(), (_cut(ctx, "y", y) if y is not None else Silu.apply(_cut(ctx, "z", z))).t())
        gb = ColSum.apply(g) if ctx.has_bias and _wanted(ctx, 3) else None
        gr = g if ctx.needs_input_grad[4] else None
        return cy, gz, gw, gb, gr


class SplitCols(_Fused):
    """The column blocks x[:, i*width:(i+1)*width] of x as views (no copy);
    backward: the blocks' gradients side by side (one concatenation instead of
    a zero-filled full-width gradient per block summed by the engine)."""

    @staticmethod
    def forward(ctx, x, width):
        ctx.width = width
        ctx.shape = x.shape
        ctx.set_materialize_grads(False)
        return tuple(x[:, i * width:(i + 1) * width] for i in range(x.shape[1] // width))

    @staticmethod
    def backward(ctx, *grads):
        some = next((g for g in grads if g is not None), None)
        if some is None:
            return None, None
        parts = [g if g is not None else torch.zeros(ctx.shape[0], ctx.width, device=some.device, dtype=some.dtype)
                 for g in grads]
        return torch.cat(parts, dim=1), None


# ---------------------------------------------------------------------------
# Row normalisation (LayerNorm without its affine part)
# ---------------------------------------------------------------------------


class RowNorm(_Fused):
    @staticmethod
    def forward(ctx, x, eps):
        x = _f32(x, "rownorm")
        out = torch.empty_like(x)
        native.call("cg_rownorm_fwd", x.data_ptr(), x.shape[0], x.shape[1], eps, out.data_ptr(), None,
                    _stream())
        ctx.save_for_backward(x)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, g):
        (x,) = ctx.saved_tensors
        return RowNormGrad.apply(g, x, ctx.eps, None), None


class BranchNorm(_Fused):
    """(x, rownorm(x)): a residual branch point. Backward sums the two branch
    gradients inside the row-normalisation backward kernel (one pass, no
    separate add of the residual gradient)."""

    @staticmethod
    def forward(ctx, x, eps):
        x = _f32(x, "rownorm")

        def compute():
            out = torch.empty_like(x)
            native.call("cg_rownorm_fwd", x.data_ptr(), x.shape[0], x.shape[1], eps, out.data_ptr(), None,
                        _stream())
            return out

        # inside checkpointed blocks at a budget of 0.5 or more the recomputes
        # take the first forward's normalised rows
        out = _kept_across_recomputes(compute, _block_slot(), min_budget=0.5)
        ctx.save_for_backward(x)
        ctx.eps = eps
        ctx.set_materialize_grads(False)
        ctx.op = _op_slot()
        return x.view_as(x), out

    @staticmethod
    def backward(ctx, g_x, g_norm):
        (x,) = ctx.saved_tensors
        c = _deferred(ctx, "x")
        if g_norm is None:
            return _plus(g_x, c), None
        return _plus(RowNormGrad.apply(g_norm, _cut(ctx, "x", x), ctx.eps, g_x), c), None


class RowNormGrad(_Fused):
    """gx = J(x)^T g (+ add) of the row normalisation; backward is the bwd2
    kernel (and add's gradient is h itself)."""

    @staticmethod
    def forward(ctx, g, x, eps, add):
        g, x = _f32(g, "rownorm_bwd1"), _f32(x, "rownorm_bwd1")
        if add is not None:
            add = _f32(add, "rownorm_bwd1")
        out = torch.empty_like(g)
        native.call("cg_rownorm_bwd1_add", x.data_ptr(), g.data_ptr(), native.ptr(add), x.shape[0], x.shape[1],
                    eps, out.data_ptr(), _stream())
        ctx.save_for_backward(g, x)
        ctx.eps = eps
        return out

    @staticmethod
    def backward(ctx, h):
        g, x = ctx.saved_tensors
        h = _f32(h, "rownorm_bwd2")
        dx, dg = torch.empty_like(x), torch.empty_like(g)
        native.call("cg_rownorm_bwd2", x.data_ptr(), g.data_ptr(), h.data_ptr(), x.shape[0], x.shape[1], ctx.eps,
                    dx.data_ptr(), dg.data_ptr(), _stream())
        return dg, dx, None, h if ctx.needs_input_grad[3] else None


# ---------------------------------------------------------------------------
# Gather / segment sum over a sorted CSR
# ---------------------------------------------------------------------------


@dataclasses.dataclass
class Csr:
    """A many-to-one map: element e goes to row index[e] (-1: nowhere). row_ptr
    (rows + 1) and perm (the elements grouped by row, ascending within a row)
    make the reduction direction a fixed-order segment sum."""

    index: Tensor      # (elements,) int32
    row_ptr: Tensor    # (rows + 1,) int32
    perm: Tensor       # (elements mapped somewhere,) int32
    rows: int

    @staticmethod
    def from_index(index: Tensor, rows: int) -> Csr:
        """Build on the index's device, deterministically. On a CUDA device the
        kernels build it without reading anything back to the host (capturable
        in a CUDA graph); perm then has one slot per element, -1 past the
        mapped ones. A CPU index takes a stable torch sort."""
        if index.is_cuda:
            index = index.to(torch.int32).contiguous()
            row_ptr = torch.empty(rows + 1, dtype=torch.int32, device=index.device)
            perm = torch.empty(max(index.numel(), 1), dtype=torch.int32, device=index.device)
            native.call("cg_csr_from_index", index.data_ptr(), index.numel(), rows, row_ptr.data_ptr(),
                        perm.data_ptr(), _stream())
            return Csr(index, row_ptr, perm, rows)
        index = index.to(torch.int64)
        valid = index >= 0
        order = torch.argsort(torch.where(valid, index, rows), stable=True)
        counts = torch.bincount(index[valid], minlength=rows)
        row_ptr = torch.zeros(rows + 1, dtype=torch.int64, device=index.device)
        row_ptr[1:] = torch.cumsum(counts, 0)
        nnz = int(valid.sum())
        return Csr(index.to(torch.int32), row_ptr.to(torch.int32), order[:nnz].to(torch.int32).contiguous(), rows)


def gather_raw(src: Tensor, csr: Csr) -> Tensor:
    src = _f32(src, "gather_rows")
    out = torch.empty(csr.index.shape[0], src.shape[1], device=src.device)
    native.call("cg_gather_rows", src.data_ptr(), src.stride(0), csr.index.data_ptr(), out.shape[0], src.shape[1],
                out.data_ptr(), out.stride(0), _stream())
    return out


def segment_sum_raw(src: Tensor, csr: Csr) -> Tensor:
    src = _f32(src, "segment_sum")
    out = torch.empty(csr.rows, src.shape[1], device=src.device)
    native.call("cg_segment_sum", src.data_ptr(), src.stride(0), csr.row_ptr.data_ptr(), csr.perm.data_ptr(),
                csr.rows, src.shape[1], out.data_ptr(), out.stride(0), 0, _stream())
    return out


class Gather(_Fused):
    """out[e] = src[csr.index[e]]; backward: segment sum."""

    @staticmethod
    def forward(ctx, src, csr):
        ctx.csr = csr
        return gather_raw(src, csr)

    @staticmethod
    def backward(ctx, g):
        return SegmentSum.apply(g, ctx.csr), None


class SegmentSum(_Fused):
    """out[r] = sum of src[e] over index[e] == r, in ascending e; backward: gather."""

    @staticmethod
    def forward(ctx, src, csr):
        ctx.csr = csr
        return segment_sum_raw(src, csr)

    @staticmethod
    def backward(ctx, g):
        return Gather.apply(g, ctx.csr), None


# ---------------------------------------------------------------------------
# Envelope pooling over the k tokens of each atom
# ---------------------------------------------------------------------------


class Pool(_Fused):
    """m[n, c] = sum_s w[n, s] x[n, s, c]."""

    @staticmethod
    def forward(ctx, x, w):
        x, w = _f32(x, "pool"), _f32(w, "pool")
        n, k, c = x.shape
        out = torch.empty(n, c, device=x.device)
        native.call("cg_pool", x.data_ptr(), w.data_ptr(), n, k, c, out.data_ptr(), _stream())
        ctx.save_for_backward(x, w)
        return out

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        gx = Outer.apply(w, g) if ctx.needs_input_grad[0] else None
        gw = Dot.apply(g, x) if ctx.needs_input_grad[1] else None
        return gx, gw


class Outer(_Fused):
    """y[n, s, c] = w[n, s] g[n, c]."""

    @staticmethod
    def forward(ctx, w, g):
        w, g = _f32(w, "pool_outer"), _f32(g, "pool_outer")
        n, k = w.shape
        out = torch.empty(n, k, g.shape[1], device=w.device)
        native.call("cg_pool_outer", w.data_ptr(), g.data_ptr(), n, k, g.shape[1], out.data_ptr(), _stream())
        ctx.save_for_backward(w, g)
        return out

    @staticmethod
    def backward(ctx, h):
        w, g = ctx.saved_tensors
        gw = Dot.apply(g, h) if ctx.needs_input_grad[0] else None
        gg = Pool.apply(h, w) if ctx.needs_input_grad[1] else None
        return gw, gg


class Dot(_Fused):
    """y[n, s] = sum_c g[n, c] x[n, s, c]."""

    @staticmethod
    def forward(ctx, g, x):
        g, x = _f32(g, "pool_dot"), _f32(x, "pool_dot")
        n, k, c = x.shape
        out = torch.empty(n, k, device=x.device)
        native.call("cg_pool_dot", g.data_ptr(), x.data_ptr(), n, k, c, out.data_ptr(), _stream())
        ctx.save_for_backward(g, x)
        return out

    @staticmethod
    def backward(ctx, h):
        g, x = ctx.saved_tensors
        gg = Pool.apply(x, h) if ctx.needs_input_grad[0] else None
        gx = Outer.apply(h, g) if ctx.needs_input_grad[1] else None
        return gg, gx


# ---------------------------------------------------------------------------
# Edge geometry
# ---------------------------------------------------------------------------


@dataclasses.dataclass
class NeighborGraph:
    """Padded neighbour layout of a batch: slot e = i*k + s holds neighbour
    nbr[i, s] of atom i (-1 past counts[i]); ``tokens`` maps slots to their
    neighbour (the gather of per-atom features into edge tokens) and back."""

    nbr: Tensor        # (n, k) int32
    counts: Tensor     # (n,) int32
    tokens: Csr        # index = nbr.flatten(); rows = n
    k: int

    @property
    def n_atoms(self) -> int:
        return self.nbr.shape[0]


def _geom_args(pos: Tensor, graph: NeighborGraph, n_rbf: int, cutoff: float, gamma: float):
    a = native.GeomArgs()
    a.pos = pos.data_ptr()
    a.nbr = graph.nbr.data_ptr()
    a.rev_ptr = graph.tokens.row_ptr.data_ptr()
    a.rev_idx = graph.tokens.perm.data_ptr()
    a.n_atoms = graph.n_atoms
    a.k = graph.k
    a.n_rbf = n_rbf
    a.cutoff = cutoff
    a.gamma = gamma
    return a


class EdgeGeometry(_Fused):
    """(rbf (n*k, n_rbf), env (n*k,)) of the neighbour edges of pos."""

    @staticmethod
    def forward(ctx, pos, graph, n_rbf, cutoff, gamma):
        pos = _f32(pos, "edge_geom")
        e = graph.n_atoms * graph.k
        rbf = torch.empty(e, n_rbf, device=pos.device)
        env = torch.empty(e, device=pos.device)
        args = _geom_args(pos, graph, n_rbf, cutoff, gamma)
        native.invoke("cg_edge_geom_fwd", ctypes.byref(args), rbf.data_ptr(), env.data_ptr(), _stream())
        ctx.save_for_backward(pos)
        ctx.meta = (graph, n_rbf, cutoff, gamma)
        return rbf, env

    @staticmethod
    def backward(ctx, g_rbf, g_env):
        (pos,) = ctx.saved_tensors
        graph, n_rbf, cutoff, gamma = ctx.meta
        if g_rbf is None:
            g_rbf = torch.zeros(graph.n_atoms * graph.k, n_rbf, device=pos.device)
        return EdgeGeometryGrad.apply(pos, g_rbf, g_env, ctx.meta), None, None, None, None


class EdgeGeometryGrad(_Fused):
    """g_pos of (g_rbf, g_env); backward: the second-derivative kernel."""

    @staticmethod
    def forward(ctx, pos, g_rbf, g_env, meta):
        graph, n_rbf, cutoff, gamma = meta
        g_rbf = _f32(g_rbf, "edge_geom_bwd1")
        g_env = None if g_env is None else _f32(g_env, "edge_geom_bwd1")
        gvec = torch.empty(graph.n_atoms * graph.k, 3, device=pos.device)
        g_pos = torch.empty_like(pos)
        args = _geom_args(pos, graph, n_rbf, cutoff, gamma)
        native.invoke("cg_edge_geom_bwd1", ctypes.byref(args), g_rbf.data_ptr(), native.ptr(g_env), gvec.data_ptr(),
                      g_pos.data_ptr(), _stream())
        ctx.save_for_backward(pos, g_rbf, g_env)
        ctx.meta = meta
        return g_pos

    @staticmethod
    def backward(ctx, h):
        pos, g_rbf, g_env = ctx.saved_tensors
        graph, n_rbf, cutoff, gamma = ctx.meta
        h = _f32(h, "edge_geom_bwd2")
        e = graph.n_atoms * graph.k
        gvec = torch.empty(e, 3, device=pos.device)
        d_pos = torch.empty_like(pos)
        d_g_rbf = torch.empty(e, n_rbf, device=pos.device)
        d_g_env = torch.empty(e, device=pos.device)
        args = _geom_args(pos, graph, n_rbf, cutoff, gamma)
        native.invoke("cg_edge_geom_bwd2", ctypes.byref(args), g_rbf.data_ptr(), native.ptr(g_env), h.data_ptr(),
                      gvec.data_ptr(), d_pos.data_ptr(), d_g_rbf.data_ptr(), d_g_env.data_ptr(), _stream())
        return d_pos, d_g_rbf, (d_g_env if g_env is not None else None), None


# ---------------------------------------------------------------------------
# Edge attention over gathered tokens
# ---------------------------------------------------------------------------


class TokenAttention(_Fused):
    """Attention among the k edge tokens of each atom.

    Token (n, s) is [q | k | v] of atom graph.tokens.index[n*k + s], read by
    the kernels straight from the per-atom qkv rows (n_atoms, 3*h*d); bias
    (n*k, h) is the per-key additive bias and keys past graph.counts[n] are
    masked. Returns the token outputs (n, k, h*d), heads concatenated. The
    per-token q/k/v gradients are reduced to atoms by the deterministic CSR
    segment sum (the transpose of the gather). ``precision`` ("fp32" or
    "tf32") selects the kernels' tensor-core product precision.
    """

    @staticmethod
    def forward(ctx, qkv, bias, graph, heads, scale, precision="fp32"):
        meta = (graph, heads, scale, precision)
        out, lse = token_attention_forward1(qkv, bias, graph.tokens.index, graph.counts, graph.k, heads, scale,
                                            precision)
        ctx.save_for_backward(qkv, bias, lse)
        ctx.meta = meta
        return out

    @staticmethod
    def backward(ctx, g):
        qkv, bias, lse = ctx.saved_tensors
        d_qkv, dbias = TokenAttentionGrad.apply(qkv, bias, lse, g, ctx.meta)
        return d_qkv, dbias, None, None, None, None


class TokenAttentionGrad(_Fused):
    """backward1 of TokenAttention (per-atom q/k/v and bias gradients); its
    backward is the backward2 kernel followed by the same segment sum."""

    @staticmethod
    def forward(ctx, qkv, bias, lse, g, meta):
        graph, heads, scale, precision = meta
        dtok, dbias = token_attention_backward1(qkv, bias, lse, g, graph.tokens.index, graph.counts, graph.k,
                                                heads, scale, precision)
        ctx.save_for_backward(qkv, bias, lse, g)
        ctx.meta = meta
        return segment_sum_raw(dtok, graph.tokens), dbias

    @staticmethod
    def backward(ctx, h_qkv, h_bias):
        qkv, bias, lse, g = ctx.saved_tensors
        graph, heads, scale, precision = ctx.meta
        if h_qkv is None:
            h_qkv = torch.zeros_like(qkv)
        dtok, dbias, dg = token_attention_backward2(qkv, bias, lse, g, h_qkv, h_bias, graph.tokens.index,
                                                    graph.counts, graph.k, heads, scale, precision)
        return segment_sum_raw(dtok, graph.tokens), dbias, None, dg, None


def _pooled_qkv_grad(dqk: Tensor, wv: Tensor, dm: Tensor, graph, heads: int, into: Tensor | None = None) -> Tensor:
    """Per-atom q/k/v gradient (n_atoms, 3C) of the pooled attention: the
    per-token [dq | dk] rows and the rank-one v rows wv[token, h] * dm[atom of
    token, h], each reduced to atoms in a fixed order; added to ``into`` (a
    gradient of the caller's own, overwritten) when given."""
    csr = graph.tokens
    C = dm.shape[1]
    d = C // heads
    acc = int(into is not None and into.is_contiguous() and into.shape == (csr.rows, 3 * C))
    out = into if acc else torch.empty(csr.rows, 3 * C, device=dm.device)
    native.call("cg_segment_sum", dqk.data_ptr(), dqk.stride(0), csr.row_ptr.data_ptr(), csr.perm.data_ptr(),
                csr.rows, 2 * C, out.data_ptr(), out.stride(0), acc, _stream())
    dm = _f32(dm, "segment_sum_scaled")
    native.call("cg_segment_sum_scaled", wv.data_ptr(), dm.data_ptr(), dm.stride(0), graph.k, heads, d,
                csr.row_ptr.data_ptr(), csr.perm.data_ptr(), csr.rows, out.data_ptr() + 2 * C * out.element_size(),
                out.stride(0), acc, _stream())
    return out if acc or into is None else out + into


class PooledTokenAttention(_Fused):
    """m[n] = sum_i env[n*k + i] * (attention output of token (n, i)): the
    TokenAttention above followed by Pool, as one fused op whose kernels never
    form the (n, k, h*d) token outputs. Returns (n, h*d), heads concatenated.
    ``precision`` ("fp32" or "tf32") selects the product precision."""

    @staticmethod
    def forward(ctx, qkv, bias, env, graph, heads, scale, precision="fp32"):
        meta = (graph, heads, scale, precision)
        args = (graph.tokens.index, graph.counts, graph.k, heads)
        # inside a checkpointed block call, a recompute on the same inputs
        # reuses the first forward's softmax statistics (lse, w) and its
        # output (an alias of its storage, a tensor of this node's own), bit
        # for bit the same; a memory budget of 0.25 or less keeps nothing
        # across recomputes
        cache = active_recompute_cache() if active_memory_budget() > 0.25 else None
        slot = cache.slot() if cache is not None else None
        kept = cache.slots.get(slot) if cache is not None else None
        if kept is not None and kept[1].shape == (graph.n_atoms, heads, graph.k):
            lse, w, first = kept
            out = first.detach()
        else:
            out, lse, w = pooled_attention_forward(qkv, bias, env, *args[:3], heads, scale, precision)
            if cache is not None:
                cache.slots[slot] = (lse, w, out.detach())
        ctx.save_for_backward(qkv, bias, env, lse, w)
        ctx.meta = meta
        ctx.cache, ctx.slot = cache, slot
        ctx.op = _op_slot()
        return out

    @staticmethod
    def backward(ctx, dm):
        qkv, bias, env, lse, w = ctx.saved_tensors
        # inside the block's VJP (force pass or its rebuild): the rebuild sees
        # the force pass's cotangent again and takes its kept result
        reuse = (ctx.cache, ("backward1", ctx.slot)) if ctx.cache is not None and ctx.cache.in_vjp else None
        c = [_deferred(ctx, role) for role in ("qkv", "bias", "env")]
        qkv, bias, env = (_cut(ctx, role, t) for role, t in zip(("qkv", "bias", "env"), (qkv, bias, env)))
        # (the deferred q/k/v cotangent is the reduction's starting value)
        d_qkv, dbias, denv = PooledTokenAttentionGrad.apply(qkv, bias, env, lse, w, dm, ctx.meta, reuse, c[0])
        return d_qkv, _plus(dbias, c[1]), _plus(denv, c[2]), None, None, None, None


class PooledTokenAttentionGrad(_Fused):
    """backward1 of PooledTokenAttention (per-atom q/k/v, bias and envelope
    gradients); its backward is the backward2 kernel (lse and w are
    statistics, not differentiated)."""

    @staticmethod
    def forward(ctx, qkv, bias, env, lse, w, dm, meta, reuse=None, d_qkv_into=None):
        """d_qkv_into: a q/k/v gradient the result is added to (overwritten)."""
        graph, heads, scale, precision = meta
        ctx.save_for_backward(qkv, bias, env, lse, w, dm)
        ctx.meta = meta
        if reuse is not None:
            cache, key = reuse
            kept = cache.slots.pop(key, None)
            if kept is not None:
                # the same op on the same inputs earlier in this block call
                out = tuple(t.detach() for t in kept)
                return out if d_qkv_into is None else (out[0] + d_qkv_into, *out[1:])
        dqk, wv, dbias, denv = pooled_attention_backward1(qkv, bias, env, lse, w, dm, graph.tokens.index,
                                                          graph.counts, graph.k, heads, scale, precision)
        out = (_pooled_qkv_grad(dqk, wv, dm, graph, heads, d_qkv_into), dbias, denv.view_as(env))
        if out[0] is d_qkv_into:
            ctx.mark_dirty(d_qkv_into)
        if reuse is not None:
            cache.slots[key] = out
        return out

    @staticmethod
    def backward(ctx, h_qkv, h_bias, h_env):
        qkv, bias, env, lse, w, dm = ctx.saved_tensors
        graph, heads, scale, precision = ctx.meta
        if h_qkv is None:
            h_qkv = torch.zeros_like(qkv)
        dqk, wv, dbias, denv, ddm = pooled_attention_backward2(
            qkv, bias, env, lse, w, dm, h_qkv, h_bias, h_env, graph.tokens.index, graph.counts, graph.k, heads,
            scale, precision)
        return _pooled_qkv_grad(dqk, wv, dm, graph, heads), dbias, denv.view_as(env), None, None, ddm, None, None, None


# ---------------------------------------------------------------------------
# the training loss
# ---------------------------------------------------------------------------


class EnergyForceMSE(Function):
    """loss = mean((E - Et)^2) + mean((F - Ft)^2) with F = -grad_pos, as one
    kernel; backward one kernel (first order: the loss is differentiated once,
    by loss.backward())."""

    @staticmethod
    def forward(ctx, energy, grad_pos, e_target, f_target):
        e, g, et, ft = (_f32(t.detach(), "energy_force_mse") for t in (energy, grad_pos, e_target, f_target))
        if e.numel() != et.numel() or g.numel() != ft.numel():
            raise NativeError(f"energy_force_mse: energy {tuple(e.shape)} vs {tuple(et.shape)}, "
                              f"forces {tuple(g.shape)} vs {tuple(ft.shape)}")
        loss = torch.empty((), device=e.device)
        native.call("cg_mse_energy_force", e.data_ptr(), et.data_ptr(), e.numel(), g.data_ptr(), ft.data_ptr(),
                    g.numel(), loss.data_ptr(), _stream())
        ctx.save_for_backward(e, g, et, ft)
        return loss

    @staticmethod
    @torch.autograd.function.once_differentiable
    def backward(ctx, grad_loss):
        e, g, et, ft = ctx.saved_tensors
        de, dg = torch.empty_like(e), torch.empty_like(g)
        grad_loss = _f32(grad_loss, "energy_force_mse")
        native.call("cg_mse_energy_force_bwd", e.data_ptr(), et.data_ptr(), e.numel(), g.data_ptr(),
                    ft.data_ptr(), g.numel(), grad_loss.data_ptr(), de.data_ptr(), dg.data_ptr(), _stream())
        return (de if ctx.needs_input_grad[0] else None, dg if ctx.needs_input_grad[1] else None, None, None)


def energy_force_loss(energy: Tensor, grad_pos: Tensor, e_target: Tensor, f_target: Tensor) -> Tensor:
    """MSE on energies plus MSE on forces F = -grad_pos, fused."""
    return EnergyForceMSE.apply(energy, grad_pos, e_target, f_target)


# ---------------------------------------------------------------------------
# modules
# ---------------------------------------------------------------------------


class Linear(nn.Module):
    """nn.Linear on the tcgen05 GEMM (optionally with a fused SiLU)."""

    def __init__(self, fan_in: int, fan_out: int, bias: bool = True, silu: bool = False):
        super().__init__()
        bound = 1.0 / math.sqrt(fan_in)
        self.weight = nn.Parameter(torch.empty(fan_out, fan_in).uniform_(-bound, bound))
        self.bias = nn.Parameter(torch.empty(fan_out).uniform_(-bound, bound)) if bias else None
        self.silu = silu

    def forward(self, x: Tensor) -> Tensor:
        if self.silu:
            return LinearSiluFn.apply(x, self.weight, self.bias)[0]
        return LinearFn.apply(x, self.weight, self.bias)

    def residual(self, x: Tensor, r: Tensor) -> Tensor:
        """r + self(x) with the add in the GEMM epilogue."""
        if self.silu:
            raise NativeError("Linear.residual: no SiLU variant")
        return LinearResidualFn.apply(x, self.weight, self.bias, r)

    def silu_residual(self, y: Tensor, z: Tensor, r: Tensor) -> Tensor:
        """r + self(silu(z)) for (y, z) = (silu(z), z) from a SiLU linear layer:
        the SiLU derivative is applied in this layer's input-gradient GEMM."""
        if self.silu:
            raise NativeError("Linear.silu_residual: no SiLU variant")
        return SiluLinearResidualFn.apply(y, z, self.weight, self.bias, r)


class LayerNorm(nn.Module):
    """nn.LayerNorm over the last dimension: row normalisation + column affine."""

    def __init__(self, dim: int, eps: float = 1e-5):
        super().__init__()
        self.weight = nn.Parameter(torch.ones(dim))
        self.bias = nn.Parameter(torch.zeros(dim))
        self.eps = eps

    def forward(self, x: Tensor) -> Tensor:
        return ScaleShift.apply(RowNorm.apply(x, self.eps), self.weight, self.bias, x, self.eps)

    def branch(self, x: Tensor) -> tuple[Tensor, Tensor]:
        """(x, LayerNorm(x)) for a residual block: x's two gradients meet inside
        the normalisation backward kernel."""
        x_res, xhat = BranchNorm.apply(x, self.eps)
        return x_res, ScaleShift.apply(xhat, self.weight, self.bias, x, self.eps)
