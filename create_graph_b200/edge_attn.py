"""
Masked edge attention ``out = softmax(q k^T * scale + bias) v`` as a fused op.

The reference registers this op with ``cg.custom_op`` and PyTorch bodies
(kernels/edge_attn/ops.py:57-108) and says a faster version "replaces the
bodies, the registration stays" (:14-15). That is what this module does: the
same class shape (outputs ``out, lse``; saved ``q, k, v, bias, lse``; ``lse``
a statistic), registered through ``cg.custom_op`` as ``cg_b200::edge_attn``,
with forward1 / backward1 / backward2 bodies that call the sm_100a kernels
``cg_edge_attn_fwd1/bwd1/bwd2`` through the C ABI.

q, k, v are (..., S, D) with S <= 32 tokens and D <= 64; the bias broadcasts to
the scores (..., S, S). Rows whose keys are all -inf get zero probabilities.
``key_counts`` (model path, ``edge_attention_masked``) masks keys
j >= key_counts[n] without a -inf bias.

``precision`` selects how float32 products run on the tensor cores: "fp32"
(three-term tf32 split, ~1e-6 relative, the reference's float32 results) or
"tf32" (one tf32 product per tile, operands rounded to 2^-11 relative, fp32
accumulation and softmax; the precision of the tcgen05 projections).
``cg_b200::edge_attn`` is the fp32 op, ``cg_b200::edge_attn_tf32`` the tf32
one; float64 inputs always compute in float64.
"""

from __future__ import annotations

import ctypes
import math

import torch
from torch import Tensor

from create_graph_b200 import native
from create_graph_b200.errors import NativeError
from create_graph_b200.ops import custom_op


def _grid(q: Tensor) -> tuple[tuple[int, ...], int, int]:
    """Leading dims of q and their split into the kernel's (n, h) slice grid."""
    lead = tuple(q.shape[:-2])
    if not lead:
        return lead, 1, 1
    h = lead[-1]
    n = math.prod(lead[:-1])
    return lead, n, h


def _as_nhsd(t: Tensor, n: int, h: int) -> Tensor:
    """(n, h, S, D) view of t with unit column stride (a copy only if needed)."""
    v = t.reshape(n, h, t.shape[-2], t.shape[-1])
    if v.stride(-1) != 1:
        v = v.contiguous()
    return v


def _mat(t: Tensor | None) -> native.Mat:
    if t is None:
        return native.Mat(None, 0, 0, 0)
    return native.Mat(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2))


def _bias_view(bias: Tensor, lead, n: int, h: int, s: int) -> tuple[Tensor, bool]:
    """(n, h, s, s) view of the broadcast bias (stride 0 where it broadcasts), or
    a materialised copy when the leading dims cannot be merged as a view."""
    expanded = bias.expand(*lead, s, s)
    try:
        return expanded.view(n, h, s, s), False
    except RuntimeError:
        return expanded.reshape(n, h, s, s).contiguous(), True


def _bias(t: Tensor | None) -> native.Bias:
    if t is None:
        return native.Bias(None, 0, 0, 0, 0)
    return native.Bias(t.data_ptr(), t.stride(0), t.stride(1), t.stride(2), t.stride(3))


def _reduce_to(grad: Tensor, like: Tensor) -> Tensor:
    """Sum a score-shaped tensor down to ``like``'s broadcast shape (used only for
    bias layouts whose leading dims cannot be merged into a strided view)."""
    while grad.ndim > like.ndim:
        grad = grad.sum(dim=0)
    for dim, size in enumerate(like.shape):
        if size == 1 and grad.shape[dim] != 1:
            grad = grad.sum(dim=dim, keepdim=True)
    return grad


class _Call:
    """Argument block of one kernel call plus the tensors it points into."""

    def __init__(self, q: Tensor, k: Tensor, v: Tensor, bias: Tensor | None, scale: float, key_counts=None,
                 precision: str = "fp32"):
        native.require_cuda(q, k, v, bias)
        if not (q.dtype == k.dtype == v.dtype and (bias is None or bias.dtype == q.dtype)):
            raise NativeError("edge_attn: q, k, v and bias must share one dtype")
        self.lead, self.n, self.h = _grid(q)
        self.s, self.d = q.shape[-2], q.shape[-1]
        if k.shape != q.shape or v.shape[:-1] != q.shape[:-1] or v.shape[-1] != self.d:
            raise NativeError(
                f"edge_attn: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} must match"
            )
        self.q = _as_nhsd(q, self.n, self.h)
        self.k = _as_nhsd(k, self.n, self.h)
        self.v = _as_nhsd(v, self.n, self.h)
        self.bias_src = bias
        self.bias, self.bias_copied = (None, False)
        if bias is not None:
            self.bias, self.bias_copied = _bias_view(bias, self.lead, self.n, self.h, self.s)
        self.args = native.EdgeAttnArgs()
        a = self.args
        a.n, a.h, a.k, a.d = self.n, self.h, self.s, self.d
        a.dtype = native.dtype_code(q)
        a.precision = native.attn_precision(precision)
        a.scale = float(scale)
        a.key_count = None if key_counts is None else key_counts.data_ptr()
        a.q, a.k_, a.v = _mat(self.q), _mat(self.k), _mat(self.v)
        a.bias = _bias(self.bias)
        self.keep = [key_counts]

    def new(self, *shape) -> Tensor:
        return torch.empty(shape, dtype=self.q.dtype, device=self.q.device)

    def run(self, fn) -> None:
        lib = native.lib()
        args = ctypes.byref(self.args)
        scratch_bytes = lib.cg_edge_attn_scratch_bytes(args)
        if scratch_bytes > 0:
            scratch = torch.empty(scratch_bytes, dtype=torch.uint8, device=self.q.device)
            self.args.scratch = scratch.data_ptr()
            self.keep.append(scratch)
        native.invoke(fn, args, native.stream_ptr(self.q.device), info=_info(self.args))

    def dbias_buffer(self) -> Tensor | None:
        """dbias in the reduced (n_b, h_b, ki, kj) layout the kernel writes."""
        if self.bias is None:
            return None
        b = self.bias
        shape = tuple(1 if b.stride(i) == 0 else b.shape[i] for i in range(4))
        out = self.new(*shape)
        self.args.dbias = native.Bias(out.data_ptr(), *(out.stride(i) for i in range(4)))
        return out

    def finish_dbias(self, dbias: Tensor | None) -> Tensor | None:
        if dbias is None:
            return None
        if self.bias_copied:
            full = dbias.reshape(*self.lead, self.s, self.s)
            return _reduce_to(full, self.bias_src).contiguous()
        return dbias.reshape(self.bias_src.shape)

    def set_hb(self, hb: Tensor | None) -> None:
        if hb is None or self.bias is None:
            return
        view, _ = _bias_view(hb, self.lead, self.n, self.h, self.s)
        if view.stride(-1) != 1 and view.stride(-1) != 0:
            view = view.contiguous()
        self.keep.append(view)
        self.args.hb = _bias(view)

    def mat_arg(self, name: str, t: Tensor) -> Tensor:
        view = _as_nhsd(t, self.n, self.h)
        self.keep.append(view)
        setattr(self.args, name, _mat(view))
        return view


def attn_forward1(q, k, v, bias, scale, key_counts=None, precision="fp32") -> tuple[Tensor, Tensor]:
    c = _Call(q, k, v, bias, scale, key_counts, precision)
    out = c.new(c.n, c.h, c.s, c.d)
    lse = c.new(c.n, c.h, c.s)
    c.args.out = _mat(out)
    c.args.lse = lse.data_ptr()
    c.run("cg_edge_attn_fwd1")
    return out.view(*c.lead, c.s, c.d), lse.view(*c.lead, c.s)


def attn_backward1(q, k, v, bias, lse, grad_out, scale, key_counts=None, precision="fp32"):
    c = _Call(q, k, v, bias, scale, key_counts, precision)
    lse_c = lse.reshape(c.n, c.h, c.s).contiguous()
    c.keep.append(lse_c)
    c.args.lse = lse_c.data_ptr()
    c.mat_arg("grad_out", grad_out)
    dq, dk, dv = (c.new(c.n, c.h, c.s, c.d) for _ in range(3))
    c.args.dq, c.args.dk, c.args.dv = _mat(dq), _mat(dk), _mat(dv)
    dbias = c.dbias_buffer()
    c.run("cg_edge_attn_bwd1")
    shape = (*c.lead, c.s, c.d)
    return dq.view(shape), dk.view(shape), dv.view(shape), c.finish_dbias(dbias)


def attn_backward2(q, k, v, bias, lse, grad_out, scale, hq, hk, hv, hb, key_counts=None, precision="fp32"):
    c = _Call(q, k, v, bias, scale, key_counts, precision)
    lse_c = lse.reshape(c.n, c.h, c.s).contiguous()
    c.keep.append(lse_c)
    c.args.lse = lse_c.data_ptr()
    c.mat_arg("grad_out", grad_out)
    c.mat_arg("hq", hq)
    c.mat_arg("hk", hk)
    c.mat_arg("hv", hv)
    c.set_hb(hb)
    dq, dk, dv, dg = (c.new(c.n, c.h, c.s, c.d) for _ in range(4))
    c.args.dq, c.args.dk, c.args.dv, c.args.dgrad_out = _mat(dq), _mat(dk), _mat(dv), _mat(dg)
    dbias = c.dbias_buffer()
    c.run("cg_edge_attn_bwd2")
    shape = (*c.lead, c.s, c.d)
    return dq.view(shape), dk.view(shape), dv.view(shape), c.finish_dbias(dbias), dg.view(shape)


def _edge_attention_op(name: str, precision: str):
    """The reference's EdgeAttention (kernels/edge_attn/ops.py:57-104) with
    sm_100a kernel bodies, registered as ``name`` for one precision."""

    class EdgeAttention:
        outputs = ("out", "lse")
        save = ("q", "k", "v", "bias", "lse")
        nondiff = ("lse",)

        @staticmethod
        def forward1(q: Tensor, k: Tensor, v: Tensor, bias: Tensor, scale: float) -> tuple[Tensor, Tensor]:
            return attn_forward1(q, k, v, bias, scale, precision=precision)

        @staticmethod
        def fake(q, k, v, bias, scale):
            return q.new_empty((*q.shape[:-1], v.shape[-1])), q.new_empty(q.shape[:-1])

        @staticmethod
        def backward1(q, k, v, bias, lse, grad_out, scale):
            return attn_backward1(q, k, v, bias, lse, grad_out, scale, precision=precision)

        @staticmethod
        def backward2(q, k, v, bias, lse, grad_out, scale, hq, hk, hv, hb):
            return attn_backward2(q, k, v, bias, lse, grad_out, scale, hq, hk, hv, hb, precision=precision)

    return custom_op(name)(EdgeAttention)


EdgeAttention = _edge_attention_op("cg_b200::edge_attn", "fp32")
EdgeAttentionTF32 = _edge_attention_op("cg_b200::edge_attn_tf32", "tf32")
_OPS = {"fp32": EdgeAttention, "tf32": EdgeAttentionTF32}


def edge_attention(q, k, v, bias, scale: float, precision: str = "fp32") -> Tensor:
    """``softmax(q k^T * scale + bias) v`` through the fused op."""
    native.attn_precision(precision)
    return _OPS[precision](q, k, v, bias, scale)[0]


# ---------------------------------------------------------------------------
# Token layout of the energy network: per atom n, k edge tokens; token (n, s)
# holds [q | k | v] (heads contiguous) of atom index[n*k + s], read by the
# kernels straight from the per-atom qkv rows (n_atoms, 3*h*d) through the
# index (no materialised token tensor). The per-key bias is (n*k, h); keys
# j >= counts[n] are masked. Token-level outputs (attention output, its
# gradient, and the per-token q/k/v gradients) are (n, k, ...) tensors.
# ---------------------------------------------------------------------------


def _token_mats(t: Tensor, n: int, k: int, heads: int, d: int, parts: int):
    """cg_mat views of the `parts` blocks of a token tensor (n*k, parts*h*d)."""
    c = heads * d
    width = parts * c
    esz = t.element_size()
    return [native.Mat(t.data_ptr() + p * c * esz, k * width, d, width) for p in range(parts)]


def _atom_mats(t: Tensor, heads: int, d: int):
    """cg_mat views of q, k, v in per-atom rows (n_atoms, 3*h*d), read through the token index."""
    c = heads * d
    esz = t.element_size()
    return [native.Mat(t.data_ptr() + p * c * esz, 0, d, 3 * c) for p in range(3)]


def _token_bias(t: Tensor | None, k: int, heads: int) -> native.Bias:
    if t is None:
        return native.Bias(None, 0, 0, 0, 0)
    return native.Bias(t.data_ptr(), k * heads, 1, 0, heads)


def _gathered_args(qkv: Tensor, bias: Tensor, index: Tensor, counts: Tensor, k: int, heads: int, scale: float,
                   precision: str):
    native.require_cuda(qkv, bias, counts, index)
    if qkv.dtype != torch.float32 or bias.dtype != torch.float32:
        raise NativeError("token attention: qkv and bias must be float32")
    if counts.dtype != torch.int32 or index.dtype != torch.int32:
        raise NativeError("token attention: counts and index must be int32")
    n = counts.shape[0]
    d = qkv.shape[1] // (3 * heads)
    if qkv.shape[1] != 3 * heads * d or index.numel() != n * k or bias.shape[0] != n * k or bias.shape[-1] != heads:
        raise NativeError(
            f"token attention: qkv {tuple(qkv.shape)}, bias {tuple(bias.shape)}, index {index.numel()}, n {n}, k {k}"
        )
    a = native.EdgeAttnArgs()
    a.n, a.h, a.k, a.d = n, heads, k, d
    a.dtype = native.F32
    a.precision = native.attn_precision(precision)
    a.scale = float(scale)
    a.key_count = counts.data_ptr()
    a.token_index = index.data_ptr()
    a.q, a.k_, a.v = _atom_mats(qkv, heads, d)
    a.bias = _token_bias(bias, k, heads)
    return a, n, d


def _info(a) -> tuple[int, int, int, int]:
    return (int(a.n), int(a.h), int(a.k), int(a.d))


def _run(fn: str, a, device) -> None:
    native.invoke(fn, ctypes.byref(a), native.stream_ptr(device), info=_info(a))


def token_attention_forward1(qkv, bias, index, counts, k, heads, scale, precision="fp32"):
    """(out (n, k, h*d), lse (n, h, k)) of the gathered tokens."""
    qkv, bias = qkv.contiguous(), bias.contiguous()
    a, n, d = _gathered_args(qkv, bias, index, counts, k, heads, scale, precision)
    out = torch.empty(n, k, heads * d, device=qkv.device)
    lse = torch.empty(n, heads, k, device=qkv.device)
    (a.out,) = _token_mats(out, n, k, heads, d, 1)
    a.lse = lse.data_ptr()
    _run("cg_edge_attn_fwd1", a, qkv.device)
    return out, lse


def token_attention_backward1(qkv, bias, lse, g, index, counts, k, heads, scale, precision="fp32"):
    """(dtok (n*k, 3*h*d) per-token q/k/v gradients, dbias (n*k, h))."""
    qkv, bias, g = qkv.contiguous(), bias.contiguous(), g.contiguous()
    a, n, d = _gathered_args(qkv, bias, index, counts, k, heads, scale, precision)
    a.lse = lse.data_ptr()
    (a.grad_out,) = _token_mats(g, n, k, heads, d, 1)
    dtok = torch.empty(n * k, qkv.shape[1], device=qkv.device)
    dbias = torch.empty_like(bias)
    a.dq, a.dk, a.dv = _token_mats(dtok, n, k, heads, d, 3)
    a.dbias = _token_bias(dbias, k, heads)
    _run("cg_edge_attn_bwd1", a, qkv.device)
    return dtok, dbias


def token_attention_backward2(qkv, bias, lse, g, h_qkv, h_bias, index, counts, k, heads, scale, precision="fp32"):
    """Second derivative: per-token (dtok, dbias, dg) for the per-atom
    cotangent h_qkv of the q/k/v gradient (read through the same index) and
    the cotangent h_bias of dbias."""
    qkv, bias, g, h_qkv = qkv.contiguous(), bias.contiguous(), g.contiguous(), h_qkv.contiguous()
    a, n, d = _gathered_args(qkv, bias, index, counts, k, heads, scale, precision)
    a.lse = lse.data_ptr()
    (a.grad_out,) = _token_mats(g, n, k, heads, d, 1)
    a.hq, a.hk, a.hv = _atom_mats(h_qkv, heads, d)
    if h_bias is not None:
        h_bias = h_bias.contiguous()
        a.hb = _token_bias(h_bias, k, heads)
    dtok = torch.empty(n * k, qkv.shape[1], device=qkv.device)
    dbias = torch.empty_like(bias)
    dg = torch.empty_like(g)
    a.dq, a.dk, a.dv = _token_mats(dtok, n, k, heads, d, 3)
    a.dbias = _token_bias(dbias, k, heads)
    (a.dgrad_out,) = _token_mats(dg, n, k, heads, d, 1)
    _run("cg_edge_attn_bwd2", a, qkv.device)
    return dtok, dbias, dg


# ---------------------------------------------------------------------------
# Envelope-pooled token attention: token attention followed by the
# envelope-weighted sum over each atom's tokens, as one op
# (cg_pooled_attn_fwd / bwd1 / bwd2). The v gradient of token (n, j) is rank
# one, wv[n*k + j, h] * dout[n, h]; callers reduce it with
# cg_segment_sum_scaled.
# ---------------------------------------------------------------------------


def _rows(t: Tensor) -> Tensor:
    """t itself when its columns are contiguous (rows may be strided), else a copy."""
    return t if t.stride(-1) == 1 and t.stride(0) >= t.shape[-1] else t.contiguous()


def _pooled_args(qkv, bias, env, index, counts, k, heads, scale, precision):
    native.require_cuda(qkv, bias, env, counts, index)
    if qkv.dtype != torch.float32 or bias.dtype != torch.float32 or env.dtype != torch.float32:
        raise NativeError("pooled attention: qkv, bias and env must be float32")
    if counts.dtype != torch.int32 or index.dtype != torch.int32:
        raise NativeError("pooled attention: counts and index must be int32")
    n = counts.shape[0]
    d = qkv.shape[1] // (3 * heads)
    if (qkv.shape[1] != 3 * heads * d or index.numel() != n * k or tuple(bias.shape) != (n * k, heads)
            or bias.stride(1) != 1 or env.numel() != n * k or qkv.stride(1) != 1):
        raise NativeError(
            f"pooled attention: qkv {tuple(qkv.shape)}, bias {tuple(bias.shape)}, env {tuple(env.shape)}, "
            f"index {index.numel()}, n {n}, k {k}, heads {heads}"
        )
    a = native.PooledAttnArgs()
    a.n, a.h, a.k, a.d = n, heads, k, d
    a.precision = native.attn_precision(precision)
    a.scale = float(scale)
    a.token_index = index.data_ptr()
    a.key_count = counts.data_ptr()
    a.qkv = qkv.data_ptr()
    a.ld_qkv = qkv.stride(0)
    a.bias = bias.data_ptr()
    a.ld_bias = bias.stride(0)
    a.env = env.data_ptr()
    return a, n, d


def pooled_attention_forward(qkv, bias, env, index, counts, k, heads, scale, precision="fp32"):
    """(out (n, h*d), lse (n, h, k), w (n, h, k)) with w_j = sum_i env_i P_ij. bias
    may be a column block of a wider matrix (unit column stride)."""
    qkv, bias, env = qkv.contiguous(), _rows(bias), env.contiguous()
    a, n, d = _pooled_args(qkv, bias, env, index, counts, k, heads, scale, precision)
    out = torch.empty(n, heads * d, device=qkv.device)
    lse = torch.empty(n, heads, k, device=qkv.device)
    w = torch.empty(n, heads, k, device=qkv.device)
    a.out, a.lse, a.w = out.data_ptr(), lse.data_ptr(), w.data_ptr()
    _run("cg_pooled_attn_fwd", a, qkv.device)
    return out, lse, w


def pooled_attention_out(qkv, w, index, counts, k, heads):
    """out (n, h*d) = sum_j w[n, h, j] v_j for known weights w (n, h, k): the
    forward's output, bit for bit, without recomputing the softmax."""
    qkv = qkv.contiguous()
    native.require_cuda(qkv, w, index, counts)
    n = counts.shape[0]
    d = qkv.shape[1] // (3 * heads)
    if w.shape != (n, heads, k) or not w.is_contiguous():
        raise NativeError(f"pooled attention: w {tuple(w.shape)} must be a contiguous ({n}, {heads}, {k})")
    a = native.PooledAttnArgs()
    a.n, a.h, a.k, a.d = n, heads, k, d
    a.token_index, a.key_count = index.data_ptr(), counts.data_ptr()
    a.qkv, a.ld_qkv, a.w = qkv.data_ptr(), qkv.stride(0), w.data_ptr()
    out = torch.empty(n, heads * d, device=qkv.device)
    a.out = out.data_ptr()
    _run("cg_pooled_attn_out", a, qkv.device)
    return out


def pooled_attention_backward1(qkv, bias, env, lse, w, dout, index, counts, k, heads, scale, precision="fp32"):
    """(dqk (n*k, 2*h*d) per-token [dq | dk], wv (n*k, h), dbias (n*k, h), denv (n, k))."""
    qkv, bias, env, dout = qkv.contiguous(), _rows(bias), env.contiguous(), dout.contiguous()
    a, n, d = _pooled_args(qkv, bias, env, index, counts, k, heads, scale, precision)
    dqk = torch.empty(n * k, 2 * heads * d, device=qkv.device)
    wv = torch.empty(n * k, heads, device=qkv.device)
    dbias = torch.empty(n * k, heads, device=qkv.device)
    denv = torch.empty(n, k, device=qkv.device)
    a.lse, a.w, a.dout = lse.data_ptr(), w.data_ptr(), dout.data_ptr()
    a.dqk, a.ld_dqk, a.wv = dqk.data_ptr(), dqk.stride(0), wv.data_ptr()
    a.dbias, a.denv = dbias.data_ptr(), denv.data_ptr()
    _run("cg_pooled_attn_bwd1", a, qkv.device)
    return dqk, wv, dbias, denv


def pooled_attention_backward2(qkv, bias, env, lse, w, dout, h_qkv, h_bias, h_env, index, counts, k, heads, scale,
                               precision="fp32"):
    """Second derivative: (dqk, wv, dbias, denv, ddout) of <h_qkv, d_qkv> +
    <h_bias, dbias> + <h_env, denv> (h_bias, h_env may be None: zero)."""
    qkv, env, dout, h_qkv = (t.contiguous() for t in (qkv, env, dout, h_qkv))
    bias = _rows(bias)
    a, n, d = _pooled_args(qkv, bias, env, index, counts, k, heads, scale, precision)
    if h_qkv.shape != qkv.shape or h_qkv.stride(0) != qkv.stride(0):
        raise NativeError(f"pooled attention: h_qkv {tuple(h_qkv.shape)} must match qkv {tuple(qkv.shape)}")
    keep = []
    if h_bias is not None:
        h_bias = _rows(h_bias)
        keep.append(h_bias)
        a.hbias = h_bias.data_ptr()
        a.ld_hbias = h_bias.stride(0)
    if h_env is not None:
        h_env = h_env.contiguous()
        keep.append(h_env)
        a.henv = h_env.data_ptr()
    dqk = torch.empty(n * k, 2 * heads * d, device=qkv.device)
    wv = torch.empty(n * k, heads, device=qkv.device)
    dbias = torch.empty(n * k, heads, device=qkv.device)
    denv = torch.empty(n, k, device=qkv.device)
    ddout = torch.empty(n, heads * d, device=qkv.device)
    a.lse, a.w, a.dout, a.hqkv = lse.data_ptr(), w.data_ptr(), dout.data_ptr(), h_qkv.data_ptr()
    a.dqk, a.ld_dqk, a.wv = dqk.data_ptr(), dqk.stride(0), wv.data_ptr()
    a.dbias, a.denv, a.ddout = dbias.data_ptr(), denv.data_ptr(), ddout.data_ptr()
    _run("cg_pooled_attn_bwd2", a, qkv.device)
    return dqk, wv, dbias, denv, ddout
