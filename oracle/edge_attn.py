"""
Masked edge attention in numpy float64: the oracle for cg_edge_attn_fwd1/bwd1/bwd2.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Every function restates the
reference's PyTorch code in kernels/edge_attn/ops.py line by line:
``scores`` = _scores (:26-34), ``reduce_like`` = _reduce (:37-44),
``first`` = _first (:47-54), ``forward1`` (:64-68), ``backward1`` (:75-76),
``backward2`` (:79-104). ``key_counts`` (the model path's key mask) is applied
as a -inf bias on keys j >= key_counts[n], which is what the kernels do.
Pinned against tests/golden/edge_attn_*.npz, produced by the reference itself.
"""

from __future__ import annotations

import numpy as np


def _t(x):
    return np.swapaxes(x, -1, -2)


def apply_key_counts(bias, shape, key_counts):
    """bias (broadcast to the score shape (..., S, S)) with keys j >= key_counts[n]
    set to -inf; n indexes the product of the leading dims but the last."""
    full = np.broadcast_to(bias, shape).copy() if bias is not None else np.zeros(shape)
    if key_counts is None:
        return full
    s = shape[-1]
    lead = shape[:-2]
    n = int(np.prod(lead[:-1])) if len(lead) > 1 else 1
    h = lead[-1] if lead else 1
    view = full.reshape(n, h, s, s)
    for i, c in enumerate(np.asarray(key_counts).reshape(-1)):
        view[i, :, :, max(int(c), 0):] = -np.inf
    return view.reshape(shape)


def scores(q, k, bias, scale):
    """probs, lse with -inf-safe masking (ops.py:26-34)."""
    logits = np.matmul(q, _t(k)) * scale + bias
    finite = np.isfinite(logits)
    safe = np.where(finite, logits, -np.inf)
    m = safe.max(axis=-1, keepdims=True)
    m_ok = np.where(np.isfinite(m), m, 0.0)
    with np.errstate(divide="ignore", invalid="ignore", over="ignore"):
        lse = np.log(np.exp(safe - m_ok).sum(axis=-1, keepdims=True)) + m_ok
    lse = np.where(finite.any(axis=-1, keepdims=True), lse, -np.inf)[..., 0]
    row_ok = finite.any(axis=-1, keepdims=True)
    shift = np.where(np.isfinite(lse), lse, 0.0)[..., None]
    with np.errstate(over="ignore", invalid="ignore"):
        probs = np.exp(safe - shift)
    probs = np.where(finite & row_ok, probs, 0.0)
    return probs, lse


def reduce_like(grad, like_shape):
    """Sum a score-shaped array down to the bias's broadcast shape (ops.py:37-44)."""
    while grad.ndim > len(like_shape):
        grad = grad.sum(axis=0)
    for dim, size in enumerate(like_shape):
        if size == 1 and grad.shape[dim] != 1:
            grad = grad.sum(axis=dim, keepdims=True)
    return grad


def first(q, k, v, bias, grad_out, scale):
    """First-order gradients and the intermediates backward2 reuses (ops.py:47-54)."""
    probs, _ = scores(q, k, bias, scale)
    grad_v = np.matmul(_t(probs), grad_out)
    grad_probs = np.matmul(grad_out, _t(v))
    grad_logits = probs * (grad_probs - (probs * grad_probs).sum(axis=-1, keepdims=True))
    grad_q = np.matmul(grad_logits, k) * scale
    grad_k = np.matmul(_t(grad_logits), q) * scale
    return grad_q, grad_k, grad_v, grad_logits, probs, grad_probs


def forward1(q, k, v, bias, scale, key_counts=None):
    full = apply_key_counts(bias, q.shape[:-1] + (k.shape[-2],), key_counts)
    probs, lse = scores(q, k, full, scale)
    return np.matmul(probs, v), lse


def backward1(q, k, v, bias, grad_out, scale, key_counts=None):
    """(dq, dk, dv, dbias) with dbias in the bias's own shape (ops.py:75-76)."""
    shape = q.shape[:-1] + (k.shape[-2],)
    full = apply_key_counts(bias, shape, key_counts)
    gq, gk, gv, gl, _, _ = first(q, k, v, full, grad_out, scale)
    bshape = np.shape(bias) if bias is not None else shape
    return gq, gk, gv, reduce_like(gl, bshape)


def backward2(q, k, v, bias, grad_out, scale, hq, hk, hv, hb, key_counts=None):
    """Gradients of <hq,dq>+<hk,dk>+<hv,dv>+<hb,dbias> w.r.t. q, k, v, bias and
    grad_out (ops.py:79-104)."""
    shape = q.shape[:-1] + (k.shape[-2],)
    full = apply_key_counts(bias, shape, key_counts)
    _, _, _, grad_logits, probs, gp = first(q, k, v, full, grad_out, scale)
    d_logits = scale * (np.matmul(hq, _t(k)) + np.matmul(q, _t(hk)))
    if hb is not None:
        d_logits = d_logits + hb
    grad_q = scale * np.matmul(grad_logits, hk)
    grad_k = scale * np.matmul(_t(grad_logits), hq)
    centered = gp - (probs * gp).sum(axis=-1, keepdims=True)
    d_probs = d_logits * centered
    d_gp = d_logits * probs
    d_rowsum = -(d_logits * probs).sum(axis=-1, keepdims=True)
    d_probs = d_probs + d_rowsum * gp
    d_gp = d_gp + d_rowsum * probs
    grad_out_cot = np.matmul(d_gp, v) + np.matmul(probs, hv)
    grad_v = np.matmul(_t(d_gp), grad_out)
    d_probs = d_probs + np.matmul(grad_out, _t(hv))
    d_scores = probs * (d_probs - (probs * d_probs).sum(axis=-1, keepdims=True))
    grad_q = grad_q + np.matmul(d_scores, k) * scale
    grad_k = grad_k + np.matmul(_t(d_scores), q) * scale
    bshape = np.shape(bias) if bias is not None else shape
    return grad_q, grad_k, grad_v, reduce_like(d_scores, bshape), grad_out_cot
