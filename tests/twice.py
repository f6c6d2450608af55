"""Second-order comparison of two implementations of one function.

``twice_errors(mine, ref, inputs)`` evaluates both on copies of the inputs and
returns relative errors of: the outputs; the input gradients for fixed random
output cotangents (taken with create_graph=True, the force pass); and the
gradients of a fixed random linear function of those input gradients w.r.t.
the inputs and the cotangents (the parameter backward through the force).
The same three levels as ``cg.testing.check_op``, for any function.
"""

from __future__ import annotations

import torch


def rel(a, b) -> float:
    a, b = a.detach().double().cpu(), b.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-300)).item()


def _tuple(x):
    return tuple(x) if isinstance(x, (tuple, list)) else (x,)


def twice_errors(mine, ref, inputs, *, ref_dtype=torch.float64, seed=7, diff=None):
    """diff: indices of the inputs to differentiate (default: all float tensors)."""
    gen = torch.Generator().manual_seed(seed)
    idx = diff if diff is not None else [i for i, x in enumerate(inputs) if torch.is_tensor(x) and x.is_floating_point()]

    def leaves(dtype):
        out = []
        for i, x in enumerate(inputs):
            if torch.is_tensor(x) and x.is_floating_point():
                y = x.detach().to(dtype).clone()
                out.append(y.requires_grad_(i in idx))
            else:
                out.append(x)
        return out

    xm, xr = leaves(inputs[idx[0]].dtype), leaves(ref_dtype)
    om, orf = _tuple(mine(*xm)), _tuple(ref(*xr))
    errors = {f"out{i}": rel(a, b) for i, (a, b) in enumerate(zip(om, orf))}
    cots = [torch.randn(o.shape, generator=gen, dtype=torch.float64) for o in orf]
    cm = [c.to(om[i]).requires_grad_(True) for i, c in enumerate(cots)]
    cr = [c.to(orf[i]).requires_grad_(True) for i, c in enumerate(cots)]
    inm, inr = [xm[i] for i in idx], [xr[i] for i in idx]
    gm = torch.autograd.grad(om, inm, cm, create_graph=True, allow_unused=True)
    gr = torch.autograd.grad(orf, inr, cr, create_graph=True, allow_unused=True)
    for i, (a, b) in enumerate(zip(gm, gr)):
        errors[f"grad{idx[i]}"] = rel(a, b)
    ws = [torch.randn(g.shape, generator=gen, dtype=torch.float64) for g in gr]
    sm = sum((w.to(g) * g).sum() for w, g in zip(ws, gm))
    sr = sum((w.to(g) * g).sum() for w, g in zip(ws, gr))
    hm = torch.autograd.grad(sm, [*inm, *cm], allow_unused=True)
    hr = torch.autograd.grad(sr, [*inr, *cr], allow_unused=True)
    names = [f"in{i}" for i in idx] + [f"cot{i}" for i in range(len(cots))]
    for name, a, b in zip(names, hm, hr):
        if a is None and b is None:
            continue
        a = torch.zeros_like(b) if a is None else a
        b = torch.zeros_like(a) if b is None else b
        errors[f"second.{name}"] = rel(a, b)
    return errors
