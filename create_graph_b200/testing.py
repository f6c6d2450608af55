"""
Acceptance checks for models and fused operators.

The same checks as src/create_graph/testing.py:21-208, so parity tests read
like the reference's own: errors are relative norms; for parameter gradients
two numbers are reported, the error of all gradients concatenated and the
worst single tensor, whose scale is floored at 1e-4 of the whole gradient's
norm (tensors whose reference gradient is ~0 would otherwise report pure
rounding noise).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor, nn

from create_graph_b200.api import create_graph
from create_graph_b200.region import select_output


def rel_err(got: Tensor, want: Tensor) -> float:
    """||got - want|| / ||want|| in float64 (want's norm floored at 1e-300)."""
    a = got.detach().double().cpu()
    b = want.detach().double().cpu()
    return ((a - b).norm() / b.norm().clamp_min(1e-300)).item()


def grad_errors(got: Sequence[Tensor], want: Sequence[Tensor]) -> dict[str, float]:
    a = [g.detach().double().cpu() for g in got]
    b = [w.detach().double().cpu() for w in want]
    flat_a = torch.cat([g.flatten() for g in a])
    flat_b = torch.cat([w.flatten() for w in b])
    floor = 1e-4 * flat_b.norm()
    worst = max(((g - w).norm() / torch.maximum(w.norm(), floor)).item() for g, w in zip(a, b))
    return {"all": rel_err(flat_a, flat_b), "worst_tensor": worst}


def param_grads(model: nn.Module) -> list[Tensor]:
    return [
        torch.zeros_like(p) if p.grad is None else p.grad.detach().clone()
        for p in model.parameters()
        if p.requires_grad
    ]


def coupled_loss(seed: int = 0) -> Callable:
    """A loss coupling the output and its gradients linearly and quadratically,
    with fixed random weights (one draw per quantity, reused by every call)."""
    drawn: dict = {}

    def weights(key, like: Tensor) -> Tensor:
        if key not in drawn:
            gen = torch.Generator().manual_seed(seed + len(drawn))
            drawn[key] = torch.randn(like.shape, generator=gen, dtype=torch.float64)
        return drawn[key].to(like)

    def loss(target: Tensor, grads: dict[str, Tensor]) -> Tensor:
        total = (weights("out", target) * target).sum() + 0.5 * target.square().sum()
        for name, g in grads.items():
            total = total + (weights(name, g) * g).sum() + 0.5 * g.square().sum()
        return total

    return loss


def run_step(model, data, *, outputs, inputs, loss: Callable, exact: bool):
    """One training step; returns output, input grads, loss and parameter grads."""
    params = [p for p in model.parameters() if p.requires_grad]
    for p in params:
        p.grad = None
    out, grads = create_graph(model, data, outputs=outputs, inputs=inputs, train=True, exact=exact)
    target = select_output(out, outputs)
    value = loss(target, grads)
    value.backward()
    result = {
        "out": target.detach(),
        "grads": {k: g.detach() for k, g in grads.items()},
        "loss": value.detach(),
        "params": param_grads(model),
    }
    for p in params:
        p.grad = None
    return result


def step_errors(got: dict, want: dict) -> dict[str, float]:
    errors = {"out": rel_err(got["out"], want["out"]), "loss": rel_err(got["loss"], want["loss"])}
    for name in got["grads"]:
        errors[f"grad_{name}"] = rel_err(got["grads"][name], want["grads"][name])
    params = grad_errors(got["params"], want["params"])
    errors["params"] = params["all"]
    errors["params_worst_tensor"] = params["worst_tensor"]
    return errors


def check_create_graph(
    model: nn.Module,
    data,
    *,
    outputs="energy",
    inputs=("pos",),
    loss: Callable | None = None,
) -> dict[str, float]:
    """Relative errors of create_graph against ``exact=True`` on the same
    parameters and data: output, input grads, loss and parameter grads."""
    loss = loss or coupled_loss()
    got = run_step(model, data, outputs=outputs, inputs=inputs, loss=loss, exact=False)
    want = run_step(model, data, outputs=outputs, inputs=inputs, loss=loss, exact=True)
    return step_errors(got, want)


def check_float32(
    model32: nn.Module,
    data32,
    model64: nn.Module,
    data64,
    *,
    outputs="energy",
    inputs=("pos",),
    loss: Callable | None = None,
) -> dict[str, dict[str, float]]:
    """create_graph and eager create_graph in float32, each against eager
    create_graph in float64 (``model64`` holds ``model32``'s parameters).
    Returns ``{"create_graph": errors, "eager": errors}``."""
    loss = loss or coupled_loss()
    want = run_step(model64, data64, outputs=outputs, inputs=inputs, loss=loss, exact=True)
    result = {}
    for name, exact in (("create_graph", False), ("eager", True)):
        got = run_step(model32, data32, outputs=outputs, inputs=inputs, loss=loss, exact=exact)
        result[name] = step_errors(got, want)
    return result


def as_close_as_eager(result: dict, floor: dict[str, float], factor: float = 4.0) -> dict:
    """Quantities where create_graph's float32 error exceeds both ``floor`` and
    ``factor`` times eager create_graph's (empty when it passes)."""
    return {
        k: (v, result["eager"][k])
        for k, v in result["create_graph"].items()
        if k in floor and v > max(floor[k], factor * result["eager"][k])
    }


def check_op(op, reference: Callable, args: Sequence, *, seed: int = 20260917) -> dict[str, float]:
    """forward1, backward1 and backward2 of a ``cg.custom_op`` against a
    differentiable ``reference`` with the same signature
    (src/create_graph/testing.py:155-208): the outputs; the input gradients for
    random cotangents of the differentiable outputs; and the gradients of a
    random linear function of those input gradients w.r.t. the inputs and the
    cotangents. Random weights come from ``seed``'s stream, on the args' device."""
    gen = torch.Generator().manual_seed(seed)

    def fresh_leaves():
        return [
            a.detach().clone().requires_grad_(a.is_floating_point()) if isinstance(a, Tensor) else a
            for a in args
        ]

    def call(fn, xs):
        return _as_tuple(fn(*xs))

    xs_ref, xs_op = fresh_leaves(), fresh_leaves()
    out_ref, out_op = call(reference, xs_ref), call(op, xs_op)
    errors = {}
    for name, a, b in zip(op.outputs, out_op, out_ref):
        errors[f"forward1.{name}"] = rel_err(a, b)
    diff = [i for i, name in enumerate(op.outputs) if name not in op.nondiff]
    in_ref = [x for x in xs_ref if isinstance(x, Tensor) and x.requires_grad]
    in_op = [x for x in xs_op if isinstance(x, Tensor) and x.requires_grad]
    cots = [torch.randn(out_ref[i].shape, generator=gen, dtype=torch.float64).to(out_ref[i]) for i in diff]
    cot_ref = [c.clone().requires_grad_(True) for c in cots]
    cot_op = [c.clone().requires_grad_(True) for c in cots]
    g_ref = torch.autograd.grad([out_ref[i] for i in diff], in_ref, cot_ref, create_graph=True)
    g_op = torch.autograd.grad([out_op[i] for i in diff], in_op, cot_op, create_graph=True)
    names = [n for n, a in zip(op.params, args) if isinstance(a, Tensor)]
    for name, a, b in zip(names, g_op, g_ref):
        errors[f"backward1.{name}"] = rel_err(a, b)
    ws = [torch.randn(g.shape, generator=gen, dtype=torch.float64).to(g) for g in g_ref]
    s_ref = sum((w * g).sum() for w, g in zip(ws, g_ref))
    s_op = sum((w * g).sum() for w, g in zip(ws, g_op))
    h_ref = torch.autograd.grad(s_ref, [*in_ref, *cot_ref], allow_unused=True)
    h_op = torch.autograd.grad(s_op, [*in_op, *cot_op], allow_unused=True)
    targets = [*names, *[f"grad_{op.outputs[i]}" for i in diff]]
    for name, a, b in zip(targets, h_op, h_ref):
        if a is None and b is None:
            continue
        a = torch.zeros_like(b) if a is None else a
        b = torch.zeros_like(a) if b is None else b
        errors[f"backward2.{name}"] = rel_err(a, b)
    return errors


def _as_tuple(out) -> tuple:
    return tuple(out) if isinstance(out, tuple | list) else (out,)
