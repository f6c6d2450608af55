"""
Acceptance checks for models and fused operators.

The public checks of src/create_graph/testing.py:21-208 there, with the same
names, arguments and error keys, so parity tests read like the reference's own
and report comparable numbers:

- ``check_create_graph(model, data)``: create_graph against ``exact=True`` on
  the same parameters and data (output, input gradients, a loss coupling
  both, parameter gradients);
- ``check_float32(...)`` / ``as_close_as_eager(...)``: float32 create_graph
  and float32 eager create_graph, each against float64 eager;
- ``check_op(op, reference, args)``: a ``cg.custom_op`` against a
  differentiable reference at three derivative levels.

Errors are relative norms in float64 on the CPU. For parameter gradients two
numbers are reported: all gradients concatenated, and the worst single tensor,
whose scale is floored at 1e-4 of the whole gradient's norm (a tensor whose
reference gradient is ~0 would otherwise report rounding noise).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor, nn

from create_graph_b200.api import create_graph
from create_graph_b200.region import select_output


def _f64(t: Tensor) -> Tensor:
    return t.detach().to(device="cpu", dtype=torch.float64)


def rel_err(got: Tensor, want: Tensor) -> float:
    """||got - want|| / ||want|| in float64 (want's norm floored at 1e-300)."""
    want64 = _f64(want)
    return float(torch.linalg.vector_norm(_f64(got) - want64) / torch.linalg.vector_norm(want64).clamp_min(1e-300))


def grad_errors(got: Sequence[Tensor], want: Sequence[Tensor]) -> dict[str, float]:
    """``all``: relative error of the concatenated gradients; ``worst_tensor``:
    the largest per-tensor error, each scaled by max(its norm, 1e-4 x total)."""
    pairs = [(_f64(g).flatten(), _f64(w).flatten()) for g, w in zip(got, want)]
    diff_sq = [torch.dot(g - w, g - w) for g, w in pairs]
    want_sq = [torch.dot(w, w) for _, w in pairs]
    total = torch.stack(want_sq).sum().sqrt()
    floor = 1e-4 * total
    worst = max(float(d.sqrt() / torch.maximum(w.sqrt(), floor)) for d, w in zip(diff_sq, want_sq))
    return {"all": float(torch.stack(diff_sq).sum().sqrt() / total.clamp_min(1e-300)), "worst_tensor": worst}


def param_grads(model: nn.Module) -> list[Tensor]:
    """Copies of the trainable parameters' gradients (zeros where unset)."""
    return [p.grad.detach().clone() if p.grad is not None else torch.zeros_like(p)
            for p in model.parameters() if p.requires_grad]


class CoupledLoss:
    """sum(w_out * out) + |out|^2 / 2 + sum over input gradients g of
    (sum(w_g * g) + |g|^2 / 2): couples the output and its gradients linearly
    and quadratically. Each quantity's weights are drawn once, in first-use
    order, from torch.Generator seeds seed, seed + 1, ..., and reused by every
    later call, so two steps of one model see the same loss."""

    def __init__(self, seed: int = 0):
        self.seed = seed
        self._weights: dict[str, Tensor] = {}

    def weight(self, key: str, like: Tensor) -> Tensor:
        w = self._weights.get(key)
        if w is None:
            gen = torch.Generator().manual_seed(self.seed + len(self._weights))
            w = self._weights[key] = torch.randn(like.shape, generator=gen, dtype=torch.float64)
        return w.to(like)

    def __call__(self, target: Tensor, grads: dict[str, Tensor]) -> Tensor:
        terms = [(self.weight("out", target) * target).sum() + 0.5 * target.square().sum()]
        terms += [(self.weight(name, g) * g).sum() + 0.5 * g.square().sum() for name, g in grads.items()]
        return torch.stack(terms).sum()


def coupled_loss(seed: int = 0) -> Callable:
    """A ``CoupledLoss`` (callable as ``loss(target, grads)``)."""
    return CoupledLoss(seed)


def run_step(model, data, *, outputs, inputs, loss: Callable, exact: bool) -> dict:
    """One training step from cleared gradients: create_graph (train=True),
    ``loss(target, grads).backward()``; returns the detached output, input
    grads, loss and parameter grads, and leaves the parameters' grads cleared."""
    trainable = [p for p in model.parameters() if p.requires_grad]
    for p in trainable:
        p.grad = None
    out, grads = create_graph(model, data, outputs=outputs, inputs=inputs, train=True, exact=exact)
    target = select_output(out, outputs)
    value = loss(target, grads)
    value.backward()
    record = {"out": target.detach(), "grads": {k: g.detach() for k, g in grads.items()}, "loss": value.detach(),
              "params": param_grads(model)}
    for p in trainable:
        p.grad = None
    return record


def step_errors(got: dict, want: dict) -> dict[str, float]:
    """Per quantity of two ``run_step`` results: out, loss, grad_<input>,
    params (all) and params_worst_tensor."""
    errors = {key: rel_err(got[key], want[key]) for key in ("out", "loss")}
    errors.update({f"grad_{name}": rel_err(g, want["grads"][name]) for name, g in got["grads"].items()})
    stats = grad_errors(got["params"], want["params"])
    errors["params"], errors["params_worst_tensor"] = stats["all"], stats["worst_tensor"]
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
    loss = loss if loss is not None else CoupledLoss()
    kw = {"outputs": outputs, "inputs": inputs, "loss": loss}
    return step_errors(run_step(model, data, exact=False, **kw), run_step(model, data, exact=True, **kw))


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
    loss = loss if loss is not None else CoupledLoss()
    kw = {"outputs": outputs, "inputs": inputs, "loss": loss}
    want = run_step(model64, data64, exact=True, **kw)
    return {label: step_errors(run_step(model32, data32, exact=exact, **kw), want)
            for label, exact in (("create_graph", False), ("eager", True))}


def as_close_as_eager(result: dict, floor: dict[str, float], factor: float = 4.0) -> dict:
    """Quantities (among ``floor``'s keys) where create_graph's float32 error
    exceeds both the floor and ``factor`` times eager create_graph's; empty when
    create_graph is as accurate as eager."""
    mine, eager = result["create_graph"], result["eager"]
    return {key: (mine[key], eager[key]) for key in floor
            if key in mine and mine[key] > max(floor[key], factor * eager[key])}


class _Derivatives:
    """A callable's outputs and its first and second derivatives at fixed
    random probes: backward1 = the input gradients for output cotangents c
    (taken with create_graph); backward2 = the gradients of sum(w * backward1)
    w.r.t. the inputs and the cotangents."""

    def __init__(self, fn: Callable, args: Sequence):
        self.args = [a.detach().clone().requires_grad_(a.is_floating_point()) if isinstance(a, Tensor) else a
                     for a in args]
        out = fn(*self.args)
        self.outputs = tuple(out) if isinstance(out, (tuple, list)) else (out,)
        self.inputs = [a for a in self.args if isinstance(a, Tensor) and a.requires_grad]

    def backward1(self, diff: list[int], cotangents: list[Tensor]) -> tuple:
        self.cotangents = [c.clone().requires_grad_(True) for c in cotangents]
        self.first = torch.autograd.grad([self.outputs[i] for i in diff], self.inputs, self.cotangents,
                                         create_graph=True)
        return self.first

    def backward2(self, weights: list[Tensor]) -> tuple:
        s = torch.stack([(w * g).sum() for w, g in zip(weights, self.first)]).sum()
        return torch.autograd.grad(s, [*self.inputs, *self.cotangents], allow_unused=True)


def check_op(op, reference: Callable, args: Sequence, *, seed: int = 20260917) -> dict[str, float]:
    """forward1, backward1 and backward2 of a ``cg.custom_op`` against a
    differentiable ``reference`` with the same signature: the outputs; the
    input gradients for random cotangents of the differentiable outputs; and
    the gradients of a random linear function of those input gradients w.r.t.
    the inputs and the cotangents. The random cotangents and weights come from
    ``seed``'s stream (draw the inputs from another one), on the args' device."""
    gen = torch.Generator().manual_seed(seed)
    mine, ref = _Derivatives(op, args), _Derivatives(reference, args)
    errors = {f"forward1.{name}": rel_err(a, b) for name, a, b in zip(op.outputs, mine.outputs, ref.outputs)}

    diff = [i for i, name in enumerate(op.outputs) if name not in op.nondiff]
    cotangents = [torch.randn(ref.outputs[i].shape, generator=gen, dtype=torch.float64).to(ref.outputs[i])
                  for i in diff]
    first_mine, first_ref = mine.backward1(diff, cotangents), ref.backward1(diff, cotangents)
    tensor_names = [name for name, a in zip(op.params, args) if isinstance(a, Tensor)]
    errors.update({f"backward1.{name}": rel_err(a, b) for name, a, b in zip(tensor_names, first_mine, first_ref)})

    weights = [torch.randn(g.shape, generator=gen, dtype=torch.float64).to(g) for g in first_ref]
    second_mine, second_ref = mine.backward2(weights), ref.backward2(weights)
    targets = [*tensor_names, *(f"grad_{op.outputs[i]}" for i in diff)]
    for name, a, b in zip(targets, second_mine, second_ref):
        if a is None and b is None:
            continue
        errors[f"backward2.{name}"] = rel_err(a if a is not None else torch.zeros_like(b),
                                              b if b is not None else torch.zeros_like(a))
    return errors
