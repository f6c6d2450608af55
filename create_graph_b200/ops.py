"""
Fused operators on the path from positions to the energy: ``cg.custom_op``.

The plugin contract is the reference's (src/create_graph/ops.py:1-36 there),
kept so that its op classes register unchanged. create_graph differentiates
such an op twice: its VJP is part of the force pass (backward1) and the
parameter backward differentiates that VJP (backward2). One class declares all
three kernels:

    @cg.custom_op("mylib::attn")
    class Attention:
        outputs = ("out", "lse")
        save = ("q", "k", "v", "lse")      # what forward1 keeps for backward1
        nondiff = ("lse",)                 # outputs that are statistics

        @staticmethod
        def forward1(q: Tensor, k: Tensor, v: Tensor, scale: float) -> tuple[Tensor, Tensor]: ...
        @staticmethod
        def backward1(q, k, v, lse, grad_out, scale): ...       # grads of q, k, v
        @staticmethod
        def backward2(q, k, v, lse, grad_out, scale, gg_q, gg_k, gg_v): ...
                                       # grads of q, k, v, grad_out (not of statistics)
        @staticmethod
        def fake(q, k, v, scale): ...   # output shapes of forward1

backward1 takes the saved tensors, the cotangents ``grad_<name>`` of the
differentiable outputs and the non-tensor arguments of forward1, and returns
one gradient per tensor input of forward1. backward2 takes backward1's
arguments followed by the cotangents ``gg_<input>`` of backward1's outputs,
and returns the gradients of backward1's tensor arguments except statistics.

How it is built here: a ``_Plan`` works out the argument list of each of the
three operators from the class once; the three ``torch.library`` operators,
their fakes and the two autograd links (forward1 -> backward1 -> backward2)
are all derived from it. The package's own edge-attention op is registered
through this very class with sm_100a kernel bodies.
"""

from __future__ import annotations

import dataclasses
import inspect
import typing

import torch
from torch import Tensor

from create_graph_b200.checkpoint import cut_forward_tensor, deferral_slot, deferred_cotangent, plus
from create_graph_b200.errors import ContractError

# schema types of the non-tensor arguments forward1 may take
_SCALAR_TYPES = {float: "float", int: "SymInt", bool: "bool", str: "str"}


def _as_tuple(x) -> tuple:
    return tuple(x) if isinstance(x, (tuple, list)) else (x,)


def _returns(count: int) -> str:
    return "Tensor" if count == 1 else f"({', '.join(['Tensor'] * count)})"


def _pack(values: tuple, count: int):
    """A single tensor for one-output schemas, the tuple otherwise."""
    return values[0] if count == 1 else values


def _owned(results: tuple, args: tuple) -> tuple:
    """Results as the registered fakes promise them: fresh contiguous tensors.
    An op body may hand back one of its arguments (an identity gradient); the
    operator returns a copy instead (torch custom ops may not alias inputs)."""
    out = []
    for r in results:
        if isinstance(r, Tensor):
            if any(r is a for a in args):
                r = r.clone()
            r = r.contiguous()
        out.append(r)
    return tuple(out)


@dataclasses.dataclass(frozen=True)
class _Plan:
    """Argument lists of forward1, backward1 and backward2 for one op class."""

    name: str
    params: tuple[str, ...]          # forward1's arguments, in order
    tensors: tuple[str, ...]         # those typed Tensor
    scalars: tuple[tuple[str, str], ...]  # (name, schema type) of the others
    outputs: tuple[str, ...]
    save: tuple[str, ...]
    nondiff: tuple[str, ...]

    @staticmethod
    def of(name: str, spec: type) -> _Plan:
        hints = typing.get_type_hints(spec.forward1)
        params = tuple(inspect.signature(spec.forward1).parameters)
        tensors = tuple(p for p in params if hints.get(p) is Tensor)
        scalars = []
        for p in params:
            if p in tensors:
                continue
            kind = _SCALAR_TYPES.get(hints.get(p)) if isinstance(hints.get(p), type) else None
            if kind is None:
                raise ContractError(
                    f"cg.custom_op: argument {p!r} of forward1 has type {hints.get(p)!r}; non-tensor "
                    f"arguments must be one of {[t.__name__ for t in _SCALAR_TYPES]}"
                )
            scalars.append((p, kind))
        plan = _Plan(name, params, tensors, tuple(scalars), tuple(spec.outputs), tuple(spec.save),
                     tuple(getattr(spec, "nondiff", ())))
        known = set(plan.params) | set(plan.outputs)
        for n in (*plan.save, *plan.nondiff):
            if n not in known:
                raise ContractError(f"cg.custom_op {name}: {n!r} is not an argument or output")
        return plan

    @property
    def scalar_names(self) -> tuple[str, ...]:
        return tuple(n for n, _ in self.scalars)

    @property
    def diff_outputs(self) -> tuple[str, ...]:
        return tuple(o for o in self.outputs if o not in self.nondiff)

    @property
    def bwd1_tensors(self) -> tuple[str, ...]:
        """backward1's tensor arguments: the saved tensors, then the cotangents."""
        return (*self.save, *(f"grad_{o}" for o in self.diff_outputs))

    @property
    def bwd1_diff(self) -> tuple[str, ...]:
        """backward1's tensor arguments backward2 differentiates (not statistics)."""
        return tuple(n for n in self.bwd1_tensors if n not in self.nondiff)

    def schema(self, level: int) -> str:
        """Schema of backward1 (level 1) or backward2 (level 2)."""
        args = [f"Tensor {n}" for n in self.bwd1_tensors] + [f"{kind} {n}" for n, kind in self.scalars]
        if level == 1:
            return f"({', '.join(args)}) -> {_returns(len(self.tensors))}"
        args += [f"Tensor gg_{p}" for p in self.tensors]
        return f"({', '.join(args)}) -> {_returns(len(self.bwd1_diff))}"


class FusedOp:
    """The three registered operators of a ``cg.custom_op`` class. Calling it
    calls forward1."""

    def __init__(self, name: str, spec: type):
        plan = _Plan.of(name, spec)
        self.plan = plan
        self.name = name
        self.params = list(plan.params)
        self.tensor_args = list(plan.tensors)
        self.other_args = list(plan.scalar_names)
        self.outputs, self.save, self.nondiff = plan.outputs, plan.save, plan.nondiff
        self.diff_outputs = list(plan.diff_outputs)
        self.bwd1_tensors = list(plan.bwd1_tensors)
        self.bwd1_params = [*plan.bwd1_tensors, *plan.scalar_names]
        self.bwd1_diff = list(plan.bwd1_diff)

        self.op = torch.library.custom_op(name, mutates_args=())(spec.forward1)
        if hasattr(spec, "fake"):
            self.op.register_fake(spec.fake)
        n1, n2 = len(plan.tensors), len(plan.bwd1_diff)
        self.backward1_op = torch.library.custom_op(
            f"{name}_backward1", lambda *a: _pack(_owned(_as_tuple(spec.backward1(*a)), a), n1),
            mutates_args=(), schema=plan.schema(1))
        self.backward2_op = torch.library.custom_op(
            f"{name}_backward2", lambda *a: _pack(_owned(_as_tuple(spec.backward2(*a)), a), n2),
            mutates_args=(), schema=plan.schema(2))
        self.backward1_op.register_fake(self._backward1_fake(spec, n1))
        self.backward2_op.register_fake(self._shapes_of(plan.bwd1_diff, n2))
        self._link_first_derivative()
        self._link_second_derivative()

    def _shapes_of(self, names, count: int):
        """A fake returning empty tensors shaped like the named backward1 args."""
        where = [self.plan.bwd1_tensors.index(n) for n in names]

        def fake(*args):
            return _pack(tuple(torch.empty_like(args[i], memory_format=torch.contiguous_format) for i in where),
                         count)

        return fake

    def _backward1_fake(self, spec, count: int):
        if hasattr(spec, "backward1_fake"):
            return spec.backward1_fake
        if not set(self.plan.tensors) <= set(self.plan.save):
            raise ContractError(
                f"cg.custom_op {self.name}: backward1 returns a gradient for every tensor input "
                "of forward1, so save them all, or give backward1_fake"
            )
        return self._shapes_of(self.plan.tensors, count)

    def _link_first_derivative(self) -> None:
        """forward1's backward is backward1 on the saved tensors. Inside
        checkpointed blocks the op takes part in the deferred first-order
        backward (create_graph_b200.checkpoint): backward1 reads the saved
        tensors through cut_forward_tensor, and the deferred cotangents of saved
        inputs join their gradients, those of saved outputs their cotangents."""
        plan = self.plan
        backward1_op = self.backward1_op

        def setup(ctx, inputs, output):
            values = dict(zip(plan.params, inputs))
            values.update(zip(plan.outputs, _as_tuple(output)))
            ctx.save_for_backward(*(values[n] for n in plan.save))
            ctx.scalars = [values[n] for n in plan.scalar_names]
            statistics = [values[n] for n in plan.nondiff if n in plan.outputs]
            if statistics:
                ctx.mark_non_differentiable(*statistics)
            ctx.op = deferral_slot()

        def backward(ctx, *cotangents):
            saved = [cut_forward_tensor(ctx, n, t) for n, t in zip(plan.save, ctx.saved_tensors)]
            wanted = [plus(c, deferred_cotangent(ctx, o)) if o in plan.save else c
                      for o, c in zip(plan.outputs, cotangents) if o not in plan.nondiff]
            grads = dict(zip(plan.tensors, _as_tuple(backward1_op(*saved, *wanted, *ctx.scalars))))
            return tuple(plus(grads.get(p), deferred_cotangent(ctx, p)) if p in plan.save else grads.get(p)
                         for p in plan.params)

        self.op.register_autograd(backward, setup_context=setup)

    def _link_second_derivative(self) -> None:
        """backward1's backward is backward2 on backward1's own arguments."""
        plan = self.plan
        backward2_op = self.backward2_op
        n_tensors = len(plan.bwd1_tensors)

        def setup(ctx, inputs, output):
            ctx.save_for_backward(*inputs[:n_tensors])
            ctx.scalars = list(inputs[n_tensors:])

        def backward(ctx, *cotangents):
            grads = dict(zip(plan.bwd1_diff, _as_tuple(backward2_op(*ctx.saved_tensors, *ctx.scalars, *cotangents))))
            return tuple(grads.get(n) for n in (*plan.bwd1_tensors, *plan.scalar_names))

        self.backward1_op.register_autograd(backward, setup_context=setup)

    def __call__(self, *args, **kwargs):
        return self.op(*args, **kwargs)


def custom_op(name: str):
    """Register a class with ``forward1`` / ``backward1`` / ``backward2`` as a
    fused operator that create_graph differentiates twice (module docstring)."""

    def decorate(spec: type) -> FusedOp:
        return FusedOp(name, spec)

    return decorate
