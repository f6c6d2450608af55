"""
Fused operators on the path from positions to the energy: ``cg.custom_op``.

The contract is that of src/create_graph/ops.py:1-36. create_graph
differentiates such an op twice: its VJP is part of the force pass
(backward1), and the parameter backward differentiates that VJP (backward2).
One class declares all three kernels:

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
Underneath are three ``torch.library.custom_op`` operators (``name``,
``name_backward1``, ``name_backward2``) and two ``register_autograd`` calls;
the package's own edge-attention op is registered through this very class
with sm_100a kernel bodies.
"""

from __future__ import annotations

import inspect
import typing

import torch
from torch import Tensor

from create_graph_b200.errors import ContractError

_SCALARS = {float: "float", int: "SymInt", bool: "bool", str: "str"}


def _scalar_schema(hint, name: str) -> str:
    try:
        return _SCALARS[hint]
    except (KeyError, TypeError):
        allowed = [t.__name__ for t in _SCALARS]
        raise ContractError(
            f"cg.custom_op: argument {name!r} of forward1 has type {hint!r}; non-tensor "
            f"arguments must be one of {allowed}"
        ) from None


def _tuple(out) -> tuple:
    return tuple(out) if isinstance(out, tuple | list) else (out,)


def _fresh(outs: tuple, args: tuple) -> tuple:
    """Outputs as the fakes describe them: new contiguous tensors (an op may not
    return one of its arguments, src/create_graph/ops.py:64-71)."""
    arg_ids = {id(a) for a in args if isinstance(a, Tensor)}
    fixed = []
    for o in outs:
        if isinstance(o, Tensor):
            if id(o) in arg_ids:
                o = o.clone()
            o = o.contiguous()
        fixed.append(o)
    return tuple(fixed)


def _like(t: Tensor) -> Tensor:
    return torch.empty(t.shape, dtype=t.dtype, device=t.device)


def _result_schema(n: int) -> str:
    return "Tensor" if n == 1 else "(" + ", ".join("Tensor" for _ in range(n)) + ")"


def _single_or_tuple(outs: tuple, n: int):
    return outs if n > 1 else outs[0]


class FusedOp:
    """The three registered operators of a ``cg.custom_op`` class. Calling it
    calls forward1."""

    def __init__(self, name: str, spec: type):
        forward1 = spec.forward1
        hints = typing.get_type_hints(forward1)
        self.name = name
        self.params = list(inspect.signature(forward1).parameters)
        self.tensor_args = [p for p in self.params if hints.get(p) is Tensor]
        self.other_args = [p for p in self.params if p not in self.tensor_args]
        self.outputs = tuple(spec.outputs)
        self.save = tuple(spec.save)
        self.nondiff = tuple(getattr(spec, "nondiff", ()))
        self.diff_outputs = [o for o in self.outputs if o not in self.nondiff]
        known = {*self.params, *self.outputs}
        for n in (*self.save, *self.nondiff):
            if n not in known:
                raise ContractError(f"cg.custom_op {name}: {n!r} is not an argument or output")

        self.op = torch.library.custom_op(name, mutates_args=())(forward1)
        if hasattr(spec, "fake"):
            self.op.register_fake(spec.fake)

        scalars = [f"{_scalar_schema(hints[p], p)} {p}" for p in self.other_args]
        self.bwd1_tensors = [*self.save, *(f"grad_{o}" for o in self.diff_outputs)]
        self.bwd1_params = [*self.bwd1_tensors, *self.other_args]
        self.bwd1_diff = [n for n in self.bwd1_tensors if n not in self.nondiff]
        n1, n2 = len(self.tensor_args), len(self.bwd1_diff)
        tensors1 = [f"Tensor {n}" for n in self.bwd1_tensors]
        ggs = [f"Tensor gg_{p}" for p in self.tensor_args]
        schema1 = f"({', '.join(tensors1 + scalars)}) -> {_result_schema(n1)}"
        schema2 = f"({', '.join(tensors1 + scalars + ggs)}) -> {_result_schema(n2)}"

        def backward1_body(*args):
            return _single_or_tuple(_fresh(_tuple(spec.backward1(*args)), args), n1)

        def backward2_body(*args):
            return _single_or_tuple(_fresh(_tuple(spec.backward2(*args)), args), n2)

        self.backward1_op = torch.library.custom_op(
            f"{name}_backward1", backward1_body, mutates_args=(), schema=schema1
        )
        self.backward2_op = torch.library.custom_op(
            f"{name}_backward2", backward2_body, mutates_args=(), schema=schema2
        )
        self._fakes(spec, n1, n2)
        self._autograd()

    def _fakes(self, spec, n1: int, n2: int) -> None:
        order = self.bwd1_tensors
        if hasattr(spec, "backward1_fake"):
            self.backward1_op.register_fake(spec.backward1_fake)
        elif all(p in self.save for p in self.tensor_args):
            where = [order.index(p) for p in self.tensor_args]

            def backward1_fake(*args):
                return _single_or_tuple(tuple(_like(args[i]) for i in where), n1)

            self.backward1_op.register_fake(backward1_fake)
        else:
            raise ContractError(
                f"cg.custom_op {self.name}: backward1 returns a gradient for every tensor input "
                "of forward1, so save them all, or give backward1_fake"
            )
        where2 = [order.index(n) for n in self.bwd1_diff]

        def backward2_fake(*args):
            return _single_or_tuple(tuple(_like(args[i]) for i in where2), n2)

        self.backward2_op.register_fake(backward2_fake)

    def _autograd(self) -> None:
        op = self

        def setup1(ctx, inputs, output):
            named = dict(zip(op.params, inputs))
            named.update(zip(op.outputs, _tuple(output)))
            ctx.save_for_backward(*[named[n] for n in op.save])
            ctx.others = [named[p] for p in op.other_args]
            stats = [named[n] for n in op.nondiff if n in op.outputs]
            if stats:
                ctx.mark_non_differentiable(*stats)

        def backward1(ctx, *grads):
            diff = [g for o, g in zip(op.outputs, grads) if o not in op.nondiff]
            found = iter(_tuple(op.backward1_op(*ctx.saved_tensors, *diff, *ctx.others)))
            return tuple(next(found) if p in op.tensor_args else None for p in op.params)

        self.op.register_autograd(backward1, setup_context=setup1)

        def setup2(ctx, inputs, output):
            named = dict(zip(op.bwd1_params, inputs))
            ctx.save_for_backward(*[named[n] for n in op.bwd1_tensors])
            ctx.others = [named[p] for p in op.other_args]

        def backward2(ctx, *ggs):
            found = iter(_tuple(op.backward2_op(*ctx.saved_tensors, *ctx.others, *ggs)))
            return tuple(next(found) if n in op.bwd1_diff else None for n in op.bwd1_params)

        self.backward1_op.register_autograd(backward2, setup_context=setup2)

    def __call__(self, *args, **kwargs):
        return self.op(*args, **kwargs)


def custom_op(name: str):
    """Register a class with ``forward1`` / ``backward1`` / ``backward2`` as a
    fused operator that create_graph differentiates twice (module docstring)."""

    def decorate(spec: type) -> FusedOp:
        return FusedOp(name, spec)

    return decorate
