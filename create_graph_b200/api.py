"""
The entry points ``create_graph``, ``compile`` and ``reset``.

    out, grads = cg.create_graph(model, data, outputs="energy", inputs=("pos",))
    loss = loss_fn(out, -grads["pos"])
    loss.backward()

The contract is the reference's (src/create_graph/api.py:148-253 there): the
named entries of ``data`` (dict keys or attributes) are differentiated,
``model(data)`` runs once, and ``grads[name]`` is the gradient of
``sum(out[outputs])`` with respect to ``data[name]``, differentiable with
respect to the parameters in training. The arguments, defaults and
``ContractError`` texts are kept so that user code and tests run unchanged.

How it is done here: an ``_InputSwap`` puts fresh leaves into ``data`` for
the duration of the model call (guarded so that the model itself cannot
differentiate them); the one ``cg.compile`` region whose inputs depend on them
records its differentiated output and the gradients of its inputs while it
runs (create_graph_b200.region), and ``create_graph`` chains those back to
the leaves.
"""

from __future__ import annotations

import warnings
from collections.abc import Callable, Sequence

import torch
from torch import Tensor, nn

from create_graph_b200.compile_config import (
    CompileConfig,
    reset_compiled,
    supports_in_graph_grad,
    warn_eager_fallback,
)
from create_graph_b200.errors import ContractError
from create_graph_b200.pytree import tree_map_tensors
from create_graph_b200.region import (
    STATES,
    Region,
    RegionModule,
    State,
    reset_regions,
    select_output,
)

_GRAD_IN_MODEL = (
    "create_graph: the model computed a gradient w.r.t. a differentiated input during "
    "create_graph (torch.autograd.grad or backward). The model must only compute the "
    "energy here (switch off the force computation of its heads); create_graph computes "
    "the gradients."
)


def get_input(data, key: str) -> Tensor:
    """``data[key]`` for mappings, ``data.key`` otherwise."""
    return data[key] if isinstance(data, dict) else getattr(data, key)


class _InputSwap:
    """Fresh leaves in place of the differentiated entries of ``data`` while the
    model runs; the original tensors are back afterwards, whatever happens.
    A hook on every leaf turns any gradient the model itself takes w.r.t. them
    into the contract error (create_graph computes those gradients)."""

    def __init__(self, data, names: Sequence[str]):
        self.data = data
        self.leaves = {name: get_input(data, name).detach().requires_grad_(True) for name in names}
        self._saved: dict[str, Tensor] = {}
        self._hooks: list = []

    def _write(self, key: str, value) -> None:
        if isinstance(self.data, dict):
            self.data[key] = value
        else:
            setattr(self.data, key, value)

    def __enter__(self) -> _InputSwap:
        for key, leaf in self.leaves.items():
            self._saved[key] = get_input(self.data, key)
            self._write(key, leaf)
            self._hooks.append(leaf.register_hook(_refuse_gradient))
        return self

    def __exit__(self, *exc) -> None:
        for hook in self._hooks:
            hook.remove()
        for key, original in self._saved.items():
            self._write(key, original)


def _refuse_gradient(_grad):
    raise ContractError(_GRAD_IN_MODEL)


def _default_train(model) -> bool:
    return torch.is_grad_enabled() and bool(getattr(model, "training", True))


def _check_output(target: Tensor, state: State) -> None:
    """The region computed the VJP of sum(selected); the model's differentiated
    output may be selected itself (or a view with its entries), or selected
    plus terms that do not depend on the differentiated inputs.

    The region ran on detached copies of its inputs, so selected's autograd
    graph never reaches the create_graph leaves: one gradient query of
    sum(target) w.r.t. (selected, leaves) gives both the coefficient of every
    entry of selected (must be exactly 1) and whether target reaches a leaf
    along some other path (any gradient that is not None). Returning the
    region's output itself skips the query and its host synchronisation."""
    selected = state.region.selected
    if target is selected or (
        target.numel() == selected.numel()
        and target.data_ptr() == selected.data_ptr()
        and target.untyped_storage().data_ptr() == selected.untyped_storage().data_ptr()
    ):
        return
    message = (
        "create_graph: the differentiated model output is not the output of region "
        f"{state.region.name} (or a view with the same entries)"
    )
    if not (target.requires_grad and selected.requires_grad):
        raise ContractError(message + ".")
    leaves = list(state.leaves.values())
    weight, *through_leaves = torch.autograd.grad(
        target.sum(), [selected, *leaves], retain_graph=True, allow_unused=True
    )
    if weight is None:
        raise ContractError(message + ", and it is not computed from it.")
    if any(g is not None for g in through_leaves):
        raise ContractError(
            message + ": it also depends on the differentiated inputs through code after the "
            "region. Move that code into the region."
        )
    if not bool((weight == 1).all()):
        raise ContractError(
            message + ": code after the region scales or drops entries of the region's output. "
            "Move that code into the region, or let the region return what the model returns."
        )


_WARNED_NO_REGION: set[int] = set()


def _warn_no_region(model, names) -> None:
    if id(model) in _WARNED_NO_REGION:
        return
    _WARNED_NO_REGION.add(id(model))
    warnings.warn(
        "create_graph: the model ran no cg.compile region that depends on "
        f"{', '.join(names)}, so the gradients come from eager create_graph. Mark the "
        "part of the model that computes the energy with cg.compile.",
        stacklevel=3,
    )


def create_graph(
    model: Callable,
    data,
    *,
    outputs: str | Callable | None = "energy",
    inputs: str | Sequence[str] = ("pos",),
    train: bool | None = None,
    exact: bool = False,
):
    """``(model(data), grads)``: the model output and, for every name in
    ``inputs``, ``grads[name]`` = d sum(out[outputs]) / d data.<name>.

    ``train`` (default: grad enabled and the model in training mode) makes the
    grads differentiable w.r.t. the parameters, so ``loss(out, grads).backward()``
    is the parameter gradient of the conservative-force loss; ``train=False``
    gives first-order grads and detached outputs (validation, MD).
    ``exact=True`` runs plain eager ``torch.autograd.grad(create_graph=True)``,
    the reference semantics for tests. Under DDP pass the wrapped model.
    """
    names = (inputs,) if isinstance(inputs, str) else tuple(inputs)
    train = _default_train(model) if train is None else train
    if not exact and not supports_in_graph_grad():
        warn_eager_fallback("create_graph")
        exact = True
    swap = _InputSwap(data, names)
    state = State(leaves=swap.leaves, train=train, exact=exact, outputs=outputs)
    STATES.append(state)
    try:
        with swap, torch.enable_grad():
            out = model(data)
    except RuntimeError as error:
        # regions differentiate detached copies of their inputs, so a gradient
        # the model takes w.r.t. an input reaches autograd as an unused tensor
        if "not have been used in the graph" in str(error):
            raise ContractError(_GRAD_IN_MODEL) from error
        raise
    finally:
        STATES.pop()

    target = select_output(out, outputs)
    leaves = list(swap.leaves.values())
    if state.exact or state.region is None:
        if not exact:
            _warn_no_region(model, names)
        found = torch.autograd.grad(target.sum(), leaves, create_graph=train, allow_unused=True)
        if not train:
            out = tree_map_tensors(Tensor.detach, out)
    else:
        _check_output(target, state)
        found = state.region.input_grads(leaves, train)
    grads = {name: g if g is not None else torch.zeros_like(leaf)
             for (name, leaf), g in zip(swap.leaves.items(), found)}
    return out, grads


def compile(
    fn: Callable | nn.Module | None = None,
    *,
    config: CompileConfig | None = None,
    outputs: str | Callable | None = None,
):
    """Mark ``fn`` (a function, method or nn.Module) as a create_graph region; a
    drop-in for ``torch.compile``, also as a decorator. Inside create_graph the
    region computes its differentiated output (``outputs``, default the
    create_graph call's) and its VJP over the package's fused kernels."""
    if fn is None:
        return lambda f: compile(f, config=config, outputs=outputs)
    return RegionModule(fn, config, outputs) if isinstance(fn, nn.Module) else Region(fn, config, outputs)


def reset() -> None:
    """Forget region plans and checks; the next call builds them again."""
    reset_regions()
    reset_compiled()
