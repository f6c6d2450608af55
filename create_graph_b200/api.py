"""
The entry points ``create_graph``, ``compile`` and ``reset``.

    out, grads = cg.create_graph(model, data, outputs="energy", inputs=("pos",))
    loss = loss_fn(out, -grads["pos"])
    loss.backward()

Behaviour follows src/create_graph/api.py:148-253: ``data.<input>`` (or
``data[input]``) is swapped for a fresh leaf, ``model(data)`` runs once, and
``grads[input]`` is the gradient of ``sum(out[outputs])`` w.r.t. it,
differentiable w.r.t. the parameters when training.
"""

from __future__ import annotations

import contextlib
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

_grad = torch.autograd.grad


def get_input(data, key: str) -> Tensor:
    return data[key] if isinstance(data, dict) else getattr(data, key)


def _set_input(data, key: str, value) -> None:
    if isinstance(data, dict):
        data[key] = value
    else:
        setattr(data, key, value)


@contextlib.contextmanager
def swapped_inputs(data, values: dict[str, Tensor]):
    originals = {key: get_input(data, key) for key in values}
    for key, value in values.items():
        _set_input(data, key, value)
    try:
        yield
    finally:
        for key, value in originals.items():
            _set_input(data, key, value)


_GRAD_IN_MODEL = (
    "create_graph: the model computed a gradient w.r.t. a differentiated input during "
    "create_graph (torch.autograd.grad or backward). The model must only compute the "
    "energy here (switch off the force computation of its heads); create_graph computes "
    "the gradients."
)


def _forbidden_grad(grad):
    raise ContractError(_GRAD_IN_MODEL)


@contextlib.contextmanager
def _no_input_gradients(leaves: dict[str, Tensor]):
    """While the model runs, nothing may differentiate w.r.t. the inputs."""
    handles = [leaf.register_hook(_forbidden_grad) for leaf in leaves.values()]
    try:
        yield
    finally:
        for handle in handles:
            handle.remove()


def _same_entries(target: Tensor, selected: Tensor) -> bool:
    """``target`` is ``selected`` or a view of it with the same elements."""
    if target is selected:
        return True
    return (
        target.numel() == selected.numel()
        and target.data_ptr() == selected.data_ptr()
        and target.untyped_storage().data_ptr() == selected.untyped_storage().data_ptr()
    )


def _reaches_inputs_besides(target: Tensor, selected: Tensor, state: State) -> bool:
    """Whether ``target`` depends on the differentiated inputs other than through ``selected``."""
    inputs = state.leaf_index()
    stop = selected.grad_fn
    todo = [target.grad_fn] if target.grad_fn is not None else []
    seen = set()
    while todo:
        node = todo.pop()
        if node is None or node is stop or node in seen:
            continue
        seen.add(node)
        variable = getattr(node, "variable", None)
        if variable is not None and id(variable) in inputs:
            return True
        todo.extend(child for child, _ in node.next_functions)
    return False


def _check_output(target: Tensor, state: State) -> None:
    """The region's VJP is that of sum(selected): the model's output must have the
    same entries, or add to them terms independent of the differentiated inputs
    (src/create_graph/api.py:115-142). Returning the region's output itself
    avoids the one host synchronisation this check can cost."""
    selected = state.region.selected
    if _same_entries(target, selected):
        return
    message = (
        "create_graph: the differentiated model output is not the output of region "
        f"{state.region.name} (or a view with the same entries)"
    )
    if not (target.requires_grad and selected.requires_grad):
        raise ContractError(message + ".")
    (weight,) = _grad(target.sum(), selected, retain_graph=True, allow_unused=True)
    if weight is None:
        raise ContractError(message + ", and it is not computed from it.")
    if _reaches_inputs_besides(target, selected, state):
        raise ContractError(
            message + ": it also depends on the differentiated inputs through code after the "
            "region. Move that code into the region."
        )
    if not bool(torch.all(weight == 1)):
        raise ContractError(
            message + ": code after the region scales or drops entries of the region's output. "
            "Move that code into the region, or let the region return what the model returns."
        )


_NO_REGION_WARNED: set[int] = set()


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
    if train is None:
        train = torch.is_grad_enabled() and bool(getattr(model, "training", True))
    if not exact and not supports_in_graph_grad():
        warn_eager_fallback("create_graph")
        exact = True
    leaves = {name: get_input(data, name).detach().requires_grad_(True) for name in names}
    state = State(leaves=leaves, train=train, exact=exact, outputs=outputs)
    STATES.append(state)
    try:
        with swapped_inputs(data, leaves), torch.enable_grad(), _no_input_gradients(leaves):
            out = model(data)
    except RuntimeError as error:
        # the region works on detached copies, so a gradient taken inside the
        # model w.r.t. an input surfaces as autograd's "not been used" error
        if "not have been used in the graph" in str(error):
            raise ContractError(_GRAD_IN_MODEL) from error
        raise
    finally:
        STATES.pop()
    target = select_output(out, outputs)
    leaf_list = list(leaves.values())
    if state.exact or state.region is None:
        if not exact and id(model) not in _NO_REGION_WARNED:
            _NO_REGION_WARNED.add(id(model))
            warnings.warn(
                "create_graph: the model ran no cg.compile region that depends on "
                f"{', '.join(names)}, so the gradients come from eager create_graph. Mark the "
                "part of the model that computes the energy with cg.compile.",
                stacklevel=2,
            )
        found = _grad(target.sum(), leaf_list, create_graph=train, allow_unused=True)
        if not train:
            out = tree_map_tensors(lambda t: t.detach(), out)
    else:
        _check_output(target, state)
        found = state.region.input_grads(leaf_list, train)
    grads = {
        name: torch.zeros_like(leaf) if g is None else g
        for (name, leaf), g in zip(leaves.items(), found)
    }
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
    if isinstance(fn, nn.Module):
        return RegionModule(fn, config, outputs)
    return Region(fn, config, outputs)


def reset() -> None:
    """Forget region plans and checks; the next call builds them again."""
    reset_regions()
    reset_compiled()
