"""
``cg.compile`` regions and what they do inside ``cg.create_graph``.

Semantics follow src/create_graph/region.py:1-431. Outside create_graph a
region simply runs its function. Inside, the region whose inputs depend on the
differentiated inputs runs its function and
``torch.autograd.grad(sum(selected output), region inputs, create_graph=train)``
back to back: the force pass. Inside the region every compute op is a fused op
with sm_100a forward1 / backward1 / backward2 kernels, so the force pass is
autograd calling backward1 kernels, and the later ``loss.backward()`` calls
their backward2 kernels: one first-order graph of hand-written kernels. The
region-input gradients are chained to the differentiated inputs through the
eager code before the region afterwards (``RegionResult.input_grads``).

Region inputs, classified by what their autograd graph reaches
(src/create_graph/region.py:14-21, 125-154):

- only the differentiated inputs (geometry): enter as detached leaves, so the
  parameter backward does not run through the eager geometry twice;
- the differentiated inputs and other leaves (parameters mixed with geometry
  before the region): enter unchanged, their cotangents are chained as well;
- other leaves only: enter unchanged and need no gradient from the force pass.
"""

from __future__ import annotations

import contextlib
import dataclasses
import functools
import types
from collections.abc import Callable
from typing import Any

import torch
from torch import Tensor, nn

from create_graph_b200.checkpoint import checkpointed_blocks, forces_pass
from create_graph_b200.compile_config import (
    DEFAULT_CONFIG,
    CompileConfig,
    compile_context,
    is_python_function_node,
    note_plan,
)
from create_graph_b200.errors import ContractError
from create_graph_b200.pytree import flatten, is_float, tree_map_tensors, unflatten

_grad = torch.autograd.grad

# bits of what a tensor's autograd graph reaches
INPUT, OTHER = 1, 2


def select_output(out, outputs):
    """The differentiated tensor of ``out``: ``outputs`` names a key or an
    attribute, or is a callable, or is None (``out`` itself). A tensor ``out``
    is taken as it is (src/create_graph/region.py:58-67)."""
    if outputs is None or isinstance(out, Tensor):
        return out
    if callable(outputs):
        return outputs(out)
    return out[outputs] if isinstance(out, dict) else getattr(out, outputs)


@dataclasses.dataclass
class RegionResult:
    """The differentiated output of the one region that depends on the
    differentiated inputs, and the gradients it computed for them.

    ``items`` holds ("chain", region input, grad) for region inputs computed
    from the differentiated inputs by eager code, and ("direct", index, grad)
    for a differentiated input passed to the region as it is.
    """

    name: str
    selected: Tensor
    items: list[tuple[str, Any, Tensor | None]]

    def input_grads(self, leaves: list[Tensor], train: bool) -> list[Tensor | None]:
        """Gradients w.r.t. ``leaves``: chained cotangents through the eager code
        before the region, plus the direct ones (src/create_graph/region.py:86-102)."""
        result: list[Tensor | None] = [None] * len(leaves)
        chained = [(x, g) for kind, x, g in self.items if kind == "chain" and g is not None]
        if chained:
            result = list(
                _grad(
                    [x for x, _ in chained],
                    leaves,
                    [g for _, g in chained],
                    create_graph=train,
                    allow_unused=True,
                )
            )
        for kind, index, g in self.items:
            if kind != "direct" or g is None:
                continue
            result[index] = g if result[index] is None else result[index] + g
        return result


@dataclasses.dataclass
class State:
    """One create_graph call in progress."""

    leaves: dict[str, Tensor]
    train: bool
    exact: bool
    outputs: Any
    memo: dict = dataclasses.field(default_factory=dict)
    region: RegionResult | None = None

    def leaf_index(self) -> dict[int, int]:
        return {id(t): i for i, t in enumerate(self.leaves.values())}


STATES: list[State] = []


def active_state() -> State | None:
    return STATES[-1] if STATES else None


def _reach(node, state: State) -> int:
    """INPUT/OTHER bits of the leaves below ``node``, memoised per call."""
    memo = state.memo
    if node in memo:
        return memo[node]
    inputs = state.leaf_index()
    # iterative post-order walk: graphs of deep models overflow recursion
    todo = [(node, False)]
    while todo:
        current, expanded = todo.pop()
        if current in memo:
            continue
        below = [child for child, _ in current.next_functions if child is not None]
        if not expanded:
            todo.append((current, True))
            todo.extend((child, False) for child in below if child not in memo)
            continue
        bits = 0
        variable = getattr(current, "variable", None)
        if variable is not None:
            bits = INPUT if id(variable) in inputs else OTHER
        for child in below:
            bits |= memo[child]
        memo[current] = bits
    return memo[node]


def tensor_kinds(t: Tensor, state: State) -> int:
    if not (is_float(t) and t.requires_grad):
        return 0
    if t.grad_fn is None:
        return INPUT if id(t) in state.leaf_index() else OTHER
    return _reach(t.grad_fn, state)


def fn_key(fn) -> Any:
    if isinstance(fn, types.FunctionType):
        return fn.__code__
    if isinstance(fn, types.MethodType):
        return (id(fn.__self__), fn.__func__.__code__)
    return id(fn)


_PLANS: set = set()
_CHECKED: set = set()


def _plan(kind: str, region: Region) -> None:
    key = (kind, fn_key(region.fn), region.config)
    if key not in _PLANS:
        _PLANS.add(key)
        note_plan()


def reset_regions() -> None:
    _PLANS.clear()
    _CHECKED.clear()


def _refuse_functions(region: Region, args, kwargs, wrt: list[Tensor]) -> None:
    """Once per region and config (unless backend="eager"): run the region and
    refuse user ``torch.autograd.Function`` nodes on the path from the
    differentiated inputs to its output, as the reference does for compiled
    regions (src/create_graph/region.py:223-275). A Function applied to
    parameters only is accepted."""
    key = (fn_key(region.fn), region.config)
    if region.config.backend == "eager" or key in _CHECKED:
        return
    _CHECKED.add(key)
    with torch.enable_grad():
        out = region.fn(*args, **kwargs)
    targets = {id(t) for t in wrt}
    reaches: dict = {}

    def reaches_inputs(node) -> bool:
        todo = [(node, False)]
        while todo:
            current, expanded = todo.pop()
            if current in reaches:
                continue
            below = [child for child, _ in current.next_functions if child is not None]
            if not expanded:
                todo.append((current, True))
                todo.extend((child, False) for child in below if child not in reaches)
                continue
            variable = getattr(current, "variable", None)
            mine = variable is not None and id(variable) in targets
            reaches[current] = mine or any(reaches[child] for child in below)
        return reaches[node]

    roots = [t.grad_fn for t in flatten(out)[0] if isinstance(t, Tensor) and t.grad_fn is not None]
    seen: set = set()
    while roots:
        node = roots.pop()
        if node in seen:
            continue
        seen.add(node)
        below = [child for child, _ in node.next_functions if child is not None]
        if is_python_function_node(node) and any(reaches_inputs(c) for c in below):
            name = type(node).__name__.removesuffix("Backward")
            raise ContractError(
                f"create_graph: region {region.name} applies the torch.autograd.Function "
                f"{name} on the path from the differentiated inputs to its output. Its backward "
                "is not differentiated again inside a compiled region (wrong parameter "
                "gradients). Register the kernel with cg.custom_op (forward1, backward1, "
                "backward2) or torch.library.custom_op + register_autograd, or use "
                "CompileConfig(backend='eager') for this region."
            )
        roots.extend(below)


def _force_pass(region: Region, args, kwargs, wrt, keep, outputs, create: bool):
    """The region's forward and its VJP w.r.t. ``wrt`` (src/create_graph/region.py:191-198)."""
    with torch.enable_grad():
        out = region.fn(*args, **kwargs)
        target = select_output(out, outputs)
        with forces_pass():
            grads = _grad(target.sum(), wrt, create_graph=create, allow_unused=True)
    if not create:
        out = tree_map_tensors(lambda t: t.detach(), out)
    return out, tuple(g for g, k in zip(grads, keep) if k)


class Region:
    """``cg.compile(fn)``: ``fn`` itself outside create_graph; inside it, the
    region's forward and force pass over fused sm_100a ops."""

    def __init__(self, fn: Callable, config: CompileConfig | None = None, outputs=None):
        self.fn = fn
        self.config = config if config is not None else DEFAULT_CONFIG
        self.outputs = outputs
        functools.update_wrapper(self, fn, updated=())

    @property
    def name(self) -> str:
        return getattr(self.fn, "__qualname__", None) or type(self.fn).__name__

    def __get__(self, obj, objtype=None):
        if obj is None:
            return self
        return Region(types.MethodType(self.fn, obj), self.config, self.outputs)

    def normal(self, *args, **kwargs):
        """A call outside create_graph (or one that does not depend on the
        differentiated inputs): the function under the region's config."""
        if self.config.backend != "eager":
            _plan("normal", self)
        with compile_context(self.config):
            return self.fn(*args, **kwargs)

    def __call__(self, *args, **kwargs):
        if torch.compiler.is_compiling():
            return self.fn(*args, **kwargs)
        state = active_state()
        if state is None:
            return self.normal(*args, **kwargs)
        if state.exact:
            return self.fn(*args, **kwargs)
        return region_call(state, self, args, kwargs)


class RegionModule(nn.Module):
    """``cg.compile(module)``: the whole module is one region."""

    def __init__(self, module: nn.Module, config: CompileConfig | None = None, outputs=None):
        super().__init__()
        self.module = module
        self._region = Region(module.forward, config, outputs)

    def forward(self, *args, **kwargs):
        return self._region(*args, **kwargs)


def _module_roots(region: Region, leaves: list) -> list[nn.Module]:
    roots = []
    owner = getattr(region.fn, "__self__", None)
    if isinstance(owner, nn.Module):
        roots.append(owner)
    roots.extend(x for x in leaves if isinstance(x, nn.Module))
    return roots


_SCALAR_TYPES = (Tensor, nn.Module, int, float, bool, str)


def _object_attributes(state: State, leaves: list) -> list[tuple[object, str, Tensor, int]]:
    """Float tensor attributes of plain objects among the region's arguments
    (fairchem's AtomicData and the like) that require grad: (object, name,
    tensor, kinds)."""
    found = []
    for obj in leaves:
        if obj is None or isinstance(obj, _SCALAR_TYPES):
            continue
        attrs = getattr(obj, "__dict__", None)
        if not isinstance(attrs, dict):
            continue
        for name, value in list(attrs.items()):
            if isinstance(value, Tensor):
                bits = tensor_kinds(value, state)
                if bits:
                    found.append((obj, name, value, bits))
    return found


def region_call(state: State, region: Region, args, kwargs):
    """The region inside create_graph (src/create_graph/region.py:359-431)."""
    leaves, spec = flatten((args, kwargs))
    kinds = [tensor_kinds(x, state) if isinstance(x, Tensor) else 0 for x in leaves]
    attributes = _object_attributes(state, leaves)
    if not any(k & INPUT for k in kinds) and not any(a[3] & INPUT for a in attributes):
        return region.normal(*args, **kwargs)
    if state.region is not None:
        raise ContractError(
            f"create_graph: regions {state.region.name} and {region.name} both depend on the "
            "differentiated inputs. Exactly one region may produce the differentiated output: "
            "merge them into one cg.compile region (e.g. backbone network and energy head)."
        )

    inputs = state.leaf_index()
    wrt: list[Tensor] = []
    keep: list[bool] = []
    items: list[tuple[str, Any]] = []
    entered: dict[int, Tensor] = {}

    def enter(x: Tensor, bits: int) -> Tensor:
        if id(x) in entered:
            return entered[id(x)]
        if bits == INPUT or id(x) in inputs:
            new = x.detach().requires_grad_(True)
            wrt.append(new)
            keep.append(True)
            items.append(("direct", inputs[id(x)]) if id(x) in inputs else ("chain", x))
        else:
            new = x
            wrt.append(x)
            keep.append(bool(bits & INPUT))
            if bits & INPUT:
                items.append(("chain", x))
        entered[id(x)] = new
        return new

    new_leaves = [enter(x, k) if k else x for x, k in zip(leaves, kinds)]
    swaps = [(obj, name, value, enter(value, k)) for obj, name, value, k in attributes]
    new_args, new_kwargs = unflatten(spec, new_leaves)
    outputs = region.outputs if region.outputs is not None else state.outputs

    for obj, name, _, new in swaps:
        setattr(obj, name, new)
    try:
        _refuse_functions(region, new_args, new_kwargs, wrt)
        if region.config.checkpoint is not None:
            out, grads = _checkpointed(state, region, new_args, new_kwargs, new_leaves, wrt, keep, outputs)
        else:
            _plan("train" if state.train else "eval", region)
            with compile_context(region.config):
                out, grads = _force_pass(
                    region, new_args, new_kwargs, tuple(wrt), tuple(keep), outputs, state.train
                )
    finally:
        for obj, name, original, _ in swaps:
            setattr(obj, name, original)

    selected = select_output(out, outputs)
    if not is_float(selected):
        raise ContractError(
            f"create_graph: region {region.name} must return the differentiated output as a "
            f"float tensor (selected with outputs={outputs!r}), got {type(selected).__name__}."
        )
    state.region = RegionResult(
        name=region.name,
        selected=selected,
        items=[(kind, ref, g) for (kind, ref), g in zip(items, grads)],
    )
    return out


def _checkpointed(state, region, args, kwargs, leaves, wrt, keep, outputs):
    """A region with per-block recompute (src/create_graph/region.py:434-444)."""
    _plan("blocks", region)
    roots = _module_roots(region, leaves)
    with contextlib.ExitStack() as stack:
        stack.enter_context(compile_context(region.config))
        stack.enter_context(checkpointed_blocks(roots, region.config))
        stack.enter_context(torch.enable_grad())
        out = region.fn(*args, **kwargs)
    target = select_output(out, outputs)
    with compile_context(region.config), forces_pass():
        grads = _grad(target.sum(), wrt, create_graph=state.train, allow_unused=True)
    if not state.train:
        out = tree_map_tensors(lambda t: t.detach(), out)
    return out, tuple(g for g, k in zip(grads, keep) if k)
