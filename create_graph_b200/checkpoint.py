"""
Per-block recompute of a region (``CompileConfig.checkpoint``).

Semantics follow src/create_graph/checkpoint.py:1-334. The region runs
eagerly, and each submodule whose path matches the pattern (``re.fullmatch``
over ``named_modules()``) becomes one ``BlockFn`` node of the autograd graph:

- forward: the block runs without grad; only its inputs are kept;
- force pass (``forces_pass()`` is active): the node's backward returns the
  input cotangents from a ``VjpFn`` node, which runs the block's forward and
  VJP without keeping anything;
- parameter backward: ``VjpFn`` recomputes forward + VJP with grad and
  differentiates it (backward2); ``BlockFn`` recomputes the forward and returns
  its first-order gradients.

So a block's forward runs four times and its VJP twice, and at most one
block's activations are alive at a time. Each call keeps a RecomputeCache:
the pooled attention keeps its softmax statistics and its output (n x C)
from the first forward, and the linear layers and LayerNorms their outputs
(the larger ones from a memory budget of 0.5), so the three recomputes take them instead of
running those kernels again, and the VJP's pooled-attention backward1 and
input-gradient GEMMs keep their outputs from the force pass for the VJP's
rebuild in the parameter backward, which takes them instead of recomputing;
the memory budget decides whether they may (create_graph_b200.nn).

Deferred first-order backward (budget above 0.25): VjpFn.backward
differentiates the block's VJP; the second-order terms that reach the forward
tensors the VJP's ops read would run the block's forward ops' backward, which
BlockFn.backward runs again on the energy's cotangent. So while the VJP is
rebuilt the ops read those tensors through leaves, VjpFn.backward stops at
them, and the cotangents they receive are added by each op's backward inside
BlockFn.backward (backward is linear in its cotangents): the forward ops'
backward runs once per block. Block i's own backward waits for the gradient
of its output, which the VJP of block i+1 produces after block i's, so the
deferred cotangents are there; if the block's backward ever ran first,
VjpFn.backward does the whole differentiation itself. The block's fused ops are
the same sm_100a kernels as elsewhere; the recompute runs under the region's
config, so its memory budget applies inside the blocks too.
"""

from __future__ import annotations

import contextlib
import re
from collections.abc import Iterable

import torch
from torch import Tensor, nn

from create_graph_b200.compile_config import compile_context
from create_graph_b200.errors import ContractError
from create_graph_b200.pytree import flatten, is_float, unflatten

_grad = torch.autograd.grad

FORCES_PASS: list[bool] = [False]


class RecomputeCache:
    """Small results a checkpointed block's ops keep across the recomputes of
    one block call (its first forward and every recompute see the same inputs,
    so they produce the same values): ops ask for a slot in call order and
    either find what the first run left there or fill it."""

    def __init__(self):
        self.slots: dict[object, object] = {}
        self._next = 0
        self._next_op = 0
        # set while the block's VJP (create_graph's force pass, or its rebuild
        # in the parameter backward) runs: both see the same output cotangents
        self.in_vjp = False
        # deferred first-order backward (VjpFn.backward / BlockFn.backward):
        # while ``cutting``, ops building the VJP's graph read their forward
        # tensors through leaves (``cuts``, keyed by (op, role)); the cotangents
        # those leaves receive wait in ``pending`` for the block's own backward
        self.cutting = False
        self.cuts: dict[tuple[int, str], Tensor] = {}
        self.pending: dict[tuple[int, str], Tensor] = {}

    def start(self) -> None:
        self._next = 0
        self._next_op = 0

    def slot(self) -> int:
        self._next += 1
        return self._next - 1

    def op(self) -> int:
        """The next op's index in this forward (the same in every run of the call)."""
        self._next_op += 1
        return self._next_op - 1


_CACHES: list[RecomputeCache] = []


def active_recompute_cache() -> RecomputeCache | None:
    """The cache of the checkpointed block call whose forward is running, if any."""
    return _CACHES[-1] if _CACHES else None


# ---------------------------------------------------------------------------
# Deferred first-order backward: the hooks an op uses to take part
#
# The parameter backward differentiates a block's VJP (VjpFn.backward); the
# second-order terms that reach the forward tensors the VJP's ops read would
# then run the block's forward ops' backward, which the block's own backward
# (BlockFn.backward, on the energy's cotangent) runs again later. An op that
# takes part records ``ctx.op = deferral_slot()`` in its forward; its backward
# reads the forward tensors it builds on through ``cut_forward_tensor`` (leaves
# while the VJP is rebuilt, so the differentiation stops there) and adds
# ``deferred_cotangent`` (what those leaves received, handed out once in the
# block's own backward) to the gradient of the same tensor. Ops without the
# hooks are differentiated in full, which is also correct.
# ---------------------------------------------------------------------------


def deferral_slot():
    """(cache, index) of an op inside a checkpointed block call (the same in
    every run of the call's forward), else None."""
    cache = active_recompute_cache()
    return (cache, cache.op()) if cache is not None else None


def cut_forward_tensor(ctx, role: str, t: Tensor | None) -> Tensor | None:
    """t, or a leaf standing for it while the block's VJP is rebuilt with its
    forward ops' share deferred (one leaf per op and role)."""
    op = getattr(ctx, "op", None)
    if op is None or t is None or not op[0].cutting:
        return t
    cache, index = op
    leaf = cache.cuts.get((index, role))
    if leaf is None:
        leaf = t.detach().requires_grad_(t.requires_grad)
        cache.cuts[(index, role)] = leaf
    return leaf


def deferred_cotangent(ctx, role: str) -> Tensor | None:
    """The deferred cotangent of the op's tensor ``role``, taken once (in the
    block's own backward), or None."""
    op = getattr(ctx, "op", None)
    if op is None or not op[0].pending:
        return None
    cache, index = op
    return cache.pending.pop((index, role), None)


def plus(g: Tensor | None, c: Tensor | None) -> Tensor | None:
    """g + c where either may be None."""
    if c is None:
        return g
    return c if g is None else g + c


@contextlib.contextmanager
def forces_pass():
    """Marks the region's force pass (the VJP create_graph computes)."""
    FORCES_PASS.append(True)
    try:
        yield
    finally:
        FORCES_PASS.pop()


def in_forces_pass() -> bool:
    return FORCES_PASS[-1]


class _BlockCall:
    """One call of a checkpointed block: its arguments, differentiable slots
    and outputs."""

    def __init__(self, block: nn.Module, config, args, kwargs):
        self.block = block
        self.config = config
        self.leaves, self.spec = flatten((args, kwargs))
        self.slots = tuple(i for i, x in enumerate(self.leaves) if is_float(x) and x.requires_grad)
        self.params = [p for p in block.parameters() if p.requires_grad]
        self.out_leaves: list = []
        self.out_spec = None
        self.out_slots: tuple[int, ...] = ()
        self.cache = RecomputeCache()
        # whether the parameter backward has run this call's first-order
        # backward (BlockFn.backward) yet
        self.backward_done = False

    def defers(self) -> bool:
        """Whether VjpFn.backward may leave the forward ops' part of its
        backward to BlockFn.backward: the block's own backward is still to
        come and the memory budget (above 0.25) allows holding the cotangents."""
        budget = self.config.memory_budget
        return not self.backward_done and (budget is None or budget > 0.25)

    @property
    def inputs(self) -> list[Tensor]:
        return [self.leaves[i] for i in self.slots]

    def run(self, tensors):
        """The block's own forward on ``tensors`` in its differentiable slots."""
        leaves = list(self.leaves)
        for i, t in zip(self.slots, tensors):
            leaves[i] = t
        args, kwargs = unflatten(self.spec, leaves)
        self.cache.start()
        _CACHES.append(self.cache)
        try:
            with compile_context(self.config):
                return type(self.block).forward(self.block, *args, **kwargs)
        finally:
            _CACHES.pop()

    def vjp(self, tensors, g_outs, create: bool):
        """Cotangents of the block inputs for output cotangents ``g_outs``."""
        with torch.enable_grad():
            outs = self.selected(self.run(tensors))
            pairs = [(o, g) for o, g in zip(outs, g_outs) if o.requires_grad]
            if not pairs:
                return [None] * len(tensors)
            self.cache.in_vjp = True
            try:
                return _grad(
                    [o for o, _ in pairs],
                    list(tensors),
                    [g for _, g in pairs],
                    create_graph=create,
                    allow_unused=True,
                )
            finally:
                self.cache.in_vjp = False

    def keep_output(self, out) -> tuple[Tensor, ...]:
        """The block's float outputs become the node's outputs, except tensors it
        passes through unchanged from non-differentiable arguments."""
        self.out_leaves, self.out_spec = flatten(out)
        constant = {
            id(x)
            for i, x in enumerate(self.leaves)
            if isinstance(x, Tensor) and i not in set(self.slots)
        }
        self.out_slots = tuple(
            i for i, x in enumerate(self.out_leaves) if is_float(x) and id(x) not in constant
        )
        return tuple(self.out_leaves[i] for i in self.out_slots)

    def selected(self, out) -> list[Tensor]:
        leaves = flatten(out)[0]
        return [leaves[i] for i in self.out_slots]

    def rebuild(self, tensors):
        leaves = list(self.out_leaves)
        for i, t in zip(self.out_slots, tensors):
            leaves[i] = t
        self.out_leaves = []  # the node keeps the call alive: drop the forward's outputs
        return unflatten(self.out_spec, leaves)


def _leaf(t: Tensor, requires_grad: bool | None = None) -> Tensor:
    flag = t.requires_grad if requires_grad is None else requires_grad
    return t.detach().requires_grad_(flag)


class VjpFn(torch.autograd.Function):
    """The block's VJP as a node: input cotangents from (inputs, output
    cotangents, parameters); its backward is the block's backward2."""

    @staticmethod
    def forward(ctx, call: _BlockCall, n_out: int, *tensors):
        n = len(call.slots)
        inputs, g_outs = tensors[:n], tensors[n : n + n_out]
        ctx.call = call
        ctx.save_for_backward(*inputs, *g_outs)
        grads = call.vjp([_leaf(t, True) for t in inputs], [g.detach() for g in g_outs], False)
        return tuple(torch.zeros_like(t) if g is None else g for g, t in zip(grads, inputs))

    @staticmethod
    def backward(ctx, *ggs):
        call: _BlockCall = ctx.call
        saved = ctx.saved_tensors
        n = len(call.slots)
        inputs, g_outs = saved[:n], saved[n:]
        cache = call.cache
        cache.pending = {}
        with torch.enable_grad():
            li = [_leaf(t, True) for t in inputs]
            lg = [_leaf(g, True) for g in g_outs]
            # deferred: the ops that build the VJP's graph read their forward
            # tensors through leaves, so this backward stops at them; the
            # cotangents the leaves get are the forward ops' share, which the
            # block's own backward (BlockFn.backward) adds to its output
            # cotangents' so that the forward ops' backward runs once
            cache.cutting, cache.cuts = call.defers(), {}
            try:
                outs = call.vjp(li, lg, True)
            finally:
                cache.cutting = False
            cuts = [(key, leaf) for key, leaf in cache.cuts.items() if leaf.requires_grad]
            cache.cuts = {}
            pairs = [
                (o, gg)
                for o, gg in zip(outs, ggs)
                if o is not None and gg is not None and o.requires_grad
            ]
            wanted = [*li, *lg, *call.params, *(leaf for _, leaf in cuts)]
            if pairs:
                grads = _grad([o for o, _ in pairs], wanted, [gg for _, gg in pairs], allow_unused=True)
            else:
                grads = [None] * len(wanted)
        if cuts:
            found = grads[len(grads) - len(cuts):]
            cache.pending = {key: g for (key, _), g in zip(cuts, found) if g is not None}
            grads = grads[: len(grads) - len(cuts)]
        return (None, None, *grads)


class BlockFn(torch.autograd.Function):
    """A checkpointed block: keeps its inputs only."""

    @staticmethod
    def forward(ctx, call: _BlockCall, *tensors):
        inputs = tensors[: len(call.slots)]
        ctx.call = call
        ctx.save_for_backward(*inputs)
        with torch.no_grad():
            out = call.run([t.detach() for t in inputs])
        return call.keep_output(out)

    @staticmethod
    def backward(ctx, *g_outs):
        call: _BlockCall = ctx.call
        inputs = ctx.saved_tensors
        n_params = len(call.params)
        if in_forces_pass():
            grads_in = VjpFn.apply(call, len(g_outs), *inputs, *g_outs, *call.params)
            return (None, *grads_in, *([None] * n_params))
        call.backward_done = True
        pending = call.cache.pending
        with torch.enable_grad():
            leaves = [_leaf(t) for t in inputs]
            outs = call.selected(call.run(leaves))
            if pending:
                # the VJP's deferred cotangents enter inside the block (each op's
                # backward adds its own): every op must be reached
                g_outs = [torch.zeros_like(o) if g is None and o.requires_grad else g for o, g in zip(outs, g_outs)]
            pairs = [(o, g) for o, g in zip(outs, g_outs) if g is not None and o.requires_grad]
            every = [*leaves, *call.params]
            wanted = [t for t in every if t.requires_grad]
            if pairs and wanted:
                found = iter(_grad([o for o, _ in pairs], wanted, [g for _, g in pairs], allow_unused=True))
            else:
                found = iter([None] * len(wanted))
            grads = [next(found) if t.requires_grad else None for t in every]
        if pending:
            left = sorted(pending)
            pending.clear()
            raise RuntimeError(f"checkpoint: deferred cotangents of {left} reached no op of the block's backward")
        return (None, *grads)


def _wrapped_forward(block: nn.Module, config):
    def forward(*args, **kwargs):
        call = _BlockCall(block, config, args, kwargs)
        outs = BlockFn.apply(call, *call.inputs, *call.params)
        return call.rebuild(outs)

    return forward


def matching_blocks(roots: Iterable[nn.Module], pattern: str) -> list[nn.Module]:
    """Submodules whose path ``re.fullmatch``es ``pattern``; a match nested in an
    earlier match belongs to that block (src/create_graph/checkpoint.py:302-314)."""
    found: list[nn.Module] = []
    seen: set[int] = set()
    for root in roots:
        for name, module in root.named_modules():
            if id(module) in seen or not re.fullmatch(pattern, name):
                continue
            if any(module in set(outer.modules()) for outer in found):
                continue
            seen.add(id(module))
            found.append(module)
    return found


@contextlib.contextmanager
def checkpointed_blocks(roots: list[nn.Module], config):
    pattern = config.checkpoint
    blocks = matching_blocks(roots, pattern)
    if not blocks:
        names = ", ".join(type(r).__name__ for r in roots) or "no nn.Module"
        raise ContractError(
            f"create_graph: CompileConfig(checkpoint={pattern!r}) matched no submodule of the "
            f"region's modules ({names}). The pattern is matched with re.fullmatch against "
            "names from named_modules() of the region's self and module arguments."
        )
    for block in blocks:
        block.forward = _wrapped_forward(block, config)
    try:
        yield blocks
    finally:
        for block in blocks:
            del block.forward
