"""
How a create_graph region runs, and the only module of the package that
touches private torch APIs.

``CompileConfig`` keeps the fields, defaults and validation of
src/create_graph/compile_config.py:25-66. What they mean here:

- ``backend``: "inductor" (default) and "aot_eager" run the region's forward
  and its force pass over the package's sm_100a fused ops, with the refusal
  of user ``torch.autograd.Function`` nodes on the differentiated path that
  the reference applies to compiled regions (src/create_graph/region.py:223-275);
  "eager" runs the same ops without that check. There is no tracing compiler:
  the first-order graph is built by autograd over opaque fused kernels.
- ``dynamic``: accepted for compatibility. Every kernel takes its sizes at run
  time, so no batch size ever recompiles anything.
- ``memory_budget``: fraction in (0, 1] of the activation bytes a region may
  keep (None: 1). The reference hands it to AOTAutograd's min-cut
  partitioner; here the fused ops read it through ``active_memory_budget()``
  when they record their saved tensors, and give up the intermediates that
  are cheapest to rebuild, in three tiers:

  - below 1: the FFN's second-order factor u = g W2 (rows x FFN width) is not
    kept by the force pass; the parameter backward rebuilds it with one GEMM;
  - 0.5 or less: also the FFN's SiLU activation (rows x FFN width), rebuilt
    from its pre-activation by one elementwise kernel;
  - 0.25 or less: also every LayerNorm output held for the gamma gradient
    (rows x hidden), rebuilt from the normalisation input.

  Rebuilt tensors equal the kept ones bit for bit (same kernels, same
  inputs), so a budget changes peak memory and time, not results. Inside
  ``checkpoint`` blocks it applies to the block being recomputed; above 0.25
  checkpointed blocks also keep results across their recomputes and defer
  part of the parameter backward (create_graph_b200.checkpoint), which sums
  the parameter gradients in another order than at 0.25 or less.
- ``checkpoint``: regex of block module paths recomputed per block
  (create_graph_b200.checkpoint).
- ``options``: free (key, value) pairs, kept sorted and hashable.
- ``recompile_error``: accepted for compatibility (nothing recompiles).
"""

from __future__ import annotations

import contextlib
import dataclasses
import functools
import warnings
from typing import Any

import torch

BACKENDS = ("inductor", "aot_eager", "eager")


@dataclasses.dataclass(frozen=True)
class CompileConfig:
    """How a create_graph region runs (see the module docstring)."""

    backend: str = "inductor"
    dynamic: bool | None = True
    memory_budget: float | None = None
    checkpoint: str | None = None
    options: tuple[tuple[str, Any], ...] = ()
    recompile_error: bool = False

    def __post_init__(self):
        if self.backend not in BACKENDS:
            raise ValueError(f"backend must be one of {BACKENDS}, got {self.backend!r}")
        budget = self.memory_budget
        if budget is not None and not (0.0 < budget <= 1.0):
            raise ValueError(f"memory_budget must be in (0, 1], got {budget}")
        if isinstance(self.options, dict):
            object.__setattr__(self, "options", tuple(sorted(self.options.items())))

    def replace(self, **changes) -> CompileConfig:
        return dataclasses.replace(self, **changes)


DEFAULT_CONFIG = CompileConfig()


@functools.cache
def supports_in_graph_grad() -> bool:
    """Whether regions can put the force pass into the region's own graph.

    Always true here: the force pass is autograd over fused ops, which needs no
    tracing support from torch (the reference needs torch >= 2.11 for Dynamo
    to trace ``torch.autograd.grad``, src/create_graph/compile_config.py:88-102).
    """
    return True


_FALLBACK_WARNED: set[str] = set()


def warn_eager_fallback(where: str) -> None:
    """One warning per call site when a region runs as plain eager create_graph."""
    if where in _FALLBACK_WARNED:
        return
    _FALLBACK_WARNED.add(where)
    warnings.warn(
        f"create_graph: torch {torch.__version__} cannot trace torch.autograd.grad into a "
        f"compiled graph (needs torch >= 2.11), so {where} runs as eager create_graph: exact, "
        "but not compiled.",
        stacklevel=3,
    )


# ---------------------------------------------------------------------------
# the scope of a region call
# ---------------------------------------------------------------------------

_ACTIVE: list[CompileConfig] = []


@contextlib.contextmanager
def compile_context(config: CompileConfig, recompile_limit: int | None = None):
    """Scope of every region and block call: makes ``config`` the active one,
    so fused ops see its memory budget."""
    _ACTIVE.append(config)
    try:
        yield
    finally:
        _ACTIVE.pop()


def active_config() -> CompileConfig | None:
    return _ACTIVE[-1] if _ACTIVE else None


def active_memory_budget() -> float:
    """The memory budget of the innermost active region (1.0 outside regions)."""
    config = active_config()
    if config is None or config.memory_budget is None:
        return 1.0
    return float(config.memory_budget)


# ---------------------------------------------------------------------------
# autograd-graph introspection (private torch APIs live here only)
# ---------------------------------------------------------------------------


def is_python_function_node(node) -> bool:
    """Whether an autograd node belongs to a user ``torch.autograd.Function``.

    Nodes of torch.library custom ops (their generated Functions) and of the
    package's own fused ops are not user Functions.
    """
    if not isinstance(node, torch.autograd.function.BackwardCFunction):
        return False
    if getattr(getattr(node, "_forward_cls", None), "_cg_fused", False):
        return False
    name = type(node).__name__
    return not name.startswith("GeneratedBackwardFor")


def gradient_edge(t: torch.Tensor):
    """The autograd node a gradient for ``t`` flows into (None if ``t`` needs none)."""
    if not t.requires_grad:
        return None
    try:
        return torch.autograd.graph.get_gradient_edge(t).node
    except AssertionError:
        # a view made in no-grad mode (inside a backward without create_graph):
        # the op recording it is never differentiated again
        return None


def engine_will_execute(node) -> bool:
    """Whether the backward pass running now reaches ``node``.

    Used by fused ops to skip gradients nobody asked for: during the force pass
    (``autograd.grad`` w.r.t. positions) the parameters' accumulation nodes are
    not executed, so weight gradients are not computed there.
    """
    if node is None:
        return False
    try:
        return bool(torch._C._will_engine_execute_node(node))
    except RuntimeError:
        # not inside a backward pass: be conservative
        return True


_PLANS: list[int] = [0]


def note_plan() -> None:
    """Count a new region plan (a region, config and mode seen for the first time)."""
    _PLANS[0] += 1


def compiled_graph_count() -> int:
    """Region plans built in this process: one per region, config and mode,
    never one per batch size (kernels take sizes at run time)."""
    return _PLANS[0]


def reset_compiled() -> None:
    _PLANS[0] = 0
