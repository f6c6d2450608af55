"""Flattening of region arguments and outputs into leaves and a hashable spec.

Behaviour follows src/create_graph/pytree.py:20-80: tuples, lists, namedtuples,
dicts (and OrderedDicts) and dataclasses whose fields are all ``init`` fields
are containers; everything else (tensors, numbers, strings, plain objects such
as fairchem's AtomicData) is a leaf. A spec is built from tuples of types,
names and child specs only, so it can key a cache.
"""

from __future__ import annotations

import dataclasses
from collections import OrderedDict
from typing import Any

from torch import Tensor

_SEQ, _MAP, _DC = "seq", "map", "dc"


def _is_namedtuple(obj) -> bool:
    return isinstance(obj, tuple) and hasattr(type(obj), "_fields")


def _spec_of(obj, out: list):
    kind = type(obj)
    if kind in (tuple, list) or _is_namedtuple(obj):
        return (_SEQ, kind, tuple(_spec_of(child, out) for child in obj))
    if kind in (dict, OrderedDict):
        keys = tuple(obj.keys())
        return (_MAP, kind, keys, tuple(_spec_of(obj[key], out) for key in keys))
    if dataclasses.is_dataclass(obj) and not isinstance(obj, type):
        fields = dataclasses.fields(obj)
        if all(field.init for field in fields):
            names = tuple(field.name for field in fields)
            return (_DC, kind, names, tuple(_spec_of(getattr(obj, n), out) for n in names))
    out.append(obj)
    return None


def flatten(obj) -> tuple[list, Any]:
    """``(leaves, spec)`` of ``obj``; ``unflatten(spec, leaves)`` rebuilds it."""
    leaves: list = []
    spec = _spec_of(obj, leaves)
    return leaves, spec


def _build(spec, it):
    if spec is None:
        return next(it)
    tag = spec[0]
    if tag == _SEQ:
        _, kind, children = spec
        values = [_build(child, it) for child in children]
        if kind in (tuple, list):
            return kind(values)
        return kind(*values)
    _, kind, names, children = spec
    values = [_build(child, it) for child in children]
    if tag == _MAP:
        return kind(zip(names, values))
    return kind(**dict(zip(names, values)))


def unflatten(spec, leaves) -> Any:
    return _build(spec, iter(leaves))


def is_float(x) -> bool:
    """A floating-point (or complex) tensor: the only kind that carries gradients."""
    return isinstance(x, Tensor) and (x.is_floating_point() or x.is_complex())


def tree_map_tensors(fn, obj):
    leaves, spec = flatten(obj)
    return unflatten(spec, [fn(x) if isinstance(x, Tensor) else x for x in leaves])
