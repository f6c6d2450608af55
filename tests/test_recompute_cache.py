"""
The checkpoint recompute cache's host logic (no GPU): inside a checkpointed
block call, an op whose backward reads only its inputs takes, on a recompute,
what the call's first forward computed (an alias), in call order; a memory
budget of 0.25 or less, or no block call, computes every time.
"""

from __future__ import annotations

import torch

import create_graph_b200 as cg
from create_graph_b200 import checkpoint
from create_graph_b200.compile_config import compile_context
from create_graph_b200.nn import _block_slot, _kept_across_recomputes


class Counter:
    def __init__(self):
        self.calls = 0

    def __call__(self, value):
        def compute():
            self.calls += 1
            return torch.full((3,), float(value))

        return compute


def _run_block(cache, counter, values):
    """One forward of a block: one kept op per value, in order."""
    cache.start()
    checkpoint._CACHES.append(cache)
    try:
        return [_kept_across_recomputes(counter(v), _block_slot()) for v in values]
    finally:
        checkpoint._CACHES.pop()


def test_recomputes_take_the_first_forward_in_call_order():
    cache, counter = checkpoint.RecomputeCache(), Counter()
    with compile_context(cg.CompileConfig(memory_budget=0.5)):
        first = _run_block(cache, counter, [1, 2, 3])
        again = _run_block(cache, counter, [7, 8, 9])  # a recompute: the kept values come back
    assert counter.calls == 3
    assert [float(t[0]) for t in again] == [1.0, 2.0, 3.0]
    for a, b in zip(first, again):
        assert a is not b  # each recompute gets a tensor of its own (an alias of the kept storage)
        assert torch.equal(a, b)


def test_budget_of_a_quarter_or_less_keeps_nothing():
    cache, counter = checkpoint.RecomputeCache(), Counter()
    with compile_context(cg.CompileConfig(memory_budget=0.25)):
        _run_block(cache, counter, [1, 2])
        again = _run_block(cache, counter, [5, 6])
    assert counter.calls == 4
    assert [float(t[0]) for t in again] == [5.0, 6.0]
    assert not cache.slots


def test_outside_a_block_call_every_call_computes():
    counter = Counter()
    with compile_context(cg.CompileConfig(memory_budget=1.0)):
        a = _kept_across_recomputes(counter(1), _block_slot())
        b = _kept_across_recomputes(counter(2), _block_slot())
    assert counter.calls == 2 and float(a[0]) == 1.0 and float(b[0]) == 2.0


def test_ops_with_several_outputs_keep_each_of_them():
    cache, calls = checkpoint.RecomputeCache(), []

    def pair():
        calls.append(1)
        return torch.full((2,), 1.0), torch.full((3,), 2.0)

    with compile_context(cg.CompileConfig(memory_budget=0.5)):
        for _ in range(3):
            cache.start()
            checkpoint._CACHES.append(cache)
            try:
                y, z = _kept_across_recomputes(pair, _block_slot())
            finally:
                checkpoint._CACHES.pop()
    assert len(calls) == 1
    assert torch.equal(y, torch.full((2,), 1.0)) and torch.equal(z, torch.full((3,), 2.0))
    kept_y, kept_z = cache.slots[0]
    assert y is not kept_y and y.data_ptr() == kept_y.data_ptr() and z.data_ptr() == kept_z.data_ptr()
