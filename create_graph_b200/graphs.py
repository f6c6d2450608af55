"""
CUDA-graph capture of a training step whose shapes do not change.

A small step (the per-atom MLP, the small MLIP) launches a few hundred
kernels of microseconds each; the Python around them (create_graph's region
logic, autograd, the ctypes calls) then takes longer than the GPU work.
``CapturedStep(fn)`` runs ``fn`` a few times on a side stream (warm-up: lazy
set-up, allocator pools), captures one call into a CUDA graph and replays it:
every kernel of the step runs again on every replay, on the same buffers, with
no Python in between. ``fn`` must read its inputs from tensors that stay put
(copy new data into them between replays), take the same autograd path each
time, and read nothing back to the host: the package's ops and
``graph.make_batch(..., max_atoms=...)`` qualify, and ``optim.FusedAdamW``
keeps its step count on the device for this. Collectives are left outside:
capture the backward and the optimizer update as two graphs and average the
gradients between them (``ddp.FlatGradients(..., overlap=False)``).
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from create_graph_b200 import native


class CapturedStep:
    """``step()`` replays the captured call of ``fn`` and returns the tensors it
    returned at capture, which every replay overwrites in place."""

    def __init__(self, fn: Callable, warmup: int = 3):
        if not torch.cuda.is_available():
            raise native.NativeError("CapturedStep needs a CUDA device")
        current = torch.cuda.current_stream()
        side = torch.cuda.Stream()
        side.wait_stream(current)
        with torch.cuda.stream(side):
            for _ in range(warmup):
                fn()
        current.wait_stream(side)
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        before = native.launch_count()
        with torch.cuda.graph(self.graph):
            self.output = fn()
        # kernels of the library captured into the graph (each replay runs them all)
        self.kernels = native.launch_count() - before

    def __call__(self):
        self.graph.replay()
        return self.output
