"""
Data-parallel gradient averaging for the training step.

The reference's only parallelism is torch DDP around the model, with one
bucketed allreduce inside ``loss.backward()`` (tests/test_ddp.py:62-106
there). Here every parameter's ``.grad`` is a view into one flat buffer (the
parameters' dtype, fp32 for the model),
so ``loss.backward()`` accumulates in place and one NCCL all-reduce (average)
of the buffer follows: over NVLink / NVSwitch that is one collective of all
gradients per step. Systems are sharded across ranks, so this is the only
exchange of the step.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


class FlatGradients:
    def __init__(self, params, world: int | None):
        self.params = [p for p in params if p.requires_grad]
        device, dtype = self.params[0].device, self.params[0].dtype
        if any(p.dtype != dtype for p in self.params):
            raise ValueError("FlatGradients: all parameters must share one dtype")
        total = sum(p.numel() for p in self.params)
        self.flat = torch.zeros(total, dtype=dtype, device=device)
        offset = 0
        for p in self.params:
            n = p.numel()
            p.grad = self.flat[offset : offset + n].view_as(p)
            offset += n
        self.world = world

    def zero(self) -> None:
        self.flat.zero_()
        for p in self.params:  # a step may have replaced a view; restore it
            if p.grad is None or p.grad.data_ptr() < self.flat.data_ptr():
                raise RuntimeError("FlatGradients: a parameter's .grad was detached from the flat buffer")

    def allreduce(self) -> None:
        """Average the gradients over the ranks (no-op on one rank)."""
        if self.world is None or self.world <= 1:
            return
        dist.all_reduce(self.flat, op=dist.ReduceOp.AVG)
