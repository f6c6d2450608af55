"""
Data-parallel gradient averaging for the training step, overlapped with the
parameter backward.

The reference's only parallelism is torch DDP around the model, with a
bucketed allreduce inside ``loss.backward()`` (tests/test_ddp.py:62-106
there). Here every parameter's ``.grad`` is a view into one flat buffer (the
parameters' dtype, fp32 for the model), so ``loss.backward()`` accumulates in
place, and the buffer is cut into buckets of whole parameters, in reverse
registration order (the last blocks' parameters finish first in a
checkpointed force-training backward). A post-accumulate-grad hook counts the
parameters of each bucket as the engine finalises their gradients (each
parameter's AccumulateGrad runs once per backward, after every contribution
to it has been summed); a complete bucket is averaged with an asynchronous
NCCL all-reduce that runs beside the rest of the backward. Buckets are
launched strictly in index order, so every rank issues the same collectives
in the same order whatever the engine's order of completion. ``allreduce()``
launches the buckets no hook completed (parameters that got no gradient this
step) and makes the current stream wait for all of them.

Systems are sharded across ranks, so this is the only exchange of the step.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

DEFAULT_BUCKET_BYTES = 64 << 20
# each parameter's slice of the flat buffers starts on a 256-byte boundary, so
# that views of it (weights read by TMA, gradients) keep an allocation's alignment
ALIGN_BYTES = 256


class FlatGradients:
    def __init__(self, params, world: int | None, bucket_bytes: int = DEFAULT_BUCKET_BYTES,
                 overlap: bool = True):
        self.params = [p for p in params if p.requires_grad]
        device, dtype = self.params[0].device, self.params[0].dtype
        if any(p.dtype != dtype for p in self.params):
            raise ValueError("FlatGradients: all parameters must share one dtype")
        align = max(1, ALIGN_BYTES // self.params[0].element_size())
        offsets = []
        offset = 0
        for p in self.params:
            offsets.append((offset, p.numel()))
            offset += -(-p.numel() // align) * align
        total = offset
        self.flat = torch.zeros(total, dtype=dtype, device=device)
        for p, (offset, n) in zip(self.params, offsets):
            p.grad = self.flat[offset : offset + n].view_as(p)
        self.offsets = offsets  # (start, numel) of each parameter; the gaps stay zero
        self.world = world
        # buckets of whole parameters from the end of the buffer backwards
        per = max(1, bucket_bytes // self.flat.element_size())
        self.buckets: list[tuple[int, int]] = []  # (start, stop) in the flat buffer
        self.bucket_of: dict[int, int] = {}
        self.bucket_size: list[int] = []
        stop, count = total, 0
        for i in reversed(range(len(self.params))):
            start, n = offsets[i]
            self.bucket_of[id(self.params[i])] = len(self.buckets)
            count += 1
            if stop - start >= per or i == 0:
                self.buckets.append((start, stop))
                self.bucket_size.append(count)
                stop, count = start, 0
        self.overlap = overlap and world is not None and world > 1
        self._pending: list[int] = []
        self._next = 0
        self._works: list = []
        self._hooks = []
        if self.overlap:
            for p in self.params:
                self._hooks.append(p.register_post_accumulate_grad_hook(self._ready))
        self._reset()

    def _reset(self) -> None:
        self._pending = list(self.bucket_size)
        self._next = 0
        self._works = []

    def _launch(self, b: int) -> None:
        start, stop = self.buckets[b]
        self._works.append(dist.all_reduce(self.flat[start:stop], op=dist.ReduceOp.AVG, async_op=True))

    def _ready(self, p: torch.Tensor) -> None:
        b = self.bucket_of[id(p)]
        self._pending[b] -= 1
        while self._next < len(self.buckets) and self._pending[self._next] == 0:
            self._launch(self._next)
            self._next += 1

    def zero(self) -> None:
        if self._works:
            raise RuntimeError("FlatGradients: zero() before allreduce() finished the previous step")
        self.flat.zero_()
        self._reset()
        for p in self.params:  # a step may have replaced a view; restore it
            if p.grad is None or p.grad.data_ptr() < self.flat.data_ptr():
                raise RuntimeError("FlatGradients: a parameter's .grad was detached from the flat buffer")

    def allreduce(self) -> None:
        """Average the gradients over the ranks (no-op on one rank): finish the
        buckets the backward launched, launch the rest, wait for all."""
        if self.world is None or self.world <= 1:
            return
        if not self.overlap:
            dist.all_reduce(self.flat, op=dist.ReduceOp.AVG)
            return
        while self._next < len(self.buckets):
            self._launch(self._next)
            self._next += 1
        for work in self._works:
            work.wait()
        self._reset()

    @property
    def launched_in_backward(self) -> int:
        """Buckets launched by the hooks so far this step (before allreduce())."""
        return self._next

    def remove_hooks(self) -> None:
        for h in self._hooks:
            h.remove()
        self._hooks = []
