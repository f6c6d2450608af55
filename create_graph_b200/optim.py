"""
The optimizer update of the training step: AdamW over the flat buffers.

``FusedAdamW(flat_grads)`` moves the parameters of a ``ddp.FlatGradients``
into one flat fp32 buffer laid out like its gradient buffer (each parameter's
``.data`` becomes a view into it, on a 256-byte boundary like a separate
allocation, so weights keep their TMA-friendly alignment), keeps the two
moment buffers beside it,
and applies torch.optim.AdamW's update (amsgrad off) to all of them with one
kernel launch per step (``cg_adamw_step``). The reference ships no optimizer:
its training loops use torch's; this is the fused equivalent for the step
that follows ``loss.backward()`` and the gradient all-reduce.
"""

from __future__ import annotations

import torch

from create_graph_b200 import native
from create_graph_b200.ddp import FlatGradients


class FusedAdamW:
    def __init__(self, grads: FlatGradients, lr: float = 1e-3, betas: tuple[float, float] = (0.9, 0.999),
                 eps: float = 1e-8, weight_decay: float = 1e-2):
        if grads.flat.dtype != torch.float32:
            raise ValueError("FusedAdamW: parameters must be float32")
        if not 0.0 <= betas[0] < 1.0 or not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"FusedAdamW: betas {betas} outside [0, 1)")
        self.grads = grads
        # the gradient buffer's layout (256-byte aligned slices, zero gaps that
        # the update keeps at zero)
        self.flat = torch.zeros_like(grads.flat)
        with torch.no_grad():
            for p, (offset, n) in zip(grads.params, grads.offsets):
                view = self.flat[offset : offset + n].view_as(p)
                view.copy_(p)
                p.data = view
        self.exp_avg = torch.zeros_like(self.flat)
        self.exp_avg_sq = torch.zeros_like(self.flat)
        self.lr, self.betas, self.eps, self.weight_decay = lr, betas, eps, weight_decay
        # step count and bias corrections on the device (cg_adamw_step_counted),
        # so that a CUDA graph holding the update replays the next step each time
        self.state = torch.zeros(2, dtype=torch.int64, device=self.flat.device)

    @property
    def steps(self) -> int:
        """Steps taken so far (reads the device counter: synchronises)."""
        return int(self.state[0])

    @torch.no_grad()
    def step(self) -> None:
        native.call("cg_adamw_step_counted", self.flat.data_ptr(), self.grads.flat.data_ptr(),
                    self.exp_avg.data_ptr(), self.exp_avg_sq.data_ptr(), self.flat.numel(), self.lr, self.betas[0],
                    self.betas[1], self.eps, self.weight_decay, self.state.data_ptr(),
                    native.stream_ptr(self.flat.device))
