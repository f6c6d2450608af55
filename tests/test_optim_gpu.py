"""
The fused AdamW step (cg_adamw_step through create_graph_b200.optim) against
torch.optim.AdamW on the same parameters and gradients, three steps, with
weight decay, a parameter count that is not a multiple of four (the scalar
tail) and parameters that stay views into the flat buffer. float32 elementwise
arithmetic in a different order from torch's: 1e-6 relative.
"""

from __future__ import annotations

import pytest
import torch

from create_graph_b200.ddp import FlatGradients
from create_graph_b200.optim import FusedAdamW

pytestmark = pytest.mark.gpu


def test_fused_adamw_matches_torch():
    gen = torch.Generator().manual_seed(0)
    shapes = [(37, 11), (5,), (64, 3), (1,)]
    init = [torch.randn(*s, generator=gen) for s in shapes]
    mine = [torch.nn.Parameter(t.clone().cuda()) for t in init]
    ref = [torch.nn.Parameter(t.clone().cuda()) for t in init]
    grads = FlatGradients(mine, None)
    opt = FusedAdamW(grads, lr=1e-2, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.1)
    ref_opt = torch.optim.AdamW(ref, lr=1e-2, betas=(0.9, 0.99), eps=1e-8, weight_decay=0.1, foreach=False)
    for step in range(3):
        g = [torch.randn(*s, generator=gen).cuda() for s in shapes]
        grads.zero()
        for p, gi in zip(mine, g):
            p.grad.copy_(gi)
        for p, gi in zip(ref, g):
            p.grad = gi.clone()
        opt.step()
        ref_opt.step()
        torch.cuda.synchronize()
        for a, b in zip(mine, ref):
            err = ((a - b).norm() / b.norm()).item()
            assert err < 1e-6, (step, err)
    # the parameters are views into the optimizer's flat buffer
    assert all(p.data_ptr() >= opt.flat.data_ptr() for p in mine)
