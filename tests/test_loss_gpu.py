"""
The fused training loss (nn.energy_force_loss: MSE on energies plus MSE on
forces F = -dE/dpos, one reduction kernel and one gradient kernel) against
the same loss in float64 torch: value and gradients w.r.t. the energies and
dE/dpos, to fp32 rounding; and bitwise repeatability of the value.
"""

from __future__ import annotations

import pytest
import torch

from create_graph_b200 import native
from create_graph_b200.nn import energy_force_loss

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n_sys, n_atoms", [(1, 1), (77, 8280), (64, 4096), (3, 20000)])
def test_fused_loss_matches_torch(n_sys, n_atoms):
    gen = torch.Generator().manual_seed(n_atoms)
    e, et = torch.randn(n_sys, generator=gen) * 20, torch.randn(n_sys, generator=gen)
    g, ft = torch.randn(n_atoms, 3, generator=gen), torch.randn(n_atoms, 3, generator=gen)
    e_d, g_d = e.cuda().requires_grad_(True), g.cuda().requires_grad_(True)
    loss = energy_force_loss(e_d, g_d, et.cuda(), ft.cuda())
    loss.backward(torch.tensor(0.5, device="cuda"))
    e64, g64 = e.double().requires_grad_(True), g.double().requires_grad_(True)
    want = (e64 - et.double()).square().mean() + (-g64 - ft.double()).square().mean()
    (0.5 * want).backward()
    assert abs(loss.item() - want.item()) <= 2e-6 * abs(want.item())
    assert torch.allclose(e_d.grad.cpu().double(), e64.grad, rtol=1e-5, atol=1e-7)
    assert torch.allclose(g_d.grad.cpu().double(), g64.grad, rtol=1e-5, atol=1e-9)
    again = energy_force_loss(e_d.detach(), g_d.detach(), et.cuda(), ft.cuda())
    assert torch.equal(again, loss.detach())
    assert native.device_error() == 0
