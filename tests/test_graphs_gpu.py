"""
Training steps captured in CUDA graphs (create_graph_b200.graphs) against the
same steps run eagerly.

- cg_csr_from_index builds the species map without host synchronisation and
  equals a stable sort's CSR exactly;
- a captured step (gradients zeroed, create_graph, loss.backward(), the fused
  AdamW update) replayed with new inputs copied into its buffers gives bit for
  bit the results of the eager step on those inputs, step after step (the
  AdamW step count lives on the device), for the per-atom MLP and for the
  small MLIP, whose neighbour lists and species map are rebuilt inside the
  graph from the positions of each replay.
"""

from __future__ import annotations

import pytest
import torch

from create_graph_b200 import mlip, mlp, native
from create_graph_b200.ddp import FlatGradients
from create_graph_b200.graph import make_batch
from create_graph_b200.graphs import CapturedStep
from create_graph_b200.nn import Csr
from create_graph_b200.optim import FusedAdamW

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n, rows", [(1, 1), (777, 10), (8280, 50), (5000, 256), (3000, 3), (20000, 257),
                                     (248400, 8280), (100, 5000), (0, 300)])
def test_csr_from_index_kernel_is_a_stable_sort(n, rows):
    """rows <= 256: the single-block kernel; more: count / scan / place / sort-rows."""
    gen = torch.Generator().manual_seed(n + rows)
    index = torch.randint(-1, rows, (n,), generator=gen, dtype=torch.int32)
    got = Csr.from_index(index.cuda(), rows)
    valid = index >= 0
    order = torch.argsort(torch.where(valid, index.long(), rows), stable=True)[: int(valid.sum())]
    counts = torch.bincount(index[valid].long(), minlength=rows)
    assert torch.equal(got.row_ptr.cpu().long(), torch.cat([torch.zeros(1, dtype=torch.long), counts.cumsum(0)]))
    nnz = int(valid.sum())
    assert torch.equal(got.perm.cpu()[:nnz].long(), order)
    assert (got.perm.cpu()[nnz:n] == -1).all()


def _restart(model, grads, opt, params0):
    """Put the parameters, moments and step count back to the start, in place."""
    with torch.no_grad():
        for p, p0 in zip(grads.params, params0):
            p.copy_(p0)
        opt.exp_avg.zero_()
        opt.exp_avg_sq.zero_()
        opt.state.zero_()
        grads.flat.zero_()


def _trainer(model):
    grads = FlatGradients(model.parameters(), None)
    opt = FusedAdamW(grads, lr=1e-3)
    return grads, opt


def test_captured_mlp_step_replays_like_eager():
    spec = mlp.MLPSpec()
    torch.manual_seed(0)
    eager_model = mlp.MLPModel(spec).cuda()
    torch.manual_seed(0)
    graph_model = mlp.MLPModel(spec).cuda()
    eg, eo = _trainer(eager_model)
    gg, go = _trainer(graph_model)
    params0 = [p.detach().clone() for p in gg.params]
    pos, e_t, f_t = (t.cuda() for t in mlp.synthetic_batch(spec, seed=0))
    molecules = mlp.molecules_csr(spec, pos.device)
    static = {"pos": pos.clone(), "molecules": molecules}

    def graph_step():
        gg.zero()
        loss = mlp.train_step(graph_model, static, e_t, f_t)
        go.step()
        return loss

    captured = CapturedStep(graph_step)
    assert captured.kernels > 10
    _restart(graph_model, gg, go, params0)
    for s in range(3):
        new_pos = pos + 0.05 * s
        static["pos"].copy_(new_pos)
        loss_g = captured().clone()
        eg.zero()
        loss_e = mlp.train_step(eager_model, {"pos": new_pos, "molecules": molecules}, e_t, f_t)
        eo.step()
        torch.cuda.synchronize()
        assert torch.equal(loss_g, loss_e), s
        for a, b in zip(gg.params, eg.params):
            assert torch.equal(a, b), s
    assert native.device_error() == 0


def test_captured_small_mlip_step_replays_like_eager():
    spec = mlip.SMALL_MLIP
    sizes = [64] * 6
    pos, species, sys_ptr = mlip.synthetic_systems(sizes, spec.n_species, seed=3)
    e_t, f_t = (t.cuda() for t in mlip.make_targets(len(sizes), pos.shape[0], seed=4))
    pos, species, sys_ptr = pos.cuda(), species.cuda(), sys_ptr.cuda()
    torch.manual_seed(0)
    eager_model = mlip.MLIP(spec).cuda()
    torch.manual_seed(0)
    graph_model = mlip.MLIP(spec).cuda()
    eg, eo = _trainer(eager_model)
    gg, go = _trainer(graph_model)
    params0 = [p.detach().clone() for p in gg.params]
    static_pos = pos.clone()

    def graph_step():
        gg.zero()
        batch = make_batch(static_pos, species, sys_ptr, spec.n_species, max_atoms=max(sizes))
        loss = mlip.train_step(graph_model, batch, e_t, f_t)
        go.step()
        return loss

    captured = CapturedStep(graph_step)
    _restart(graph_model, gg, go, params0)
    for s in range(3):
        new_pos = pos + 0.02 * s * torch.sin(pos)
        static_pos.copy_(new_pos)
        loss_g = captured().clone()
        eg.zero()
        loss_e = mlip.train_step(eager_model, make_batch(new_pos, species, sys_ptr, spec.n_species), e_t, f_t)
        eo.step()
        torch.cuda.synchronize()
        assert torch.equal(loss_g, loss_e), s
        for a, b in zip(gg.params, eg.params):
            assert torch.equal(a, b), s
    assert native.device_error() == 0
