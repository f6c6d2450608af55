"""
The whole training step on the GPU against the oracle (oracle/step.py): the
reference's eager create_graph algorithm over plain torch ops in float64 on
the CPU, with the same parameters and inputs.

- neighbour lists: bit-exact (every index equal);
- energies, forces, loss and parameter gradients: the stated tf32 bound
  (GEMM operands rounded to 10 mantissa bits, fp32 accumulation): relative
  norm error below 1e-2 for forces and gradients, 5e-3 for energies;
- the region, the force pass and the parameter backward run on the fused
  kernels only (no eager fallback warning, device error word clear).
"""

from __future__ import annotations

import warnings

import numpy as np
import pytest
import torch

import create_graph_b200 as cg
from create_graph_b200 import mlip, native
from create_graph_b200.graph import build_graph, make_batch
from oracle import neighbors as onb
from oracle import step as ostep
from tests.twice import rel

pytestmark = pytest.mark.gpu

TINY = mlip.ModelSpec(n_species=5, hidden=32, heads=4, blocks=2, ffn=64, n_rbf=16, cutoff=5.0, k=12)


def tiny_inputs(seed=0, sizes=(20, 31, 25, 40, 3)):
    pos, species, sys_ptr = mlip.synthetic_systems(list(sizes), TINY.n_species, seed=seed)
    e_t, f_t = mlip.make_targets(len(sizes), pos.shape[0], seed=seed + 1)
    return pos, species, sys_ptr, e_t, f_t


def test_neighbor_list_bit_exact():
    for seed, sizes, k in [(0, [20, 31, 25, 40, 3], 12), (1, [200, 150, 64], 30), (2, [1, 2, 64], 32)]:
        pos, species, sys_ptr = mlip.synthetic_systems(sizes, 5, seed=seed)
        g = build_graph(pos.cuda(), sys_ptr.cuda(), len(sizes), max(sizes), 6.0, k)
        nbr, counts, rev_ptr, rev_idx = onb.neighbor_list(pos.numpy(), sys_ptr.numpy(), 6.0, k)
        assert np.array_equal(g.nbr.cpu().numpy(), nbr)
        assert np.array_equal(g.counts.cpu().numpy(), counts)
        assert np.array_equal(g.tokens.row_ptr.cpu().numpy(), rev_ptr)
        assert np.array_equal(g.tokens.perm.cpu().numpy()[: rev_idx.size], rev_idx)


def gpu_step(model, pos, species, sys_ptr, e_t, f_t, spec):
    batch = make_batch(pos.cuda(), species.cuda(), sys_ptr.cuda(), spec.n_species)
    for p in model.parameters():
        p.grad = None
    with warnings.catch_warnings():
        warnings.simplefilter("error")  # no eager-fallback warning
        out, grads = cg.create_graph(model, batch)
    forces = -grads["pos"]
    loss = mlip.loss_fn(out["energy"], forces, e_t.cuda(), f_t.cuda())
    loss.backward()
    torch.cuda.synchronize()
    return {
        "energy": out["energy"].detach().cpu(),
        "forces": forces.detach().cpu(),
        "loss": loss.detach().cpu(),
        "grads": {n: p.grad.detach().cpu() for n, p in model.named_parameters()},
    }


@pytest.mark.parametrize("config", [None, cg.CompileConfig(checkpoint=r"blocks\.\d+", memory_budget=0.5)])
def test_step_matches_oracle(config):
    torch.manual_seed(0)
    model = mlip.MLIP(TINY, config=config).cuda()
    pos, species, sys_ptr, e_t, f_t = tiny_inputs()
    got = gpu_step(model, pos, species, sys_ptr, e_t, f_t, TINY)
    assert native.device_error() == 0
    params = {n: p.detach().cpu().double() for n, p in model.named_parameters()}
    want = ostep.train_step(params, TINY, pos.double(), species, sys_ptr, e_t, f_t)
    assert rel(got["energy"], want["energy"]) < 5e-3
    assert rel(got["forces"], want["forces"]) < 1e-2
    assert rel(got["loss"], want["loss"]) < 1e-2
    flat_got = torch.cat([got["grads"][n].flatten().double() for n in params])
    flat_want = torch.cat([want["grads"][n].flatten() for n in params])
    assert rel(flat_got, flat_want) < 1e-2


def test_eval_mode_forces_first_order():
    torch.manual_seed(0)
    model = mlip.MLIP(TINY).cuda()
    pos, species, sys_ptr, _, _ = tiny_inputs(seed=3)
    batch = make_batch(pos.cuda(), species.cuda(), sys_ptr.cuda(), TINY.n_species)
    out, grads = cg.create_graph(model, batch, train=False)
    assert not out["energy"].requires_grad and not grads["pos"].requires_grad
    params = {n: p.detach().cpu().double() for n, p in model.named_parameters()}
    nbr, counts, _, _ = onb.neighbor_list(pos.numpy(), sys_ptr.numpy(), TINY.cutoff, TINY.k)
    x = pos.double().requires_grad_(True)
    e = ostep.energy(params, TINY, x, species, sys_ptr, torch.from_numpy(nbr), torch.from_numpy(counts))
    (g,) = torch.autograd.grad(e.sum(), x)
    assert rel(out["energy"].cpu(), e) < 5e-3
    assert rel(grads["pos"].cpu(), g) < 1e-2
