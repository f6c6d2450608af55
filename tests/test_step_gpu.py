"""
The whole training step on the GPU against the oracle (oracle/step.py): the
reference's eager create_graph algorithm over plain torch ops in float64 on
the CPU, with the same parameters and inputs. The oracle itself is pinned to
the reference's own create_graph on this model (test_mlip_step_golden.py).

- neighbour lists: bit-exact (every index equal);
- fp32 precision (three-term tf32 products in GEMMs and attention): energies,
  forces, loss and parameter gradients within 1e-5 relative (norm-wise), on
  a tiny model and on the full small-MLIP workload (64 systems x 64 atoms);
- tf32 precision (one tf32 product, fp32 accumulation), the stated bound:
  relative error below 5e-3 for energies and 1e-2 for forces, loss and
  gradients, on a tiny model and on two blocks of the 85M model's shape
  (C 768, 12 heads of 64, k 30, FFN 3072, 128 RBF) with per-block checkpoint
  and memory budget 0.5;
- the memory budget lowers the step's peak memory (1.0 > 0.5 > 0.25) and
  leaves every result bit for bit the same;
- the region, the force pass and the parameter backward run on the fused
  kernels only (no eager fallback warning, device error word clear).
"""

from __future__ import annotations

import dataclasses
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
TINY_FP32 = dataclasses.replace(TINY, attn_precision="fp32", gemm_precision="fp32")
FP32_TOL = 1e-5
TF32_TOL = {"energy": 5e-3, "forces": 1e-2, "loss": 1e-2, "grads": 1e-2}
# two blocks of the 85M model's shape, at its precision
BLOCKS_85M = dataclasses.replace(mlip.ALLSCAIP_85M, blocks=2)


def tiny_inputs(seed=0, sizes=(20, 31, 25, 40, 3)):
    pos, species, sys_ptr = mlip.synthetic_systems(list(sizes), TINY.n_species, seed=seed)
    e_t, f_t = mlip.make_targets(len(sizes), pos.shape[0], seed=seed + 1)
    return pos, species, sys_ptr, e_t, f_t


def _lattice(nx, ny, nz, spacing=1.0):
    """Atoms on a cubic grid: many exactly equal distances (the (d2, j) tie rule)."""
    g = torch.stack(torch.meshgrid(torch.arange(nx), torch.arange(ny), torch.arange(nz), indexing="ij"), -1)
    return spacing * g.reshape(-1, 3).float()


def test_neighbor_list_bit_exact():
    """Systems of up to 256 atoms take the warp-per-atom selection and the
    counting-sort reverse; larger ones the per-thread kernels: both against
    the oracle, on random systems and on lattices full of equal distances."""
    cases = []
    for seed, sizes, k in [(0, [20, 31, 25, 40, 3], 12), (1, [200, 150, 64], 30), (2, [1, 2, 64], 32),
                           (3, [256, 30], 30), (4, [300, 40], 20), (5, [257], 64)]:
        pos, _, sys_ptr = mlip.synthetic_systems(sizes, 5, seed=seed)
        cases.append((pos, sys_ptr, sizes, k))
    for dims in ((4, 4, 4), (7, 7, 6)):
        pos = _lattice(*dims)
        cases.append((pos, torch.tensor([0, pos.shape[0]], dtype=torch.int32), [pos.shape[0]], 26))
    for pos, sys_ptr, sizes, k in cases:
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


def step_errors(spec, sizes, config=None, seed=0):
    """Relative errors of one GPU step against the oracle (float64, CPU)."""
    torch.manual_seed(seed)
    model = mlip.MLIP(spec, config=config).cuda()
    pos, species, sys_ptr = mlip.synthetic_systems(list(sizes), spec.n_species, seed=seed)
    e_t, f_t = mlip.make_targets(len(sizes), pos.shape[0], seed=seed + 1)
    got = gpu_step(model, pos, species, sys_ptr, e_t, f_t, spec)
    assert native.device_error() == 0
    params = {n: p.detach().cpu().double() for n, p in model.named_parameters()}
    want = ostep.train_step(params, spec, pos.double(), species, sys_ptr, e_t, f_t)
    flat_got = torch.cat([got["grads"][n].flatten().double() for n in params])
    flat_want = torch.cat([want["grads"][n].flatten() for n in params])
    return {
        "energy": rel(got["energy"], want["energy"]),
        "forces": rel(got["forces"], want["forces"]),
        "loss": rel(got["loss"], want["loss"]),
        "grads": rel(flat_got, flat_want),
    }


def within(errs: dict, tol) -> None:
    print({k: f"{v:.2e}" for k, v in errs.items()})
    for key, err in errs.items():
        bound = tol[key] if isinstance(tol, dict) else tol
        assert err < bound, f"{key}: relative error {err:.3e} >= {bound}"


@pytest.mark.parametrize("config", [None, cg.CompileConfig(checkpoint=r"blocks\.\d+", memory_budget=0.5)])
def test_step_matches_oracle(config):
    within(step_errors(TINY, (20, 31, 25, 40, 3), config), TF32_TOL)


@pytest.mark.parametrize("config", [None, cg.CompileConfig(checkpoint=r"blocks\.\d+", memory_budget=0.25)])
def test_step_fp32_matches_oracle(config):
    within(step_errors(TINY_FP32, (20, 31, 25, 40, 3), config), FP32_TOL)


def test_small_mlip_workload_fp32():
    """The small-MLIP workload in full: 64 systems x 64 atoms, fp32 spec."""
    assert mlip.SMALL_MLIP.gemm_precision == "fp32" and mlip.SMALL_MLIP.attn_precision == "fp32"
    within(step_errors(mlip.SMALL_MLIP, mlip.workload_sizes("small_mlip")), FP32_TOL)


def test_85m_shape_blocks_tf32():
    """Two blocks of the 85M model (tf32 GEMMs and attention), checkpointed
    per block with memory budget 0.5, as the 85M workload runs them."""
    config = cg.CompileConfig(checkpoint=r"blocks\.\d+", memory_budget=0.5)
    within(step_errors(BLOCKS_85M, (120, 57, 200, 33), config), TF32_TOL)


def _budget_run(spec, sizes, budget, checkpoint):
    torch.manual_seed(0)
    config = cg.CompileConfig(checkpoint=r"blocks\.\d+" if checkpoint else None, memory_budget=budget)
    model = mlip.MLIP(spec, config=config).cuda()
    pos, species, sys_ptr = mlip.synthetic_systems(list(sizes), spec.n_species, seed=0)
    e_t, f_t = mlip.make_targets(len(sizes), pos.shape[0], seed=1)
    torch.cuda.synchronize()
    torch.cuda.reset_peak_memory_stats()
    base = torch.cuda.memory_allocated()
    got = gpu_step(model, pos, species, sys_ptr, e_t, f_t, spec)
    peak = torch.cuda.max_memory_allocated() - base
    del model
    return peak, got


@pytest.mark.parametrize("checkpoint", [False, True])
def test_memory_budget_lowers_peak_memory(checkpoint):
    """Below 1 the force pass keeps no second-order FFN factor, at 0.5 no SiLU
    activation, at 0.25 no LayerNorm output: each is rebuilt bit for bit
    where a backward needs it, so the results stay identical. With
    checkpointed blocks, budgets above 0.25 also keep the force pass's input
    gradients for the parameter backward and defer the forward ops' share of
    the VJP's differentiation to the block's own backward (holding its
    cotangents); they set the peak, the same at 1 and 0.5. Without the
    deferral (0.25) the parameter gradients are summed in another order: equal
    to the tf32 products' rounding, not bit for bit."""
    sizes = mlip.workload_sizes("allscaip_85m", seed=0, atoms_target=3000)
    runs = {b: _budget_run(BLOCKS_85M, sizes, b, checkpoint) for b in (1.0, 0.5, 0.25)}
    peaks = {b: runs[b][0] for b in runs}
    print("peak MB:", {b: round(p / 2**20, 1) for b, p in peaks.items()})
    if checkpoint:
        assert peaks[1.0] >= peaks[0.5] > peaks[0.25]
    else:
        assert peaks[1.0] > peaks[0.5] > peaks[0.25]
    ref = runs[1.0][1]
    scale = torch.cat([g.flatten() for g in ref["grads"].values()]).norm()
    for b in (0.5, 0.25):
        got = runs[b][1]
        for key in ("energy", "forces", "loss"):
            assert torch.equal(got[key], ref[key]), (b, key)
        for name, g in ref["grads"].items():
            if b == 0.5 or not checkpoint:
                assert torch.equal(got["grads"][name], g), (b, name)
            else:
                # gradients that nearly cancel (the attention-bias bias sums
                # softmax gradients) are compared against the whole gradient's norm
                err = (got["grads"][name] - g).norm()
                assert err <= 1e-3 * max(g.norm(), 1e-2 * scale), (b, name, float(err), float(g.norm()))


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
