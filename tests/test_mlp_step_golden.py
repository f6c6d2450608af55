"""
Whole-step parity with the reference's own create_graph on the per-atom MLP
of its examples (4 molecules x 32 atoms, 3 -> 64 -> 64 -> 1 with SiLU,
float64): energy, forces F = -dE/dpos, the loss MSE(E) + MSE(F) and every
parameter gradient of loss.backward() through the force term. The fixture
``golden/mlp_step.npz`` holds the reference's outputs of its compiled
(create_graph default) and exact (eager double-backward) paths, written by
``golden/make_golden.py``.

The host mechanism runs on the CPU here in float64 (region forward, in-region
gradient, parameter backward); the same step on the GPU through the native
GEMM kernels (tf32 tensor cores, float32) is checked at the tf32 bound.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch
from torch import nn

import create_graph_b200 as cg

GOLDEN = np.load(Path(__file__).parent / "golden" / "mlp_step.npz")
N_MOL, N_ATOM = 4, 32


class Network(nn.Module):
    def __init__(self):
        super().__init__()
        self.l1, self.l2, self.l3 = nn.Linear(3, 64), nn.Linear(64, 64), nn.Linear(64, 1)

    def forward(self, x, mol):
        h = nn.functional.silu(self.l1(x))
        h = nn.functional.silu(self.l2(h))
        return torch.zeros(N_MOL, dtype=x.dtype, device=x.device).index_add(0, mol, self.l3(h)[:, 0])


class Model(nn.Module):
    def __init__(self, network):
        super().__init__()
        self.network = network

    def forward(self, batch):
        pos = batch["pos"].view(N_MOL, N_ATOM, 3)
        centred = (pos - pos.mean(dim=1, keepdim=True)).view(N_MOL * N_ATOM, 3)
        return {"energy": self.network(centred, batch["mol"])}


def _network(dtype, device) -> Network:
    net = Network()
    with torch.no_grad():
        for name, p in net.named_parameters():
            p.copy_(torch.from_numpy(GOLDEN[f"param.{name}"]))
    return net.to(dtype=dtype, device=device)


def _step(model, dtype, device, exact=False):
    pos = torch.from_numpy(GOLDEN["pos"]).to(dtype=dtype, device=device)
    mol = (torch.arange(N_MOL * N_ATOM) // N_ATOM).to(device)
    e_t = torch.from_numpy(GOLDEN["e_target"]).to(dtype=dtype, device=device)
    f_t = torch.from_numpy(GOLDEN["f_target"]).to(dtype=dtype, device=device)
    model.zero_grad()
    out, grads = cg.create_graph(model, {"pos": pos, "mol": mol}, exact=exact)
    forces = -grads["pos"]
    loss = (out["energy"] - e_t).square().mean() + (forces - f_t).square().mean()
    loss.backward()
    res = {"energy": out["energy"], "forces": forces, "loss": loss}
    for name, p in model.network.named_parameters():
        res[f"grad.{name.removeprefix('module.')}"] = p.grad
    return {k: v.detach().cpu().double().numpy() for k, v in res.items()}


def _assert_matches(res: dict, label: str, rtol: float, atol: float) -> None:
    for key, got in res.items():
        want = GOLDEN[f"{label}.{key}"]
        np.testing.assert_allclose(got, want, rtol=rtol, atol=atol, err_msg=f"{label}.{key}")


def test_reference_paths_agree():
    for key in ("energy", "forces", "loss", "grad.l1.weight", "grad.l2.weight"):
        np.testing.assert_allclose(GOLDEN[f"compiled.{key}"], GOLDEN[f"exact.{key}"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("exact", [False, True])
def test_region_step_matches_reference_cpu_f64(exact):
    cg.reset()
    model = Model(cg.compile(_network(torch.float64, "cpu")))
    res = _step(model, torch.float64, "cpu", exact=exact)
    _assert_matches(res, "exact" if exact else "compiled", rtol=1e-9, atol=1e-11)


def _native_step(precision: str) -> dict:
    """The package's config-1 model (create_graph_b200.mlp: fused Linear + SiLU
    GEMMs, CSR segment sum) with the fixture's parameters, one step on cuda:0."""
    from create_graph_b200 import mlp
    from create_graph_b200.gemm import gemm_precision

    cg.reset()
    spec = mlp.MLPSpec(n_mol=N_MOL, n_atom=N_ATOM, hidden=64)
    model = mlp.MLPModel(spec).cuda()
    with torch.no_grad():
        for name, p in model.network.named_parameters():
            p.copy_(torch.from_numpy(GOLDEN[f"param.{name.removeprefix('module.')}"]))
    pos = torch.from_numpy(GOLDEN["pos"]).float().cuda()
    e_t = torch.from_numpy(GOLDEN["e_target"]).float().cuda()
    f_t = torch.from_numpy(GOLDEN["f_target"]).float().cuda()
    batch = {"pos": pos, "molecules": mlp.molecules_csr(spec, pos.device)}
    model.zero_grad()
    with gemm_precision(precision):
        out, grads = cg.create_graph(model, batch)
        forces = -grads["pos"]
        loss = (out["energy"] - e_t).square().mean() + (forces - f_t).square().mean()
        loss.backward()
    res = {"energy": out["energy"], "forces": forces, "loss": loss}
    for name, p in model.network.named_parameters():
        res[f"grad.{name.removeprefix('module.')}"] = p.grad
    return {k: v.detach().cpu().double().numpy() for k, v in res.items()}


@pytest.mark.gpu
@pytest.mark.parametrize("precision, tol", [("tf32", 2e-2), ("fp32", 1e-5)])
def test_native_step_matches_reference_gpu(precision, tol):
    """The same step on the native kernels, float32 data: tf32 products
    (relative error ~1e-3 per product, ~1e-2 after the double-backward chain)
    or fp32 precision (three-term split, within 1e-5), against the
    reference's float64 outputs (max error over each tensor's largest entry)."""
    res = _native_step(precision)
    for key, got in res.items():
        want = GOLDEN[f"compiled.{key}"]
        err = np.abs(got - want).max() / max(np.abs(want).max(), 1e-30)
        assert err < tol, (key, err)
