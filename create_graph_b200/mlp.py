"""
The per-atom MLP workload of the reference's examples (examples/mlp.py:18-63
there: energy from positions through Linear + SiLU layers, centring outside
the region, loss on energy and forces), on the fused ops.

    molecules of n_atom atoms, pos ~ N(0, 1.5 A), centred per molecule
    (eager, outside the region, as the reference centres)
    region:  h = silu(x W1^T + b1); h = silu(h W2^T + b2); e = h W3^T + b3
             E_mol = segment sum of e over the molecule's atoms
    loss:    MSE(E, targets) + MSE(F = -dE/dpos, targets)

Widths 3 -> 64 -> 64 -> 1 by default; the SiLU is fused into each GEMM's
epilogue and the per-molecule sum is the deterministic CSR segment sum.
"""

from __future__ import annotations

import dataclasses

import torch
from torch import Tensor, nn

import create_graph_b200 as cg
from create_graph_b200 import nn as cgnn


@dataclasses.dataclass(frozen=True)
class MLPSpec:
    n_mol: int = 4
    n_atom: int = 32
    hidden: int = 64


class AtomEnergyMLP(nn.Module):
    """Per-atom energies summed per molecule: the cg.compile region."""

    def __init__(self, hidden: int = 64):
        super().__init__()
        self.l1 = cgnn.Linear(3, hidden, silu=True)
        self.l2 = cgnn.Linear(hidden, hidden, silu=True)
        self.l3 = cgnn.Linear(hidden, 1)

    def forward(self, x: Tensor, molecules: cgnn.Csr) -> Tensor:
        e_atom = self.l3(self.l2(self.l1(x)))
        return cgnn.SegmentSum.apply(e_atom, molecules).view(-1)


class MLPModel(nn.Module):
    """Centring (eager) then the region, as in the reference's example."""

    def __init__(self, spec: MLPSpec = MLPSpec(), config: cg.CompileConfig | None = None):
        super().__init__()
        self.spec = spec
        self.network = cg.compile(AtomEnergyMLP(spec.hidden), config=config)

    def forward(self, batch: dict) -> dict:
        s = self.spec
        pos = batch["pos"].view(s.n_mol, s.n_atom, 3)
        centred = (pos - pos.mean(dim=1, keepdim=True)).view(s.n_mol * s.n_atom, 3)
        return {"energy": self.network(centred, batch["molecules"])}


def molecules_csr(spec: MLPSpec, device) -> cgnn.Csr:
    """Atom a belongs to molecule a // n_atom."""
    index = torch.arange(spec.n_mol * spec.n_atom, device=device) // spec.n_atom
    return cgnn.Csr.from_index(index, spec.n_mol)


def synthetic_batch(spec: MLPSpec = MLPSpec(), seed: int = 0):
    """(pos, e_target, f_target) on the CPU: pos ~ N(0, 1.5 A), targets ~ N(0, 1)."""
    gen = torch.Generator().manual_seed(seed)
    pos = 1.5 * torch.randn(spec.n_mol * spec.n_atom, 3, generator=gen)
    e_target = torch.randn(spec.n_mol, generator=gen)
    f_target = torch.randn(spec.n_mol * spec.n_atom, 3, generator=gen)
    return pos, e_target, f_target


def train_step(model: MLPModel, batch: dict, e_target: Tensor, f_target: Tensor) -> Tensor:
    """Energy and forces through create_graph, MSE on both (one fused kernel),
    loss.backward()."""
    out, grads = cg.create_graph(model, batch)
    loss = cgnn.energy_force_loss(out["energy"], grads["pos"], e_target, f_target)
    loss.backward()
    return loss.detach()
