"""
The edge-attention MLIP of the benchmark workloads, built from the fused ops.

The reference ships no model (its headline model, AllScAIP, and fairchem are
not part of it), so this is the one frozen spec both sides use: the GPU path
here and the CPU oracle in oracle/step.py, which restates it in plain torch.

    species embedding                               h (n, C)
    per block (x n_blocks):
        x   = LN(h);  qkv = x Wqkv^T + b            (n, 3C)       tcgen05 GEMM
        tok = qkv[nbr]  (read in place by the attention kernels through the index)
        bias = rbf Wb^T + bb                        (n*k, H)      per-key RBF bias
                                                    (all blocks' Wb: one parameter)
        o   = attention among the k tokens of each atom, keys past counts masked
        m   = sum_s env[i, s] o[i, s]               (n, C)        envelope pooling
        h   = h + m Wo^T + bo
        h   = h + W2 silu(W1 LN(h) + b1) + b2                     FFN
    E_i = LN(h_i) w^T + b;  E_system = segment sum over its atoms

Edge geometry (rbf: n_rbf Gaussians on [0, cutoff]; env: cosine envelope)
comes from positions through the fused geometry op inside the region, so the
force pass and the parameter backward run on GPU kernels end to end.

Workloads (synthetic, seeded; densities and sizes of the benchmark configs):
``small_mlip`` (64 systems x 64 atoms, C 128, 4 heads, 4 blocks, 64 RBF, 10
species, k <= 32) and ``allscaip_85m`` (12 blocks, C 768, 12 heads, FFN 3072,
128 RBF, 50 species, k <= 30; systems of 20-200 atoms at 0.1 atoms/A^3).
"""

from __future__ import annotations

import dataclasses
import math

import torch
from torch import Tensor, nn

import create_graph_b200 as cg
from create_graph_b200 import nn as cgnn
from create_graph_b200.gemm import gemm_precision
from create_graph_b200.graph import AtomsBatch, build_graph, make_batch


@dataclasses.dataclass(frozen=True)
class ModelSpec:
    n_species: int
    hidden: int
    heads: int
    blocks: int
    ffn: int
    n_rbf: int
    cutoff: float
    k: int
    # tensor-core product precision of the edge attention: "fp32" (three-term
    # tf32 split) or "tf32" (one product)
    attn_precision: str = "fp32"
    # the same for the projections and FFNs (the tcgen05 GEMMs)
    gemm_precision: str = "tf32"

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def rbf_gamma(self) -> float:
        step = self.cutoff / (self.n_rbf - 1)
        return 0.5 / (step * step)


# the small MLIP is specified in fp32: every product at fp32 accuracy
SMALL_MLIP = ModelSpec(n_species=10, hidden=128, heads=4, blocks=4, ffn=512, n_rbf=64, cutoff=6.0, k=32,
                       attn_precision="fp32", gemm_precision="fp32")
# the 85M model runs TF32 GEMMs with fp32 accumulation, and tf32 attention products
ALLSCAIP_85M = ModelSpec(n_species=50, hidden=768, heads=12, blocks=12, ffn=3072, n_rbf=128, cutoff=6.0, k=30,
                         attn_precision="tf32", gemm_precision="tf32")
SPECS = {"small_mlip": SMALL_MLIP, "allscaip_85m": ALLSCAIP_85M}


class Block(nn.Module):
    def __init__(self, s: ModelSpec):
        super().__init__()
        c = s.hidden
        self.heads = s.heads
        self.scale = 1.0 / math.sqrt(s.head_dim)
        self.precision = s.attn_precision
        self.gemm_precision = s.gemm_precision
        self.norm1 = cgnn.LayerNorm(c)
        self.qkv = cgnn.Linear(c, 3 * c)
        # (the block's per-key attention bias from the RBF features is a row
        # block of EnergyNetwork.rbf_bias: one GEMM over the RBF tensor serves
        # every block)
        self.out = cgnn.Linear(c, c)
        self.norm2 = cgnn.LayerNorm(c)
        self.ffn1 = cgnn.Linear(c, s.ffn, silu=True)
        self.ffn2 = cgnn.Linear(s.ffn, c)

    def forward(self, h: Tensor, bias: Tensor, env: Tensor, graph: cgnn.NeighborGraph) -> Tensor:
        # the precision is entered here, not by the caller, so that a checkpoint
        # recompute of the block runs its GEMMs at the same precision
        with gemm_precision(self.gemm_precision):
            return self._forward(h, bias, env, graph)

    def _forward(self, h: Tensor, bias: Tensor, env: Tensor, graph: cgnn.NeighborGraph) -> Tensor:
        # attention among the atom's edge tokens, pooled by the envelope, one fused op
        # residual adds in the GEMM epilogues; each residual's two gradients meet
        # inside the LayerNorm backward kernel
        h, x = self.norm1.branch(h)
        m = cgnn.PooledTokenAttention.apply(self.qkv(x), bias, env, graph, self.heads, self.scale, self.precision)
        h, x = self.norm2.branch(self.out.residual(m, h))
        y, z = cgnn.LinearSiluFn.apply(x, self.ffn1.weight, self.ffn1.bias)
        return self.ffn2.silu_residual(y, z, h)


class EnergyNetwork(nn.Module):
    """Positions -> per-system energies (the cg.compile region)."""

    def __init__(self, s: ModelSpec):
        super().__init__()
        self.spec = s
        self.embed = nn.Parameter(torch.randn(s.n_species, s.hidden) * 0.5)
        self.blocks = nn.ModuleList(Block(s) for _ in range(s.blocks))
        # rows b*H .. (b+1)*H - 1: block b's per-key attention bias (bias_b =
        # rbf W_b^T + b_b); one parameter, so no per-step concatenation
        self.rbf_bias = cgnn.Linear(s.n_rbf, s.blocks * s.heads)
        self.norm = cgnn.LayerNorm(s.hidden)
        self.readout = cgnn.Linear(s.hidden, 1)

    def forward(self, pos: Tensor, graph: cgnn.NeighborGraph, species_csr: cgnn.Csr, system_csr: cgnn.Csr) -> Tensor:
        with gemm_precision(self.spec.gemm_precision):
            return self._forward(pos, graph, species_csr, system_csr)

    def _forward(self, pos: Tensor, graph: cgnn.NeighborGraph, species_csr: cgnn.Csr, system_csr: cgnn.Csr) -> Tensor:
        s = self.spec
        rbf, env = cgnn.EdgeGeometry.apply(pos, graph, s.n_rbf, s.cutoff, s.rbf_gamma)
        h = cgnn.Gather.apply(self.embed, species_csr)
        # every block's bias projection in one GEMM over the RBF tensor, each
        # block then reading its column block in place
        biases = cgnn.SplitCols.apply(self.rbf_bias(rbf), s.heads)
        for block, bias in zip(self.blocks, biases):
            h = block(h, bias, env, graph)
        e_atom = self.readout(self.norm(h))
        return cgnn.SegmentSum.apply(e_atom, system_csr).view(-1)


class MLIP(nn.Module):
    """The model a training step calls: neighbour graph (eager, integer work)
    then the energy region."""

    def __init__(self, s: ModelSpec, config: cg.CompileConfig | None = None):
        super().__init__()
        self.spec = s
        self.network = EnergyNetwork(s)
        self.region = cg.compile(self.network, config=config)

    def forward(self, data: AtomsBatch):
        s = self.spec
        graph = build_graph(data.pos, data.sys_ptr, data.n_systems, data.max_atoms, s.cutoff, s.k)
        return {"energy": self.region(data.pos, graph, data.species_csr, data.system_csr)}


# ---------------------------------------------------------------------------
# synthetic workloads
# ---------------------------------------------------------------------------


def synthetic_systems(sizes: list[int], n_species: int, density: float = 0.1, seed: int = 0):
    """Uniform positions in cubes of side (n/density)^(1/3), seeded; CPU tensors."""
    gen = torch.Generator().manual_seed(seed)
    pos, species = [], []
    for n in sizes:
        side = (n / density) ** (1.0 / 3.0)
        pos.append(torch.rand(n, 3, generator=gen) * side)
        species.append(torch.randint(0, n_species, (n,), generator=gen))
    sys_ptr = torch.zeros(len(sizes) + 1, dtype=torch.int32)
    sys_ptr[1:] = torch.cumsum(torch.tensor(sizes), 0)
    return torch.cat(pos), torch.cat(species).to(torch.int32), sys_ptr


def workload_sizes(name: str, seed: int = 0, atoms_target: int | None = None) -> list[int]:
    """System sizes of a named workload: small_mlip 64 x 64 atoms; allscaip_85m
    32 systems of U{20..200} atoms, or systems drawn until ~atoms_target."""
    if name == "small_mlip":
        return [64] * 64
    gen = torch.Generator().manual_seed(seed)
    if atoms_target is None:
        return [int(x) for x in torch.randint(20, 201, (32,), generator=gen)]
    sizes: list[int] = []
    while sum(sizes) < atoms_target:
        sizes.append(int(torch.randint(20, 201, (1,), generator=gen)))
    return sizes


def sharded_workload(name: str, rank: int, world: int, atoms_per_rank: int, seed: int = 1000):
    """One rank's share of a data-parallel workload: (sizes, pos, species,
    sys_ptr) on the CPU. Every rank draws the same global pool of systems
    (``workload_sizes(name, seed, world * atoms_per_rank)``, positions and
    species from ``seed``) and takes the systems that a least-loaded
    assignment in decreasing size gives it, kept in pool order. Per-rank atom
    counts then differ by less than one system's size; every kernel of the
    step works per atom or per padded neighbour slot (k per atom), so equal
    atoms are equal work. With world = 1 the share is the whole pool."""
    sizes = workload_sizes(name, seed=seed, atoms_target=world * atoms_per_rank)
    spec = SPECS[name]
    pos, species, sys_ptr = synthetic_systems(sizes, spec.n_species, seed=seed)
    load = [0] * world
    owner = [0] * len(sizes)
    for b in sorted(range(len(sizes)), key=lambda i: (-sizes[i], i)):
        r = min(range(world), key=lambda j: (load[j], j))
        owner[b] = r
        load[r] += sizes[b]
    mine = [b for b in range(len(sizes)) if owner[b] == rank]
    ptr = sys_ptr.tolist()
    atoms = torch.cat([torch.arange(ptr[b], ptr[b + 1]) for b in mine])
    my_sizes = [sizes[b] for b in mine]
    my_ptr = torch.zeros(len(mine) + 1, dtype=torch.int32)
    my_ptr[1:] = torch.cumsum(torch.tensor(my_sizes), 0)
    return my_sizes, pos[atoms], species[atoms], my_ptr


def make_targets(n_systems: int, n_atoms: int, seed: int = 1):
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(n_systems, generator=gen), torch.randn(n_atoms, 3, generator=gen)


def loss_fn(energy: Tensor, forces: Tensor, e_target: Tensor, f_target: Tensor) -> Tensor:
    """MSE on energies plus MSE on forces."""
    return (energy - e_target).square().mean() + (forces - f_target).square().mean()


def train_step(model: MLIP, batch: AtomsBatch, e_target: Tensor, f_target: Tensor) -> Tensor:
    """One conservative-force training step: energy, forces = -dE/dpos through
    create_graph, the loss (loss_fn, as one fused kernel) and the parameter
    backward through the force."""
    out, grads = cg.create_graph(model, batch, outputs="energy", inputs=("pos",))
    loss = cgnn.energy_force_loss(out["energy"], grads["pos"], e_target, f_target)
    loss.backward()
    return loss.detach()


def to_device_batch(pos, species, sys_ptr, n_species, device) -> AtomsBatch:
    return make_batch(pos.to(device), species.to(device), sys_ptr.to(device), n_species)


def reference_parameters(spec: ModelSpec) -> dict[str, Tensor]:
    """The model's freshly initialised parameters (same draws as MLIP(spec) under
    the same torch seed), on the CPU, without touching a GPU."""
    return {name: p.detach() for name, p in MLIP(spec).named_parameters()}
