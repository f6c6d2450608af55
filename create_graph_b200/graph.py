"""
Batches of atomic systems and their neighbour graphs on the GPU.

``AtomsBatch`` is the ``data`` object a training step hands to
``cg.create_graph``: ``pos`` is the differentiated input (swapped for a leaf
by create_graph), the rest are integer indices. ``build_graph`` runs the
bit-exact neighbour-list kernel (cg_neighbor_list) and returns the padded
(n_atoms, k) layout plus its reverse CSR, which every edge kernel uses.
"""

from __future__ import annotations

import dataclasses

import torch
from torch import Tensor

from create_graph_b200 import native
from create_graph_b200.nn import Csr, NeighborGraph


@dataclasses.dataclass
class AtomsBatch:
    pos: Tensor            # (n_atoms, 3) float32, atoms sorted by system
    species: Tensor        # (n_atoms,) int32
    sys_ptr: Tensor        # (n_systems + 1,) int32
    max_atoms: int         # largest system
    species_csr: Csr       # atoms grouped by species (embedding gather and its transpose)
    system_csr: Csr        # atoms grouped by system (energy readout)

    @property
    def n_atoms(self) -> int:
        return self.pos.shape[0]

    @property
    def n_systems(self) -> int:
        return self.sys_ptr.shape[0] - 1


def system_index(sys_ptr: Tensor, n_atoms: int) -> Tensor:
    counts = (sys_ptr[1:] - sys_ptr[:-1]).to(torch.int64)
    return torch.repeat_interleave(torch.arange(len(counts), device=sys_ptr.device), counts, output_size=n_atoms)


def make_batch(pos: Tensor, species: Tensor, sys_ptr: Tensor, n_species: int,
               max_atoms: int | None = None) -> AtomsBatch:
    """Index structures of a batch (on the tensors' device). ``max_atoms``
    bounds the largest system (the neighbour-list kernel's shared tile); when
    given, nothing is read back to the host, so the call can sit inside a
    captured CUDA graph."""
    n = pos.shape[0]
    sys_ptr = sys_ptr.to(torch.int32)
    counts = sys_ptr[1:] - sys_ptr[:-1]
    if max_atoms is None:
        max_atoms = int(counts.max()) if counts.numel() else 0
    species = species.to(torch.int32)
    sys_idx = system_index(sys_ptr, n).to(torch.int32)
    return AtomsBatch(
        pos=pos,
        species=species,
        sys_ptr=sys_ptr,
        max_atoms=max_atoms,
        species_csr=Csr.from_index(species, n_species),
        system_csr=Csr(sys_idx, sys_ptr, torch.arange(n, dtype=torch.int32, device=pos.device), len(counts)),
    )


def build_graph(pos: Tensor, sys_ptr: Tensor, n_systems: int, max_atoms: int, cutoff: float, k: int) -> NeighborGraph:
    """Neighbour graph of a batch: the k nearest within ``cutoff`` in each system."""
    native.require_cuda(pos, sys_ptr)
    pos = pos.detach().contiguous().float()
    n = pos.shape[0]
    dev = pos.device
    nbr = torch.empty(n, k, dtype=torch.int32, device=dev)
    counts = torch.empty(n, dtype=torch.int32, device=dev)
    rev_ptr = torch.empty(n + 1, dtype=torch.int32, device=dev)
    rev_idx = torch.empty(max(n * k, 1), dtype=torch.int32, device=dev)
    work = torch.empty(native.lib().cg_neighbor_list_workspace(n_systems), dtype=torch.int32, device=dev)
    native.call(
        "cg_neighbor_list", pos.data_ptr(), sys_ptr.data_ptr(), n_systems, n, max_atoms, float(cutoff), k,
        nbr.data_ptr(), counts.data_ptr(), rev_ptr.data_ptr(), rev_idx.data_ptr(), work.data_ptr(),
        native.stream_ptr(dev),
    )
    tokens = Csr(nbr.view(-1), rev_ptr, rev_idx, n)
    return NeighborGraph(nbr, counts, tokens, k)
