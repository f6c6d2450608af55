"""
The reference's own code, loaded from ``oracle/_ref`` (oracle/ref_build.py).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py): used by bench.py's CPU
baseline and reference legs, never by the product.
"""

from __future__ import annotations

import pathlib
import sys

REF_DIR = pathlib.Path(__file__).resolve().parent / "_ref"


def available() -> bool:
    return (REF_DIR / "create_graph" / "__init__.py").exists() and (REF_DIR / "kernels" / "edge_attn").exists()


def load():
    """(create_graph module, EdgeAttention op) of the reference, or None when
    oracle/_ref was not built."""
    if not available():
        return None
    if str(REF_DIR) not in sys.path:
        sys.path.insert(0, str(REF_DIR))
    import create_graph as ref_cg  # noqa: PLC0415
    from kernels.edge_attn import EdgeAttention  # noqa: PLC0415

    return ref_cg, EdgeAttention


def energy_model(ref_cg, params: dict, spec):
    """The reference's ``cg.compile`` region around oracle/step.py's energy
    function, as tests/golden/make_golden.py drives it; called as
    ``model({"pos", "species", "sys_ptr", "nbr", "counts"})``."""
    from torch import nn

    from oracle import step as ostep

    names = list(params)

    class Network(nn.Module):
        def __init__(self):
            super().__init__()
            self.weights = nn.ParameterList(nn.Parameter(params[n].detach().clone()) for n in names)

        def forward(self, x, species, sys_ptr, nbr, counts):
            return ostep.energy(dict(zip(names, self.weights)), spec, x, species, sys_ptr, nbr, counts)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.network = ref_cg.compile(Network())

        def forward(self, batch):
            return {"energy": self.network(batch["pos"], batch["species"], batch["sys_ptr"], batch["nbr"],
                                           batch["counts"])}

    return Model()


def mlp_model(ref_cg, hidden: int = 64, n_mol: int = 4, n_atom: int = 32):
    """The reference's examples/mlp.py-style model (3 -> hidden -> hidden -> 1,
    SiLU, per-molecule sum, centring outside the region) in plain torch."""
    import torch
    from torch import nn

    class Network(nn.Module):
        def __init__(self):
            super().__init__()
            self.layers = nn.Sequential(nn.Linear(3, hidden), nn.SiLU(), nn.Linear(hidden, hidden), nn.SiLU(),
                                        nn.Linear(hidden, 1))

        def forward(self, x, mol):
            return torch.zeros(n_mol, dtype=x.dtype).index_add(0, mol, self.layers(x)[:, 0])

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.network = ref_cg.compile(Network())

        def forward(self, batch):
            pos = batch["pos"].view(n_mol, n_atom, 3)
            centred = (pos - pos.mean(dim=1, keepdim=True)).view(n_mol * n_atom, 3)
            return {"energy": self.network(centred, batch["mol"])}

    return Model()
