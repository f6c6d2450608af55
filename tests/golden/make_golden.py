"""
Generate the golden vectors under tests/golden/ by running the reference itself.

    python tests/golden/make_golden.py --reference <reference checkout>

Imports the reference package read-only from its source tree (``src/`` and the
repository root for ``kernels.edge_attn``) and records, for seeded inputs, what
its own ``cg_kernels::edge_attn`` operators (forward1 / backward1 / backward2,
kernels/edge_attn/ops.py) and its ``create_graph`` step return: on the
examples/mlp.py-style model, and on the small edge-attention MLIP whose
energy function is oracle/step.py's (so the fixture pins the oracle's step
against the reference's own create_graph). The fixtures are small ``.npz``
files; the GPU box never needs the reference. Re-running this script
reproduces them bit for bit.
"""

from __future__ import annotations

import argparse
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent


def import_reference(root: str):
    sys.path[:0] = [f"{root}/src", root]
    import create_graph as ref_cg  # noqa: PLC0415
    from kernels.edge_attn import EdgeAttention  # noqa: PLC0415

    return ref_cg, EdgeAttention


def attn_case(op, q, k, v, bias, scale, gen):
    """Inputs, cotangents and the reference op's three outputs."""
    out, lse = op.op(q, k, v, bias, scale)
    grad_out = torch.randn(out.shape, generator=gen, dtype=q.dtype)
    b1 = op.backward1_op(q, k, v, bias, lse, grad_out, scale)
    hq, hk, hv = (torch.randn(q.shape, generator=gen, dtype=q.dtype) for _ in range(3))
    hb = torch.randn(bias.shape, generator=gen, dtype=q.dtype)
    hb = torch.where(torch.isfinite(bias), hb, torch.zeros_like(hb))
    b2 = op.backward2_op(q, k, v, bias, lse, grad_out, scale, hq, hk, hv, hb)
    arrays = dict(
        q=q, k=k, v=v, bias=bias, scale=torch.tensor(scale, dtype=torch.float64),
        out=out, lse=lse, grad_out=grad_out,
        b1_dq=b1[0], b1_dk=b1[1], b1_dv=b1[2], b1_dbias=b1[3],
        hq=hq, hk=hk, hv=hv, hb=hb,
        b2_dq=b2[0], b2_dk=b2[1], b2_dv=b2[2], b2_dbias=b2[3], b2_dgrad_out=b2[4],
    )
    return {name: t.detach().numpy() for name, t in arrays.items()}


def edge_attn_fixtures(op) -> dict[str, dict]:
    cases = {}
    # the reference test's own shapes (tests/test_custom_ops.py:24-39): fp64,
    # q/k/v (2,3,5,4), bias (2,1,1,5) broadcast, scale 0.5, with and without -inf keys
    for masked in (False, True):
        gen = torch.Generator().manual_seed(0)
        q, k, v = (torch.randn(2, 3, 5, 4, generator=gen, dtype=torch.float64) for _ in range(3))
        bias = torch.randn(2, 1, 1, 5, generator=gen, dtype=torch.float64)
        if masked:
            bias[0, 0, 0, 1] = -torch.inf
            bias[1, 0, 0, 4] = -torch.inf
        cases[f"edge_attn_testshape_{'masked' if masked else 'plain'}"] = attn_case(
            op, q, k, v, bias, 0.5, gen
        )
    # the microbenchmark's distribution at a small n: K=32, H=8, D=32,
    # bias ~ N(0, 0.1) per (n, h, i, j), keys j >= c_n masked, c_n ~ U{8..32}
    gen = torch.Generator().manual_seed(0)
    n, h, s, d = 6, 2, 32, 32
    q, k, v = (torch.randn(n, h, s, d, generator=gen, dtype=torch.float64) for _ in range(3))
    bias = 0.1 * torch.randn(n, h, s, s, generator=gen, dtype=torch.float64)
    counts = torch.randint(8, s + 1, (n,), generator=gen)
    keymask = torch.arange(s)[None, :] >= counts[:, None]  # (n, s)
    bias = bias.masked_fill(keymask[:, None, None, :], -torch.inf)
    case = attn_case(op, q, k, v, bias, 1.0 / np.sqrt(d), gen)
    case["key_counts"] = counts.numpy().astype(np.int32)
    cases["edge_attn_cfg2_small"] = case
    # the model's layout: bias (n, h, 1, s) broadcast over queries, all rows valid
    gen = torch.Generator().manual_seed(1)
    n, h, s, d = 3, 2, 30, 64
    q, k, v = (torch.randn(n, h, s, d, generator=gen, dtype=torch.float64) for _ in range(3))
    bias = torch.randn(n, h, 1, s, generator=gen, dtype=torch.float64)
    cases["edge_attn_keybias"] = attn_case(op, q, k, v, bias, 0.125, gen)
    return cases


def mlp_step_fixture(ref_cg) -> dict:
    """One config-1 training step through the reference's own create_graph:
    4 molecules x 32 atoms, pos ~ N(0, 1.5 A) from seed 0, each molecule
    centred eagerly outside the region; per-atom MLP 3 -> 64 -> 64 -> 1 with
    SiLU inside cg.compile; E = per-molecule sum; loss = MSE(E) + MSE(F),
    F = -dE/dpos. Float64, default (compiled) backend and exact=True."""
    from torch import nn

    torch.manual_seed(0)

    class Network(nn.Module):
        def __init__(self):
            super().__init__()
            self.l1, self.l2, self.l3 = nn.Linear(3, 64), nn.Linear(64, 64), nn.Linear(64, 1)

        def forward(self, x, mol):
            h = torch.nn.functional.silu(self.l1(x))
            h = torch.nn.functional.silu(self.l2(h))
            e_atom = self.l3(h)[:, 0]
            return torch.zeros(4, dtype=x.dtype).index_add(0, mol, e_atom)

    class Model(nn.Module):
        def __init__(self):
            super().__init__()
            self.network = ref_cg.compile(Network(), config=ref_cg.CompileConfig(backend="aot_eager"))

        def forward(self, batch):
            pos = batch["pos"].view(4, 32, 3)
            centred = (pos - pos.mean(dim=1, keepdim=True)).view(128, 3)
            return {"energy": self.network(centred, batch["mol"])}

    model = Model().double()
    gen = torch.Generator().manual_seed(0)
    pos = 1.5 * torch.randn(128, 3, generator=gen, dtype=torch.float64)
    mol = torch.arange(128) // 32
    e_target = torch.randn(4, generator=gen, dtype=torch.float64)
    f_target = torch.randn(128, 3, generator=gen, dtype=torch.float64)
    out = {"pos": pos.numpy(), "e_target": e_target.numpy(), "f_target": f_target.numpy()}
    for name, p in model.network.module.named_parameters():
        out[f"param.{name}"] = p.detach().numpy().copy()
    for label, exact in (("compiled", False), ("exact", True)):
        model.zero_grad()
        res, grads = ref_cg.create_graph(model, {"pos": pos, "mol": mol}, exact=exact)
        forces = -grads["pos"]
        loss = (res["energy"] - e_target).square().mean() + (forces - f_target).square().mean()
        loss.backward()
        out[f"{label}.energy"] = res["energy"].detach().numpy()
        out[f"{label}.forces"] = forces.detach().numpy()
        out[f"{label}.loss"] = loss.detach().numpy()
        for name, p in model.network.module.named_parameters():
            out[f"{label}.grad.{name}"] = p.grad.detach().numpy().copy()
    return out


MLIP_SEED = 7
MLIP_SIZES = (64, 64, 64)


def mlip_step_fixture(ref_cg) -> dict:
    """One training step of the small edge-attention MLIP through the
    reference's own create_graph: the small-MLIP spec (C 128, 4 heads of 32,
    4 blocks, FFN 512, 64 RBF, 6 A cutoff, k <= 32, 10 species) on 3 of the
    workload's 64-atom systems. Inside ``cg.compile`` runs oracle/step.py's
    ``energy``; the neighbour lists come from oracle/neighbors.py outside the
    region; loss = MSE(E) + MSE(F). Float64, compiled (aot_eager) and exact.

    Parameters are the model's own initial draws under torch.manual_seed(seed)
    (regenerated by the tests, with per-tensor sums stored to catch drift);
    gradients of more than oracle.sketch.FULL_LIMIT elements are stored as
    seeded sign-vector sketches."""
    from torch import nn

    from create_graph_b200 import mlip
    from oracle import neighbors as onb
    from oracle import step as ostep
    from oracle.sketch import sketch

    spec = mlip.SMALL_MLIP
    torch.manual_seed(MLIP_SEED)
    params = {name: t.double() for name, t in mlip.reference_parameters(spec).items()}
    names = list(params)
    pos, species, sys_ptr = mlip.synthetic_systems(list(MLIP_SIZES), spec.n_species, seed=MLIP_SEED)
    e_target, f_target = mlip.make_targets(len(MLIP_SIZES), pos.shape[0], seed=MLIP_SEED + 1)
    nbr, counts, _, _ = onb.neighbor_list(pos.numpy(), sys_ptr.numpy(), spec.cutoff, spec.k)
    nbr_t, counts_t = torch.from_numpy(nbr), torch.from_numpy(counts)

    class Network(nn.Module):
        def __init__(self):
            super().__init__()
            self.weights = nn.ParameterList(nn.Parameter(params[n].clone()) for n in names)

        def forward(self, x, species, sys_ptr, nbr, counts):
            return ostep.energy(dict(zip(names, self.weights)), spec, x, species, sys_ptr, nbr, counts)

    class Model(nn.Module):
        def __init__(self, config):
            super().__init__()
            self.network = ref_cg.compile(Network(), config=config)

        def forward(self, batch):
            return {"energy": self.network(batch["pos"], batch["species"], batch["sys_ptr"], batch["nbr"],
                                           batch["counts"])}

    out = {
        "seed": np.array(MLIP_SEED), "pos": pos.numpy(), "species": species.numpy(), "sys_ptr": sys_ptr.numpy(),
        "nbr": nbr, "counts": counts, "e_target": e_target.numpy(), "f_target": f_target.numpy(),
    }
    for name in names:
        out[f"param_sum.{name}"] = np.array([float(params[name].sum()), float(params[name].square().sum())])
    batch = {"pos": pos.double(), "species": species, "sys_ptr": sys_ptr, "nbr": nbr_t, "counts": counts_t}
    for label, exact in (("compiled", False), ("exact", True)):
        model = Model(ref_cg.CompileConfig(backend="aot_eager"))
        res, grads = ref_cg.create_graph(model, batch, exact=exact)
        forces = -grads["pos"]
        loss = (res["energy"] - e_target.double()).square().mean() + (forces - f_target.double()).square().mean()
        loss.backward()
        out[f"{label}.energy"] = res["energy"].detach().numpy()
        out[f"{label}.forces"] = forces.detach().numpy()
        out[f"{label}.loss"] = loss.detach().numpy()
        for name, p in zip(names, model.network.module.weights):
            out[f"{label}.grad.{name}"] = sketch(name, p.grad).numpy()
    return out


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, help="root of the reference checkout (read-only)")
    args = parser.parse_args()
    sys.path.insert(0, str(REPO))
    ref_cg, op = import_reference(args.reference)
    fixtures = edge_attn_fixtures(op)
    fixtures["mlp_step"] = mlp_step_fixture(ref_cg)
    fixtures["mlip_step"] = mlip_step_fixture(ref_cg)
    for name, arrays in fixtures.items():
        path = HERE / f"{name}.npz"
        np.savez_compressed(path, **arrays)
        print(path, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    main()
