"""
The small edge-attention MLIP's training step against the reference's own
create_graph.

``golden/mlip_step.npz`` holds what the reference's ``cg.create_graph``
(compiled aot_eager path and exact eager path, float64) returned for one step
of the small-MLIP spec (C 128, 4 heads of 32, 4 blocks, FFN 512, 64 RBF,
k <= 32) on three 64-atom systems, with oracle/step.py's energy function as the
region (tests/golden/make_golden.py). Here:

- on the CPU, oracle/step.py's own eager step reproduces those energies,
  forces, loss and parameter gradients to 1e-10 (float64): the oracle is
  pinned to the reference's create_graph mechanism on this model;
- on the GPU, the sm_100a step in fp32 precision (three-term tf32 products in
  the GEMMs and the attention) matches the same fixture within 1e-5 relative.

Parameters are the model's initial draws under the fixture's seed; their
per-tensor sums are checked first, so a change of the initialisation fails
loudly instead of comparing different models. Large gradients are compared
through the fixture's seeded sign sketches (oracle/sketch.py).
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest
import torch

from create_graph_b200 import mlip
from oracle import neighbors as onb
from oracle import step as ostep
from oracle.sketch import sketch

GOLDEN = np.load(Path(__file__).parent / "golden" / "mlip_step.npz")
SPEC = mlip.SMALL_MLIP


def rel(a, b) -> float:
    a, b = np.asarray(a, dtype=np.float64), np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def fixture_parameters() -> dict[str, torch.Tensor]:
    torch.manual_seed(int(GOLDEN["seed"]))
    params = mlip.reference_parameters(SPEC)
    for name, t in params.items():
        total, squares = GOLDEN[f"param_sum.{name}"]
        got = t.double()
        assert abs(float(got.sum()) - total) <= 1e-9 * max(1.0, abs(total)), f"{name}: initialisation changed"
        assert abs(float(got.square().sum()) - squares) <= 1e-9 * squares, f"{name}: initialisation changed"
    return params


def inputs():
    pos = torch.from_numpy(GOLDEN["pos"])
    species = torch.from_numpy(GOLDEN["species"])
    sys_ptr = torch.from_numpy(GOLDEN["sys_ptr"])
    e_t = torch.from_numpy(GOLDEN["e_target"])
    f_t = torch.from_numpy(GOLDEN["f_target"])
    return pos, species, sys_ptr, e_t, f_t


def compare(got: dict, label: str, tol: float) -> dict[str, float]:
    errs = {
        "energy": rel(got["energy"], GOLDEN[f"{label}.energy"]),
        "forces": rel(got["forces"], GOLDEN[f"{label}.forces"]),
        "loss": rel(got["loss"], GOLDEN[f"{label}.loss"]),
    }
    num = den = 0.0
    for name, g in got["grads"].items():
        want = GOLDEN[f"{label}.grad.{name}"]
        s = sketch(name, g).numpy()
        num += float(np.sum((s - want) ** 2))
        den += float(np.sum(want**2))
    errs["grads"] = (num / den) ** 0.5
    for key, err in errs.items():
        assert err < tol, f"{label} {key}: relative error {err:.3e} >= {tol}"
    return errs


def test_fixture_neighbor_list_is_the_oracles():
    pos, _, sys_ptr, _, _ = inputs()
    nbr, counts, _, _ = onb.neighbor_list(pos.numpy(), sys_ptr.numpy(), SPEC.cutoff, SPEC.k)
    assert np.array_equal(nbr, GOLDEN["nbr"]) and np.array_equal(counts, GOLDEN["counts"])


@pytest.mark.parametrize("label", ["exact", "compiled"])
def test_oracle_step_matches_reference_create_graph(label):
    params = {name: t.double() for name, t in fixture_parameters().items()}
    pos, species, sys_ptr, e_t, f_t = inputs()
    graph = (torch.from_numpy(GOLDEN["nbr"]), torch.from_numpy(GOLDEN["counts"]))
    got = ostep.train_step(params, SPEC, pos.double(), species, sys_ptr, e_t, f_t, graph=graph)
    compare(got, label, 1e-10)


@pytest.mark.gpu
def test_gpu_step_fp32_matches_reference_create_graph():
    import create_graph_b200 as cg
    from create_graph_b200 import native
    from create_graph_b200.graph import make_batch

    assert SPEC.gemm_precision == "fp32" and SPEC.attn_precision == "fp32"
    params = fixture_parameters()
    model = mlip.MLIP(SPEC).cuda()
    with torch.no_grad():
        for name, p in model.named_parameters():
            p.copy_(params[name])
    pos, species, sys_ptr, e_t, f_t = inputs()
    batch = make_batch(pos.float().cuda(), species.cuda(), sys_ptr.cuda(), SPEC.n_species)
    out, grads = cg.create_graph(model, batch)
    forces = -grads["pos"]
    loss = mlip.loss_fn(out["energy"], forces, e_t.float().cuda(), f_t.float().cuda())
    loss.backward()
    torch.cuda.synchronize()
    assert native.device_error() == 0
    got = {
        "energy": out["energy"].detach().cpu(),
        "forces": forces.detach().cpu(),
        "loss": loss.detach().cpu(),
        "grads": {n: p.grad.detach().cpu() for n, p in model.named_parameters()},
    }
    errs = compare(got, "exact", 1e-5)
    print("fp32 step vs the reference's create_graph:", {k: f"{v:.2e}" for k, v in errs.items()})
