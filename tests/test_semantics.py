"""
The region mechanism on the CPU in float64 (host logic only: plain torch ops
inside the regions). Every case compares ``cg.create_graph`` with
``exact=True`` (eager ``torch.autograd.grad(create_graph=True)``) on the same
model and data: output, input gradients, a loss coupling both, and that loss's
parameter gradients, at 1e-10 -- the method of the reference's own mechanism
tests (tests/test_semantics.py there). Also the contract errors, eval mode,
structured inputs and per-block recompute.
"""

from __future__ import annotations

import dataclasses
import warnings

import pytest
import torch
from torch import nn

import create_graph_b200 as cg
from create_graph_b200.compile_config import compiled_graph_count
from create_graph_b200.testing import check_create_graph

TOL = 1e-10
F64 = torch.float64


def graph_data(n=10, e=28, systems=3, seed=0):
    gen = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (e,), generator=gen)
    dst = (src + torch.randint(1, n, (e,), generator=gen)) % n
    return {
        "pos": torch.randn(n, 3, generator=gen, dtype=F64),
        "src": src,
        "dst": dst,
        "system": torch.arange(n) * systems // n,
        "n_systems": systems,
        "species": torch.randint(0, 3, (n,), generator=gen),
    }


def edges(data):
    vec = data["pos"][data["dst"]] - data["pos"][data["src"]]
    return vec, vec.norm(dim=-1)


def small_ok(errors, tol=TOL):
    bad = {k: v for k, v in errors.items() if v > tol}
    assert not bad, f"above {tol}: {bad} (all {errors})"


class EdgeEnergy(nn.Module):
    """Edge features -> per-system energies with a norm, an MLP and index_add reductions."""

    def __init__(self, width=12, norm="ln", act="silu"):
        super().__init__()
        self.inp = nn.Linear(4, width)
        self.norm = nn.LayerNorm(width) if norm == "ln" else nn.RMSNorm(width)
        acts = {"silu": nn.SiLU(), "gelu": nn.GELU(), "tanh": nn.Tanh()}
        self.mlp = nn.Sequential(nn.Linear(width, width), acts[act], nn.Linear(width, width))
        self.head = nn.Linear(width, 1)

    def forward(self, vec, dist, src, system, n_systems):
        h = self.norm(self.inp(torch.cat([vec, dist[:, None]], dim=-1)))
        h = h + self.mlp(h)
        e_edge = self.head(h * torch.sigmoid(h)).squeeze(-1)
        e_atom = torch.zeros(system.shape[0], dtype=e_edge.dtype).index_add(0, src, e_edge)
        return torch.zeros(n_systems, dtype=e_edge.dtype).index_add(0, system, e_atom)


class Model(nn.Module):
    def __init__(self, config=None, **kw):
        super().__init__()
        self.energy = EdgeEnergy(**kw)
        self.region = cg.compile(self.energy, config=config or cg.CompileConfig(backend="aot_eager"))

    def forward(self, data):
        vec, dist = edges(data)
        return {"energy": self.region(vec, dist, data["src"], data["system"], data["n_systems"])}


def make(cls=Model, **kw):
    torch.manual_seed(0)
    return cls(**kw).to(F64)


@pytest.mark.parametrize("norm", ["ln", "rms"])
@pytest.mark.parametrize("act", ["silu", "gelu", "tanh"])
def test_region_after_eager_geometry(norm, act):
    small_ok(check_create_graph(make(norm=norm, act=act), graph_data()))


@pytest.mark.parametrize("backend", ["inductor", "aot_eager", "eager"])
def test_backends(backend):
    small_ok(check_create_graph(make(config=cg.CompileConfig(backend=backend)), graph_data()))


def test_module_region_with_tensor_output():
    class Whole(nn.Module):
        def __init__(self):
            super().__init__()
            self.energy = EdgeEnergy()

        def forward(self, data):
            vec, dist = edges(data)
            return self.energy(vec, dist, data["src"], data["system"], data["n_systems"])

    torch.manual_seed(0)
    model = cg.compile(Whole().to(F64))
    small_ok(check_create_graph(model, graph_data(), outputs=None))


class Mixed(Model):
    """A parameter mixed with positions before the region, and a parameter-only input."""

    def __init__(self):
        super().__init__()
        self.scale = nn.Parameter(torch.tensor(0.8))
        self.embed = nn.Embedding(3, 3)

    def forward(self, data):
        vec, dist = edges(data)
        vec = vec + self.embed(data["species"])[data["src"]]
        dist = dist * self.scale
        return {"energy": self.region(vec, dist, data["src"], data["system"], data["n_systems"])}


def test_mixed_and_parameter_only_inputs():
    model = make(Mixed)
    small_ok(check_create_graph(model, graph_data()))
    out, grads = cg.create_graph(model, graph_data())
    (out["energy"].sum() + grads["pos"].square().sum()).backward()
    assert model.scale.grad is not None and model.embed.weight.grad.abs().sum() > 0


class Inside(nn.Module):
    """detach, no_grad, in-place and a Function on parameters inside the region."""

    class Square(torch.autograd.Function):
        @staticmethod
        def forward(ctx, x):
            ctx.save_for_backward(x)
            return x * x

        @staticmethod
        def backward(ctx, g):
            (x,) = ctx.saved_tensors
            return 2 * x * g

    def __init__(self, features):
        super().__init__()
        self.features = features
        self.lin = nn.Linear(3, 3)
        self.energy = EdgeEnergy()

    def forward(self, vec, dist, src, system, n_systems):
        v = self.lin(vec)
        if "detach" in self.features:
            v = v * dist.detach().mean()
        if "no_grad" in self.features:
            with torch.no_grad():
                top = vec.abs().max()
            v = v / top
        if "inplace" in self.features:
            v = v.clone()
            v[:, 1] += dist
        if "param_function" in self.features:
            v = v * self.Square.apply(self.lin.bias).sum()
        if "function" in self.features:
            v = self.Square.apply(v)
        return self.energy(v, dist, src, system, n_systems)


class InsideModel(nn.Module):
    def __init__(self, features, backend="aot_eager"):
        super().__init__()
        self.region = cg.compile(Inside(features), config=cg.CompileConfig(backend=backend))

    def forward(self, data):
        vec, dist = edges(data)
        return {"energy": self.region(vec, dist, data["src"], data["system"], data["n_systems"])}


@pytest.mark.parametrize(
    "features", [("detach",), ("no_grad",), ("inplace",), ("param_function",), ("detach", "no_grad", "inplace")]
)
def test_autograd_semantics_inside_region(features):
    small_ok(check_create_graph(make(InsideModel, features=features), graph_data()))


def test_user_function_on_differentiated_path_is_refused():
    with pytest.raises(cg.ContractError, match="torch.autograd.Function Square"):
        cg.create_graph(make(InsideModel, features=("function",)), graph_data())


def test_user_function_is_exact_with_eager_backend():
    small_ok(check_create_graph(make(InsideModel, features=("function",), backend="eager"), graph_data()))


def test_eval_mode_is_first_order_and_detached():
    model = make()
    data = graph_data()
    out, grads = cg.create_graph(model, data, train=False)
    assert not out["energy"].requires_grad and not grads["pos"].requires_grad
    pos = data["pos"].detach().requires_grad_(True)
    vec, dist = edges({**data, "pos": pos})
    e = model.energy(vec, dist, data["src"], data["system"], data["n_systems"])
    (want,) = torch.autograd.grad(e.sum(), pos)
    assert cg.testing.rel_err(grads["pos"], want) < TOL


def test_output_selection_by_callable():
    small_ok(check_create_graph(make(), graph_data(), outputs=lambda out: out["energy"]))


def test_several_differentiated_inputs():
    class Field(Model):
        def forward(self, data):
            vec, dist = edges(data)
            vec = vec + data["field"]
            return {"energy": self.region(vec, dist, data["src"], data["system"], data["n_systems"])}

    data = graph_data()
    data["field"] = torch.randn(3, dtype=F64)
    small_ok(check_create_graph(make(Field), data, inputs=("pos", "field")))


@dataclasses.dataclass
class EdgeSet:
    vec: torch.Tensor
    dist: torch.Tensor
    src: torch.Tensor
    system: torch.Tensor
    n_systems: int


class Record:
    """A plain object with tensor attributes (like fairchem's AtomicData)."""

    def __init__(self, d):
        self.__dict__.update(d)


class DataclassModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.energy = EdgeEnergy()
        self.region = cg.compile(self._energy)

    def _energy(self, es: EdgeSet):
        return self.energy(es.vec, es.dist, es.src, es.system, es.n_systems)

    def forward(self, data):
        vec = data.pos[data.dst] - data.pos[data.src]
        return {"energy": self.region(EdgeSet(vec, vec.norm(dim=-1), data.src, data.system, data.n_systems))}


class ObjectModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.energy = EdgeEnergy()
        self.region = cg.compile(self._energy)

    def _energy(self, data):
        vec = data.pos[data.dst] - data.pos[data.src]
        return self.energy(vec, vec.norm(dim=-1), data.src, data.system, data.n_systems)

    def forward(self, data):
        return {"energy": self.region(data)}


@pytest.mark.parametrize("cls", [DataclassModel, ObjectModel])
def test_structured_inputs(cls):
    small_ok(check_create_graph(make(cls), Record(graph_data())))


# ---------------------------------------------------------------------------
# contract errors
# ---------------------------------------------------------------------------


class TwoRegions(Model):
    def __init__(self):
        super().__init__()
        self.second = cg.compile(EdgeEnergy())

    def forward(self, data):
        vec, dist = edges(data)
        a = (data["src"], data["system"], data["n_systems"])
        return {"energy": self.region(vec, dist, *a) + self.second(vec, dist, *a)}


class GradInModel(Model):
    def forward(self, data):
        out = super().forward(data)
        torch.autograd.grad(out["energy"].sum(), data["pos"], create_graph=True)
        return out


class Doubled(Model):
    def forward(self, data):
        return {"energy": 2.0 * super().forward(data)["energy"]}


class PosAfterRegion(Model):
    def forward(self, data):
        _, dist = edges(data)
        return {"energy": super().forward(data)["energy"] + dist.sum()}


class Shifted(Model):
    def __init__(self):
        super().__init__()
        self.shift = nn.Parameter(torch.tensor([0.1, -0.2, 0.3]))

    def forward(self, data):
        return {"energy": super().forward(data)["energy"] + self.shift}


@pytest.mark.parametrize(
    "cls, match",
    [
        (TwoRegions, "both depend on the differentiated inputs"),
        (GradInModel, "computed a gradient w.r.t. a differentiated input"),
        (Doubled, "scales or drops entries"),
        (PosAfterRegion, "also depends on the differentiated inputs"),
    ],
)
def test_contract_errors(cls, match):
    with pytest.raises(cg.ContractError, match=match):
        cg.create_graph(make(cls), graph_data())


def test_position_independent_terms_may_be_added():
    small_ok(check_create_graph(make(Shifted), graph_data()))


def test_no_region_warns_and_is_exact():
    class Plain(nn.Module):
        def __init__(self):
            super().__init__()
            self.energy = EdgeEnergy()

        def forward(self, data):
            vec, dist = edges(data)
            return {"energy": self.energy(vec, dist, data["src"], data["system"], data["n_systems"])}

    with warnings.catch_warnings(record=True) as caught:
        warnings.simplefilter("always")
        small_ok(check_create_graph(make(Plain), graph_data()))
    assert any("ran no cg.compile region" in str(w.message) for w in caught)


def test_config_validation():
    with pytest.raises(ValueError, match="backend"):
        cg.CompileConfig(backend="tvm")
    with pytest.raises(ValueError, match="memory_budget"):
        cg.CompileConfig(memory_budget=0.0)
    c = cg.CompileConfig(options={"b": 1, "a": 2})
    assert c.options == (("a", 2), ("b", 1)) and hash(c) == hash(c.replace())


# ---------------------------------------------------------------------------
# per-block recompute
# ---------------------------------------------------------------------------


class Block(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.norm = nn.LayerNorm(width)
        self.ff = nn.Sequential(nn.Linear(width, 2 * width), nn.SiLU(), nn.Linear(2 * width, width))

    def forward(self, h, dist, index=None):
        out = h + self.ff(self.norm(h)) * torch.cos(dist)[:, None]
        return out if index is None or index % 2 == 0 else 0.5 * out


class Stack(nn.Module):
    def __init__(self, width=10, depth=3, indexed=False):
        super().__init__()
        self.inp = nn.Linear(4, width)
        self.blocks = nn.ModuleList(Block(width) for _ in range(depth))
        self.out = nn.Linear(width, 1)
        self.indexed = indexed

    def forward(self, vec, dist, src, system, n_systems):
        h = self.inp(torch.cat([vec, dist[:, None]], dim=-1))
        for i, block in enumerate(self.blocks):
            h = block(h, dist, index=i) if self.indexed else block(h, dist)
        e_atom = torch.zeros(system.shape[0], dtype=h.dtype).index_add(0, src, self.out(h).squeeze(-1))
        return torch.zeros(n_systems, dtype=h.dtype).index_add(0, system, e_atom)


class StackModel(nn.Module):
    def __init__(self, pattern=r"blocks\.\d+", backend="aot_eager", indexed=False, budget=None):
        super().__init__()
        self.net = Stack(indexed=indexed)
        config = cg.CompileConfig(backend=backend, checkpoint=pattern, memory_budget=budget)
        self.region = cg.compile(self.net, config=config)

    def forward(self, data):
        vec, dist = edges(data)
        return {"energy": self.region(vec, dist, data["src"], data["system"], data["n_systems"])}


@pytest.mark.parametrize("backend", ["eager", "aot_eager"])
@pytest.mark.parametrize("indexed", [False, True])
def test_checkpointed_blocks(backend, indexed):
    small_ok(check_create_graph(make(StackModel, backend=backend, indexed=indexed, budget=0.5), graph_data()))


def test_checkpointed_blocks_eval():
    model = make(StackModel)
    data = graph_data()
    _, got = cg.create_graph(model, data, train=False)
    _, want = cg.create_graph(model, data, train=False, exact=True)
    assert cg.testing.rel_err(got["pos"], want["pos"]) < TOL


def test_checkpoint_pattern_must_match():
    with pytest.raises(cg.ContractError, match="matched no submodule"):
        cg.create_graph(make(StackModel, pattern=r"nothing\.here"), graph_data())


def test_one_plan_for_every_batch_size():
    model = make()
    counts = []
    for n, e, s in [(9, 30, 2), (14, 47, 3), (19, 66, 2), (23, 80, 4)]:
        out, grads = cg.create_graph(model, graph_data(n, e, s, seed=n))
        (out["energy"].sum() + grads["pos"].square().sum()).backward()
        counts.append(compiled_graph_count())
    assert counts[-1] == counts[0], counts
