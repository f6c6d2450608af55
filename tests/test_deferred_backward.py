"""
The deferred first-order backward of checkpointed blocks, on the CPU in
float64 (host logic only). A toy fused op uses the same hooks as the package's
fused ops (checkpoint.deferral_slot / cut_forward_tensor / deferred_cotangent,
which create_graph_b200.nn names _op_slot / _cut / _deferred), and a
cg.custom_op operator takes part by itself: while the parameter backward
differentiates a block's VJP, the op's backward reads its forward tensors
through leaves, and the cotangents they receive are added where the block's
own backward passes them. Results must equal eager create_graph at 1e-10 with
the deferral on (budget above 0.25) and off, and the op's backward must run
once less per block with it on.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

import create_graph_b200 as cg
from create_graph_b200.nn import _cut, _deferred, _Fused, _op_slot, _plus
from create_graph_b200.testing import check_create_graph, check_op

F64 = torch.float64


class ToyLayer(_Fused):
    """out = x + tanh(x @ w.T) * s; backward from torch ops (differentiable
    when recorded), reading x and s through _cut."""

    calls = 0

    @staticmethod
    def forward(ctx, x, w, s):
        ctx.op = _op_slot()
        ctx.save_for_backward(x, w, s)
        return x + torch.tanh(x @ w.t()) * s

    @staticmethod
    def backward(ctx, g):
        ToyLayer.calls += 1
        x, w, s = ctx.saved_tensors
        cx, cs = _deferred(ctx, "x"), _deferred(ctx, "s")
        x, s = _cut(ctx, "x", x), _cut(ctx, "s", s)
        t = torch.tanh(x @ w.t())
        u = g * s * (1 - t * t)
        gx = g + u @ w
        gw = u.t() @ x
        gs = (g * t).sum(-1, keepdim=True)
        return _plus(gx, cx), gw, _plus(gs, cs)


class ToyBlock(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.norm = nn.LayerNorm(width)  # plain torch: its tensors are not cut
        self.w1 = nn.Parameter(torch.randn(width, width) / width**0.5)
        self.w2 = nn.Parameter(torch.randn(width, width) / width**0.5)

    def forward(self, h, dist):
        s = torch.cos(dist)[:, None]
        return h + ToyLayer.apply(ToyLayer.apply(self.norm(h), self.w1, s), self.w2, s)


class ToyStack(nn.Module):
    def __init__(self, width=8, depth=3):
        super().__init__()
        self.inp = nn.Linear(4, width)
        self.blocks = nn.ModuleList(ToyBlock(width) for _ in range(depth))
        self.out = nn.Linear(width, 1)

    def forward(self, vec, dist, system, n_systems):
        h = self.inp(torch.cat([vec, dist[:, None]], dim=-1))
        for block in self.blocks:
            h = block(h, dist)
        return torch.zeros(n_systems, dtype=h.dtype).index_add(0, system, self.out(h).squeeze(-1))


class ToyModel(nn.Module):
    def __init__(self, budget):
        super().__init__()
        config = cg.CompileConfig(backend="eager", checkpoint=r"blocks\.\d+", memory_budget=budget)
        self.region = cg.compile(ToyStack(), config=config)

    def forward(self, data):
        vec = data["pos"][data["dst"]] - data["pos"][data["src"]]
        return {"energy": self.region(vec, vec.norm(dim=-1), data["system"], data["n_systems"])}


def toy_data(e=24, n=9, systems=3, seed=0):
    gen = torch.Generator().manual_seed(seed)
    src = torch.randint(0, n, (e,), generator=gen)
    dst = (src + torch.randint(1, n, (e,), generator=gen)) % n
    return {"pos": torch.randn(n, 3, generator=gen, dtype=F64), "src": src, "dst": dst,
            "system": torch.arange(e) * systems // e, "n_systems": systems}


@pytest.mark.parametrize("budget", [1.0, 0.5, 0.25])
def test_deferred_backward_matches_eager(budget):
    torch.manual_seed(0)
    model = ToyModel(budget).to(F64)
    errors = check_create_graph(model, toy_data())
    bad = {k: v for k, v in errors.items() if v > 1e-10}
    assert not bad, errors


def _backward_calls(budget):
    torch.manual_seed(0)
    model = ToyModel(budget).to(F64)
    data = toy_data(seed=1)
    out, grads = cg.create_graph(model, data)
    ToyLayer.calls = 0
    (out["energy"].sum() + grads["pos"].square().sum()).backward()
    return ToyLayer.calls


def test_deferral_runs_the_forward_ops_backward_once():
    depth = len(ToyStack().blocks)
    # per block: the VJP's rebuild (both layers), its differentiation through
    # the first layer, whose output the second layer's backward reads (only
    # without the deferral), then the block's own backward (both layers)
    assert _backward_calls(0.25) == 5 * depth
    assert _backward_calls(0.5) == 4 * depth
    assert _backward_calls(1.0) == 4 * depth


class ForgetfulLayer(ToyLayer):
    """A planted mistake: reads x through _cut but never adds its deferred
    cotangent back."""

    @staticmethod
    def backward(ctx, g):
        x, w, s = ctx.saved_tensors
        x = _cut(ctx, "x", x)
        t = torch.tanh(x @ w.t())
        u = g * s * (1 - t * t)
        return g + u @ w, u.t() @ x, (g * t).sum(-1, keepdim=True)


def test_an_unconsumed_deferred_cotangent_is_an_error(monkeypatch):
    monkeypatch.setattr(ToyLayer, "apply", ForgetfulLayer.apply)
    torch.manual_seed(0)
    model = ToyModel(0.5).to(F64)
    out, grads = cg.create_graph(model, toy_data())
    with pytest.raises(RuntimeError, match="deferred cotangents"):
        (out["energy"].sum() + grads["pos"].square().sum()).backward()


def test_defers_only_above_a_quarter_and_before_the_block_backward():
    from create_graph_b200.checkpoint import _BlockCall

    block = nn.Linear(2, 2)
    for budget, want in ((None, True), (1.0, True), (0.5, True), (0.25, False), (0.1, False)):
        call = _BlockCall(block, cg.CompileConfig(memory_budget=budget), (torch.zeros(1, 2),), {})
        assert call.defers() is want, budget
        call.backward_done = True
        assert not call.defers()


# ---------------------------------------------------------------------------
# cg.custom_op operators take part as well
# ---------------------------------------------------------------------------


BACKWARD1_CALLS = [0]


@cg.custom_op("cg_b200_tests::scaled_tanh")
class ScaledTanh:
    """y = x + a * tanh(x * w) over rows x (n, C) and w (C,); t = tanh(x * w)
    is a statistic kept for backward1."""

    outputs = ("y", "t")
    save = ("x", "w", "t")
    nondiff = ("t",)

    @staticmethod
    def forward1(x: torch.Tensor, w: torch.Tensor, a: float) -> tuple[torch.Tensor, torch.Tensor]:
        t = torch.tanh(x * w)
        return x + a * t, t

    @staticmethod
    def fake(x, w, a):
        return torch.empty_like(x), torch.empty_like(x)

    @staticmethod
    def backward1(x, w, t, grad_y, a):
        BACKWARD1_CALLS[0] += 1
        d = 1 - t * t
        return grad_y * (1 + a * d * w), (grad_y * a * d * x).sum(0)

    @staticmethod
    def backward2(x, w, t, grad_y, a, gg_x, gg_w):
        d = 1 - t * t
        dd = -2 * t * d           # d(1 - tanh^2) / dz
        u = gg_x * w + gg_w * x   # <gg, (gx, gw)> = sum grad_y * (gg_x + a * d * u)
        dx = grad_y * a * (u * dd * w + gg_w * d)
        dw = (grad_y * a * (u * dd * x + gg_x * d)).sum(0)
        return dx, dw, gg_x + a * d * u


def scaled_tanh_ref(x, w, a):
    t = torch.tanh(x * w)
    return x + a * t, t


class OpBlock(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.lin = nn.Linear(width, width)
        self.w1 = nn.Parameter(torch.randn(width) * 0.7)
        self.w2 = nn.Parameter(torch.randn(width) * 0.7)

    def forward(self, h, dist):
        y1, _ = ScaledTanh(self.lin(h), self.w1, 0.7)
        y2, _ = ScaledTanh(y1, self.w2, 0.3)
        # (no plain op here whose backward reads y2: it would take the VJP's
        # differentiation through both ops whatever they do)
        return h + y2


class OpModel(ToyModel):
    def __init__(self, budget):
        nn.Module.__init__(self)
        stack = ToyStack()
        stack.blocks = nn.ModuleList(OpBlock(8) for _ in range(len(stack.blocks)))
        config = cg.CompileConfig(backend="eager", checkpoint=r"blocks\.\d+", memory_budget=budget)
        self.region = cg.compile(stack, config=config)


def test_custom_op_kernels_match_reference():
    gen = torch.Generator().manual_seed(0)
    args = (torch.randn(5, 4, generator=gen, dtype=F64), torch.randn(4, generator=gen, dtype=F64), 0.7)
    errors = check_op(ScaledTanh, scaled_tanh_ref, args)
    assert max(errors.values()) < 1e-10, errors


@pytest.mark.parametrize("budget", [0.5, 0.25])
def test_custom_op_deferred_backward_matches_eager(budget):
    torch.manual_seed(0)
    model = OpModel(budget).to(F64)
    errors = check_create_graph(model, toy_data())
    bad = {k: v for k, v in errors.items() if v > 1e-10}
    assert not bad, errors


def test_custom_op_backward1_runs_once_less_per_block():
    def calls(budget):
        torch.manual_seed(0)
        model = OpModel(budget).to(F64)
        out, grads = cg.create_graph(model, toy_data(seed=1))
        BACKWARD1_CALLS[0] = 0
        (out["energy"].sum() + grads["pos"].square().sum()).backward()
        return BACKWARD1_CALLS[0]

    depth = len(ToyStack().blocks)
    assert calls(0.25) == 5 * depth
    assert calls(0.5) == 4 * depth
