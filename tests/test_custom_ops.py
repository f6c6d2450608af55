"""
``cg.custom_op`` on the CPU (host logic): the three registered operators, their
schemas and autograd, checked with ``cg.testing.check_op`` against
differentiable references in float64 at 1e-10, an op inside a region against
eager create_graph, and the registration errors. The GPU kernels behind the
package's own edge-attention op are tested in test_edge_attn_gpu.py.
"""

from __future__ import annotations

import pytest
import torch
from torch import Tensor, nn

import create_graph_b200 as cg
from create_graph_b200.testing import check_create_graph, check_op

TOL = 1e-10


@cg.custom_op("cg_b200_tests::softplus_scaled")
class SoftplusScaled:
    """y = a * softplus(x * w), with a statistic s = sigmoid(x * w) kept for backward."""

    outputs = ("y", "s")
    save = ("x", "w", "s")
    nondiff = ("s",)

    @staticmethod
    def forward1(x: Tensor, w: Tensor, a: float) -> tuple[Tensor, Tensor]:
        z = x * w
        return a * torch.nn.functional.softplus(z), torch.sigmoid(z)

    @staticmethod
    def fake(x, w, a):
        return torch.empty_like(x), torch.empty_like(x)

    @staticmethod
    def backward1(x, w, s, grad_y, a):
        return a * s * w * grad_y, a * s * x * grad_y

    @staticmethod
    def backward2(x, w, s, grad_y, a, gg_x, gg_w):
        ds = s * (1 - s)  # d sigmoid / dz
        # gx = a s w g, gw = a s x g; differentiate <gg_x, gx> + <gg_w, gw>
        t = a * grad_y * (gg_x * w + gg_w * x)
        dx = t * ds * w + a * s * grad_y * gg_w
        dw = t * ds * x + a * s * grad_y * gg_x
        dg = a * s * (gg_x * w + gg_w * x)
        return dx, dw, dg


def softplus_ref(x, w, a):
    z = x * w
    return a * torch.nn.functional.softplus(z), torch.sigmoid(z)


def test_three_kernels_match_reference():
    gen = torch.Generator().manual_seed(0)
    args = (torch.randn(5, 4, generator=gen, dtype=torch.float64), torch.randn(5, 4, generator=gen, dtype=torch.float64), 0.7)
    errors = check_op(SoftplusScaled, softplus_ref, args)
    assert max(errors.values()) < TOL, errors
    assert {"forward1.y", "backward1.x", "backward1.w", "backward2.x", "backward2.w", "backward2.grad_y"} <= set(errors)


def test_registered_schemas():
    assert "float a" in str(SoftplusScaled.backward1_op._opoverload._schema)
    assert "Tensor gg_w" in str(SoftplusScaled.backward2_op._opoverload._schema)


class OpModel(nn.Module):
    def __init__(self, op: bool):
        super().__init__()
        self.op = op
        self.lin = nn.Linear(4, 4)
        self.w = nn.Parameter(torch.randn(4))
        self.region = cg.compile(self._energy)

    def _energy(self, vec, dist):
        x = self.lin(torch.cat([vec, dist[:, None]], -1))
        y = SoftplusScaled(x, self.w.expand_as(x), 0.7)[0] if self.op else softplus_ref(x, self.w, 0.7)[0]
        return y.sum().reshape(1)

    def forward(self, data):
        vec = data["pos"][1:] - data["pos"][:-1]
        return {"energy": self.region(vec, vec.norm(dim=-1))}


def test_op_inside_region_matches_eager_and_reference_model():
    data = {"pos": torch.randn(8, 3, generator=torch.Generator().manual_seed(1), dtype=torch.float64)}
    torch.manual_seed(0)
    model = OpModel(op=True).double()
    errors = check_create_graph(model, data)
    assert max(errors.values()) < TOL, errors
    loss = cg.testing.coupled_loss()
    got = cg.testing.run_step(model, data, outputs="energy", inputs=("pos",), loss=loss, exact=False)
    model.op = False
    want = cg.testing.run_step(model, data, outputs="energy", inputs=("pos",), loss=loss, exact=True)
    assert cg.testing.rel_err(got["grads"]["pos"], want["grads"]["pos"]) < TOL
    assert cg.testing.grad_errors(got["params"], want["params"])["all"] < TOL


def test_backward1_needs_every_tensor_input_saved():
    with pytest.raises(cg.ContractError, match="save them all"):

        @cg.custom_op("cg_b200_tests::bad_save")
        class Bad:
            outputs = ("y",)
            save = ("x",)

            @staticmethod
            def forward1(x: Tensor, w: Tensor) -> Tensor:
                return x * w

            @staticmethod
            def backward1(x, grad_y):
                return grad_y, grad_y

            @staticmethod
            def backward2(x, grad_y, gg_x, gg_w):
                return gg_x, gg_x


def test_non_tensor_argument_types_are_checked():
    with pytest.raises(cg.ContractError, match="non-tensor"):

        @cg.custom_op("cg_b200_tests::bad_type")
        class BadType:
            outputs = ("y",)
            save = ("x",)

            @staticmethod
            def forward1(x: Tensor, n: list[int]) -> Tensor:
                return x

            @staticmethod
            def backward1(x, grad_y, n):
                return grad_y

            @staticmethod
            def backward2(x, grad_y, n, gg_x):
                return gg_x


def test_unknown_save_name_is_refused():
    with pytest.raises(cg.ContractError, match="not an argument or output"):

        @cg.custom_op("cg_b200_tests::bad_name")
        class BadName:
            outputs = ("y",)
            save = ("nope",)

            @staticmethod
            def forward1(x: Tensor) -> Tensor:
                return x * 2
