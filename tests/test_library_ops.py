"""
The fused kernels registered as torch.library operators (create_graph_b200.library).

On the CPU, with fake CUDA tensors (FakeTensorMode, no GPU): every operator
returns the shapes and dtypes its kernel would, and a whole energy function
built from them -- neighbour list, edge geometry, SiLU linear layers, segment
sums -- traces with torch.fx (make_fx, fake mode) together with its force
(create_graph) and the gradient of a force loss, the path create_graph
differentiates twice: the traced graph contains the cg_b200 operators of both
derivative levels. On the GPU (``gpu`` marker): the operators, differentiated
twice, against plain float64 torch.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.fx.experimental.proxy_tensor import make_fx

import create_graph_b200.library  # noqa: F401  (registers the operators)

ops = torch.ops.cg_b200


def _fake_inputs(n=40, k=8, c=16):
    dev = "cuda"
    return {
        "pos": torch.empty(n, 3, device=dev),
        "sys_ptr": torch.empty(3, dtype=torch.int32, device=dev),
        "x": torch.empty(n, c, device=dev),
        "w": torch.empty(2 * c, c, device=dev),
        "b": torch.empty(2 * c, device=dev),
        "index": torch.empty(n, dtype=torch.int32, device=dev),
        "row_ptr": torch.empty(5, dtype=torch.int32, device=dev),
        "perm": torch.empty(n, dtype=torch.int32, device=dev),
    }


def test_fake_shapes_of_every_operator():
    with FakeTensorMode():
        t = _fake_inputs()
        n, c = t["x"].shape
        assert ops.mm(t["x"], t["w"]).shape == (n, 2 * c)
        assert ops.linear(t["x"], t["w"], t["b"]).shape == (n, 2 * c)
        y, z = ops.linear_silu(t["x"], t["w"], None)
        assert y.shape == z.shape == (n, 2 * c)
        assert ops.colsum(t["x"]).shape == (c,)
        assert ops.silu_grad(y, z).shape == y.shape
        assert ops.silu_grad2(y, y, z).shape == y.shape
        assert ops.segment_sum_csr(t["x"], t["index"], t["row_ptr"], t["perm"], 4).shape == (4, c)
        assert ops.gather_csr(t["x"][:4], t["index"], t["row_ptr"], t["perm"], 4).shape == (n, c)
        nbr, counts, rev_ptr, rev_idx = ops.neighbor_list(t["pos"], t["sys_ptr"], 30, 5.0, 8)
        assert nbr.shape == (n, 8) and nbr.dtype == torch.int32
        assert counts.shape == (n,) and rev_ptr.shape == (n + 1,) and rev_idx.shape == (n * 8,)
        rbf, env = ops.edge_geom(t["pos"], nbr, rev_ptr, rev_idx, 16, 5.0, 2.0)
        assert rbf.shape == (n * 8, 16) and env.shape == (n * 8,)
        g_pos = ops.edge_geom_bwd1(t["pos"], nbr, rev_ptr, rev_idx, rbf, env, 16, 5.0, 2.0)
        assert g_pos.shape == (n, 3)
        d = ops.edge_geom_bwd2(t["pos"], nbr, rev_ptr, rev_idx, rbf, env, g_pos, 16, 5.0, 2.0)
        assert [x.shape for x in d] == [(n, 3), (n * 8, 16), (n * 8,)]


def _energy(pos, sys_ptr, w1, b1, w2, sys_index, sys_row_ptr, sys_perm):
    nbr, _, rev_ptr, rev_idx = ops.neighbor_list(pos, sys_ptr, 30, 5.0, 8)
    rbf, env = ops.edge_geom(pos, nbr, rev_ptr, rev_idx, 16, 5.0, 2.0)
    h, _ = ops.linear_silu(rbf * env[:, None], w1, b1)
    e_edge = ops.linear(h, w2, None)
    atom = ops.segment_sum_csr(e_edge, rev_idx, rev_ptr, rev_idx, pos.shape[0])
    return ops.segment_sum_csr(atom, sys_index, sys_row_ptr, sys_perm, 2).sum()


def _force_loss_grad(pos, sys_ptr, w1, b1, w2, sys_index, sys_row_ptr, sys_perm):
    pos = pos.requires_grad_(True)
    e = _energy(pos, sys_ptr, w1, b1, w2, sys_index, sys_row_ptr, sys_perm)
    (g,) = torch.autograd.grad(e, pos, create_graph=True)
    loss = e + g.square().sum()
    return torch.autograd.grad(loss, [w1, b1, w2])


def test_energy_force_and_parameter_gradient_trace_under_fake_tensors():
    # fake CPU tensors: the autograd engine would look for a CUDA context for
    # fake CUDA ones, and the fakes do not depend on the device
    n, dev = 40, "cpu"
    with FakeTensorMode(allow_non_fake_inputs=False):
        pos = torch.empty(n, 3, device=dev)
        sys_ptr = torch.empty(3, dtype=torch.int32, device=dev)
        w1 = torch.empty(32, 16, device=dev, requires_grad=True)
        b1 = torch.empty(32, device=dev, requires_grad=True)
        w2 = torch.empty(1, 32, device=dev, requires_grad=True)
        sys_index = torch.empty(n, dtype=torch.int32, device=dev)
        sys_row_ptr = torch.empty(3, dtype=torch.int32, device=dev)
        sys_perm = torch.empty(n, dtype=torch.int32, device=dev)
        gm = make_fx(_force_loss_grad, tracing_mode="fake")(pos, sys_ptr, w1, b1, w2, sys_index, sys_row_ptr,
                                                             sys_perm)
    targets = {str(node.target) for node in gm.graph.nodes if node.op == "call_function"}
    for name in ("neighbor_list", "edge_geom", "edge_geom_bwd1", "edge_geom_bwd2", "linear_silu", "silu_grad",
                 "silu_grad2", "mm", "colsum", "segment_sum_csr", "gather_csr", "linear"):
        assert any(t.startswith(f"cg_b200.{name}.") for t in targets), (name, sorted(targets))


# ---------------------------------------------------------------------------
# numerics on the GPU
# ---------------------------------------------------------------------------


@pytest.mark.gpu
def test_linear_ops_twice_differentiated():
    from tests.twice import twice_errors

    gen = torch.Generator().manual_seed(0)
    x, w, b = (torch.randn(*s, generator=gen).cuda() for s in ((300, 96), (128, 96), (128,)))
    tol = 1e-2  # tf32 products (fp32 accumulation), after two derivatives
    for mine, ref in ((lambda *a: ops.linear(*a), F.linear),
                      (lambda *a: ops.linear_silu(*a)[0], lambda *a: F.silu(F.linear(*a)))):
        errs = twice_errors(mine, ref, [x, w, b])
        assert max(errs.values()) < tol, errs


@pytest.mark.gpu
def test_segment_sum_and_gather_twice_differentiated():
    from create_graph_b200.nn import Csr
    from tests.twice import twice_errors

    gen = torch.Generator().manual_seed(1)
    index = torch.randint(-1, 7, (50,), generator=gen, dtype=torch.int32).cuda()
    csr = Csr.from_index(index, 7)
    src = torch.randn(50, 12, generator=gen).cuda()

    def ref_sum(s):
        valid = index >= 0
        return torch.zeros(7, 12, dtype=s.dtype, device=s.device).index_add(0, index[valid].long(), s[valid])

    errs = twice_errors(lambda s: ops.segment_sum_csr(s, csr.index, csr.row_ptr, csr.perm, 7), ref_sum, [src])
    assert max(errs.values()) < 1e-6, errs


@pytest.mark.gpu
def test_edge_geometry_ops_twice_differentiated():
    from create_graph_b200 import mlip
    from tests.twice import twice_errors

    pos, _, sys_ptr = mlip.synthetic_systems([30, 17], 3, seed=2)
    pos, sys_ptr = pos.cuda(), sys_ptr.cuda()
    nbr, _, rev_ptr, rev_idx = ops.neighbor_list(pos, sys_ptr, 30, 5.0, 12)
    n, k = nbr.shape

    def ref(p):
        valid = (nbr >= 0).flatten()
        i = torch.arange(n, device=p.device).repeat_interleave(k)
        j = torch.where(valid, nbr.flatten().long(), (i + 1) % n)
        d = (p[j] - p[i]).norm(dim=-1)
        mu = torch.arange(16, device=p.device, dtype=p.dtype) * (5.0 / 15)
        rbf = torch.exp(-2.0 * (d[:, None] - mu) ** 2) * valid[:, None]
        env = 0.5 * (torch.cos(math.pi * d / 5.0) + 1) * (d < 5.0) * valid
        return rbf, env

    errs = twice_errors(lambda p: ops.edge_geom(p, nbr, rev_ptr, rev_idx, 16, 5.0, 2.0), ref, [pos])
    assert max(errs.values()) < 1e-4, errs
