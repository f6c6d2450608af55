"""
Data parallelism on CPU ranks (gloo, 2 processes, float64): each rank runs
cg.create_graph on its own systems, gradients live in one flat buffer
(create_graph_b200.ddp.FlatGradients) whose buckets are averaged by
all-reduces launched from inside loss.backward() as their gradients complete.
The reduced gradients must be identical on both ranks and equal the mean of
the per-rank eager create_graph gradients -- the property the reference's DDP
test asserts (tests/test_ddp.py there) -- for one bucket and for buckets of a
single parameter, and with small buckets some all-reduces must have started
before backward returned. A second case has one rank raise before its first
collective and checks the other fails with an error instead of waiting
forever. A third case checkpoints the layers (memory budget 0.5) with ops that
take part in the deferred first-order backward: each parameter's gradient
still completes once, so the same buckets and averages follow.
"""

from __future__ import annotations

import os
import socket
import tempfile
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp
from torch import nn

import create_graph_b200 as cg
from create_graph_b200.checkpoint import cut_forward_tensor, deferral_slot, deferred_cotangent, plus
from create_graph_b200.ddp import FlatGradients

pytestmark = [pytest.mark.ddp, pytest.mark.slow]


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.layers = nn.ModuleList(nn.Linear(32, 32) for _ in range(3))
        self.inp, self.out = nn.Linear(4, 32), nn.Linear(32, 1)
        self.region = cg.compile(self._energy)

    def _energy(self, vec, dist):
        h = torch.tanh(self.inp(torch.cat([vec, dist[:, None]], dim=-1)))
        for layer in self.layers:
            h = h + nn.functional.silu(layer(h))
        return self.out(h).sum().reshape(1)

    def forward(self, data):
        vec = data["pos"][data["src"]] - data["pos"][data["dst"]]
        return {"energy": self.region(vec, vec.norm(dim=-1))}


class TanhResidual(torch.autograd.Function):
    """x + tanh(x @ w.T), its backward from torch ops, with the deferral hooks."""

    @staticmethod
    def forward(ctx, x, w):
        ctx.op = deferral_slot()
        ctx.save_for_backward(x, w)
        return x + torch.tanh(x @ w.t())

    @staticmethod
    def backward(ctx, g):
        x, w = ctx.saved_tensors
        c = deferred_cotangent(ctx, "x")
        x = cut_forward_tensor(ctx, "x", x)
        t = torch.tanh(x @ w.t())
        u = g * (1 - t * t)
        return plus(g + u @ w, c), u.t() @ x


class DeferBlock(nn.Module):
    def __init__(self, width):
        super().__init__()
        self.w1 = nn.Parameter(torch.randn(width, width) / width**0.5)
        self.w2 = nn.Parameter(torch.randn(width, width) / width**0.5)

    def forward(self, h):
        return TanhResidual.apply(TanhResidual.apply(h, self.w1), self.w2)


class CheckpointedNet(Net):
    def __init__(self):
        super().__init__()
        self.layers = nn.ModuleList(DeferBlock(32) for _ in range(3))
        config = cg.CompileConfig(backend="eager", checkpoint=r"layers\.\d+", memory_budget=0.5)
        self.region = cg.compile(self._energy, config=config)


MODELS = {"plain": Net, "checkpointed": CheckpointedNet}


def rank_data(rank):
    gen = torch.Generator().manual_seed(100 + rank)
    n = 9
    src = torch.randint(0, n, (24,), generator=gen)
    return {
        "pos": torch.randn(n, 3, generator=gen, dtype=torch.float64),
        "src": src,
        "dst": (src + torch.randint(1, n, (24,), generator=gen)) % n,
    }


def step(model, data, exact=False, fail=False):
    out, grads = cg.create_graph(model, data, exact=exact)
    if fail:
        raise RuntimeError("injected failure before the all-reduce")
    (out["energy"].sum() + grads["pos"].square().sum()).backward()


def worker(rank, world, port, path, fail_rank, bucket_bytes, model_name="plain"):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    torch.set_default_dtype(torch.float64)
    torch.manual_seed(0)
    model = MODELS[model_name]()
    grads = FlatGradients(model.parameters(), world, bucket_bytes=bucket_bytes)
    try:
        for _ in range(2):  # a second step reuses the hooks and buckets
            grads.zero()
            step(model, rank_data(rank), fail=rank == fail_rank)
            in_backward = grads.launched_in_backward
            grads.allreduce()
        whole = grads.flat.clone()
        gathered = [torch.empty_like(whole) for _ in range(world)]
        dist.all_gather(gathered, whole)
        # the parameters' gradients (each slice starts on a 256-byte boundary; the gaps stay zero)
        flat = torch.cat([p.grad.flatten() for p in grads.params])
        gaps = whole.clone()
        for start, n in grads.offsets:
            gaps[start : start + n] = 0
        aligned = all((p.grad.data_ptr() - grads.flat.data_ptr()) % 256 == 0 for p in grads.params)
        if rank == 0:
            torch.save({"flat": flat, "identical": all(torch.equal(gathered[0], g) for g in gathered[1:]),
                        "buckets": len(grads.buckets), "in_backward": in_backward,
                        "gaps_zero": bool((gaps == 0).all()), "aligned": aligned}, path)
    except RuntimeError as error:
        torch.save({"error": str(error)}, f"{path}.{rank}")
    finally:
        try:
            dist.destroy_process_group()
        except Exception:  # noqa: BLE001 - the group may already be broken
            pass


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def expected_flat(model_name="plain"):
    torch.set_default_dtype(torch.float64)
    try:
        torch.manual_seed(0)
        model = MODELS[model_name]()
        total = None
        for rank in range(2):
            model.zero_grad()
            step(model, rank_data(rank), exact=True)
            flat = torch.cat([p.grad.flatten() for p in model.parameters()])
            total = flat if total is None else total + flat
        return total / 2
    finally:
        torch.set_default_dtype(torch.float32)


@pytest.mark.parametrize("bucket_bytes", [1 << 30, 1])
def test_averaged_gradients_match_eager_mean(bucket_bytes):
    want = expected_flat()
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "out.pt")
        mp.spawn(worker, args=(2, free_port(), path, -1, bucket_bytes), nprocs=2, join=True)
        got = torch.load(path)
    assert got["identical"] and got["gaps_zero"] and got["aligned"]
    assert ((got["flat"] - want).norm() / want.norm()).item() < 1e-10
    if bucket_bytes == 1:  # one bucket per parameter: most start inside backward
        assert got["buckets"] == 10
        assert got["in_backward"] >= 5


def test_failing_rank_ends_the_other_with_an_error():
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "out.pt")
        mp.spawn(worker, args=(2, free_port(), path, 1, 1), nprocs=2, join=True)
        assert "injected failure" in torch.load(f"{path}.1")["error"]
        # rank 0 is left alone in the collective: gloo ends it with an error, not a hang
        assert os.path.exists(f"{path}.0")


def test_checkpointed_layers_with_deferred_backward():
    want = expected_flat("checkpointed")
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "out.pt")
        mp.spawn(worker, args=(2, free_port(), path, -1, 1, "checkpointed"), nprocs=2, join=True)
        got = torch.load(path)
    assert got["identical"] and got["gaps_zero"] and got["aligned"]
    assert ((got["flat"] - want).norm() / want.norm()).item() < 1e-10
    assert got["buckets"] == 10 and got["in_backward"] >= 5
