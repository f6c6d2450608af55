"""
The reference's algorithm for one conservative-force training step, on CPU.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). The reference computes
forces as eager ``torch.autograd.grad(E.sum(), pos, create_graph=True)``
(``create_graph(..., exact=True)``, src/create_graph/api.py:200-211 there) and
the parameter gradients with one ``loss.backward()``
(src/create_graph/testing.py:68-84 there). This module does exactly that over
plain torch CPU ops, on the model spec of create_graph_b200/mlip.py restated
op by op (LayerNorm, Linear, SiLU, a masked softmax attention with the
-inf-safe masking of kernels/edge_attn/ops.py:26-34, index_add segment sums),
with the neighbour lists of oracle/neighbors.py. It is the parity oracle of
the GPU step and the timed CPU baseline of bench.py.
"""

from __future__ import annotations

import math

import numpy as np
import torch
import torch.nn.functional as F

from oracle.neighbors import neighbor_list


def geometry(pos, nbr, n_rbf, cutoff, gamma):
    n, k = nbr.shape
    valid = (nbr >= 0).reshape(-1)
    i = torch.arange(n).repeat_interleave(k)
    j = torch.where(valid, nbr.reshape(-1).long(), (i + 1) % max(n, 1))  # padded slots kept finite
    vec = pos[j] - pos[i]
    d = vec.norm(dim=-1)
    mu = torch.arange(n_rbf, dtype=pos.dtype) * (cutoff / (n_rbf - 1))
    rbf = torch.exp(-gamma * (d[:, None] - mu) ** 2) * valid[:, None]
    env = 0.5 * (torch.cos(math.pi * d / cutoff) + 1) * (d < cutoff) * valid
    return rbf, env, valid, j


def masked_attention(tok, bias, counts, heads, scale, n, k):
    """Attention among the k tokens of each atom, keys >= counts masked; rows
    with no valid key give zeros."""
    c3 = tok.shape[1]
    d = c3 // (3 * heads)
    t = tok.view(n, k, 3, heads, d)
    q, kk, v = (t[:, :, p].permute(0, 2, 1, 3) for p in range(3))
    b = bias.view(n, k, heads).permute(0, 2, 1)[:, :, None, :]
    keymask = torch.arange(k)[None, :] >= counts[:, None].long()  # (n, k)
    logits = torch.matmul(q, kk.transpose(-1, -2)) * scale + b
    logits = logits.masked_fill(keymask[:, None, None, :], -torch.inf)
    row_ok = (~keymask).any(dim=-1)[:, None, None, None]
    safe = torch.where(row_ok, logits, torch.zeros_like(logits))
    p = torch.softmax(safe, dim=-1) * row_ok
    return torch.matmul(p, v).permute(0, 2, 1, 3).reshape(n, k, heads * d)


def energy(params: dict, spec, pos, species, sys_ptr, nbr, counts):
    """Per-system energies; params are the GPU model's state_dict entries."""
    p = lambda name: params[f"network.{name}"]  # noqa: E731
    n, k = nbr.shape
    rbf, env, valid, j = geometry(pos, nbr, spec.n_rbf, spec.cutoff, spec.rbf_gamma)
    h = p("embed")[species.long()]
    scale = 1.0 / math.sqrt(spec.head_dim)
    w_bias, b_bias = p("rbf_bias.weight"), p("rbf_bias.bias")  # block b: rows b*H .. (b+1)*H - 1
    H = spec.heads
    for b in range(spec.blocks):
        q = lambda name, b=b: p(f"blocks.{b}.{name}")  # noqa: E731
        x = F.layer_norm(h, (spec.hidden,), q("norm1.weight"), q("norm1.bias"), 1e-5)
        qkv = F.linear(x, q("qkv.weight"), q("qkv.bias"))
        tok = qkv[j] * valid[:, None]
        bias = F.linear(rbf, w_bias[b * H:(b + 1) * H], b_bias[b * H:(b + 1) * H])
        o = masked_attention(tok, bias, counts, spec.heads, scale, n, k)
        m = (env.view(n, k, 1) * o).sum(1)
        h = h + F.linear(m, q("out.weight"), q("out.bias"))
        x = F.layer_norm(h, (spec.hidden,), q("norm2.weight"), q("norm2.bias"), 1e-5)
        h = h + F.linear(F.silu(F.linear(x, q("ffn1.weight"), q("ffn1.bias"))), q("ffn2.weight"), q("ffn2.bias"))
    x = F.layer_norm(h, (spec.hidden,), p("norm.weight"), p("norm.bias"), 1e-5)
    e_atom = F.linear(x, p("readout.weight"), p("readout.bias"))[:, 0]
    sys_idx = torch.repeat_interleave(torch.arange(len(sys_ptr) - 1), torch.diff(sys_ptr.long()))
    return torch.zeros(len(sys_ptr) - 1, dtype=pos.dtype).index_add(0, sys_idx, e_atom)


def train_step(params: dict, spec, pos, species, sys_ptr, e_target, f_target, graph=None):
    """Energy, forces, loss and parameter gradients of one step (eager create_graph).

    ``params``: name -> tensor (CPU, any float dtype; copied as leaves).
    ``graph``: (nbr, counts) from oracle.neighbors, or None to build it.
    """
    dtype = next(iter(params.values())).dtype
    if graph is None:
        nbr, counts, _, _ = neighbor_list(pos.float().numpy(), np.asarray(sys_ptr), spec.cutoff, spec.k)
        graph = (torch.from_numpy(nbr), torch.from_numpy(counts))
    nbr, counts = graph
    leaves = {name: t.detach().to(dtype).clone().requires_grad_(True) for name, t in params.items()}
    x = pos.detach().to(dtype).clone().requires_grad_(True)
    e = energy(leaves, spec, x, species, sys_ptr, nbr, counts)
    (g,) = torch.autograd.grad(e.sum(), x, create_graph=True)
    forces = -g
    loss = (e - e_target.to(dtype)).square().mean() + (forces - f_target.to(dtype)).square().mean()
    loss.backward()
    grads = {name: (t.grad if t.grad is not None else torch.zeros_like(t)) for name, t in leaves.items()}
    return {"energy": e.detach(), "forces": forces.detach(), "loss": loss.detach(), "grads": grads}
