"""
Differentiable torch restatements used as ``check_op`` references.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). ``attention`` is the
reference's oracle kernels/edge_attn/reference.py:8-11: the same attention
from ordinary differentiable torch ops (logits, logsumexp, softmax, matmul).
"""

from __future__ import annotations

import torch


def attention(q, k, v, bias, scale: float):
    logits = torch.matmul(q, k.transpose(-2, -1)) * scale + bias
    lse = torch.logsumexp(logits, dim=-1)
    return torch.matmul(torch.softmax(logits, dim=-1), v), lse
