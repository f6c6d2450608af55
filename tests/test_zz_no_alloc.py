"""
cg_gemm_tf32_noalloc: the GEMM entry point for callers that cannot allocate
device memory (their device memory belongs to another allocator and they
forbid cudaMalloc). Called through the C ABI on shapes that split K (so the
static scratch buffer is used) and on one that does not (no scratch at all);
each result must match the allocating entry point cg_gemm_tf32 and a float64
torch product within the tf32 tolerance of the GEMM tests, on two calls in a
row (the second call reuses the scratch the first one left behind). A shape
needing more than the static buffer is refused.

Kept in a file of its own that pytest collects last.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from create_graph_b200 import native
from create_graph_b200.gemm import gemm

pytestmark = pytest.mark.gpu
TF32_TOL = 3e-3


def rel(a, b):
    a, b = a.double(), b.double()
    return ((a - b).norm() / b.norm()).item()


def gemm_args(a_t: torch.Tensor, b_t: torch.Tensor, bias: torch.Tensor, out: torch.Tensor) -> native.GemmArgs:
    k, m = a_t.shape
    n = b_t.shape[1]
    args = native.GemmArgs()
    args.m, args.n, args.k = m, n, k
    args.a, args.lda = a_t.data_ptr(), a_t.stride(0)
    args.b, args.ldb = b_t.data_ptr(), b_t.stride(0)
    args.c, args.ldc = out.data_ptr(), out.stride(0)
    args.bias = bias.data_ptr()
    args.a_mn_major, args.b_mn_major = 1, 1
    args.alpha = 1.0
    return args


def noalloc_gemm(a_t: torch.Tensor, b_t: torch.Tensor, bias: torch.Tensor) -> torch.Tensor:
    """a_t (K, M) and b_t (K, N) read MN-major: out = a_t.T @ b_t + bias."""
    out = torch.empty(a_t.shape[1], b_t.shape[1], device=a_t.device)
    args = gemm_args(a_t, b_t, bias, out)
    native.check(native.lib().cg_gemm_tf32_noalloc(ctypes.byref(args), native.stream_ptr(a_t.device)))
    return out


# (m, n, k, splits K): the first three use the static scratch, the last none
@pytest.mark.parametrize(
    "mnk, split", [((12, 128, 50000), True), ((128, 12, 250000), True), ((300, 200, 1000), True),
                   ((1024, 1024, 128), False)])
def test_noalloc_matches_allocating_entry_point_twice(mnk, split):
    m, n, k = mnk
    gen = torch.Generator().manual_seed(11)
    a_host = torch.randn(k, m, generator=gen)
    b_host = torch.randn(k, n, generator=gen)
    bias_host = torch.randn(n, generator=gen)
    a_t, b_t, bias = a_host.cuda(), b_host.cuda(), bias_host.cuda()
    probe = gemm_args(a_t, b_t, bias, torch.empty(1, device="cuda"))
    need = native.lib().cg_gemm_workspace_bytes(ctypes.byref(probe))
    assert (need > 0) == split, need
    want = gemm(a_t, b_t, a_t=True, b_t=True, bias=bias)
    exact = a_host.double().T @ b_host.double() + bias_host.double()
    for _ in range(2):
        got = noalloc_gemm(a_t, b_t, bias)
        torch.cuda.synchronize()
        assert rel(got, want) < TF32_TOL
        assert rel(got.cpu(), exact) < TF32_TOL
    assert native.device_error() == 0


def test_noalloc_refuses_shapes_beyond_its_scratch():
    m, n, k = 768, 768, 8280  # splits K into more than 8 MiB of partial tiles
    a_t = torch.zeros(k, m, device="cuda")
    b_t = torch.zeros(k, n, device="cuda")
    with pytest.raises(native.NativeError, match="static buffer"):
        noalloc_gemm(a_t, b_t, torch.zeros(n, device="cuda"))
