"""
The tcgen05 GEMM of the dense projections (``cg_gemm_tf32``), on torch tensors.

``gemm(a, b)`` computes ``a @ b.T`` for a (M, K) and b (N, K); ``a_t=True``
takes ``a`` as (K, M) and ``b_t=True`` takes ``b`` as (K, N), read in place
(MN-major operands), so x W^T, g W and g^T x need no transposed copies.
Arithmetic: fp32 accumulation of tf32 products. ``precision="tf32"`` makes
one product of tf32-rounded operands; ``precision="fp32"`` splits every
operand into two tf32 terms on chip and accumulates three products
(fp32-level accuracy, a third of the tf32 rate). Without an explicit
argument the precision is the calling thread's current one
(``gemm_precision``), "tf32" by default.

Operands need 16-byte aligned bases and row pitches (the TMA rule); bases on
256-byte boundaries, as separate allocations have, keep each 128-byte TMA row
within one cache line: weights viewed at 16-byte offsets into a shared buffer
measured 20% slower on the model's GEMMs (ddp.FlatGradients and
optim.FusedAdamW lay their flat buffers out on 256-byte boundaries for this).
"""

from __future__ import annotations

import contextlib
import ctypes
import threading

import torch
from torch import Tensor

from create_graph_b200 import native
from create_graph_b200.errors import NativeError

ACT_NONE, ACT_SILU, ACT_SILU_GRAD, ACT_ADD = native.ACT_NONE, native.ACT_SILU, native.ACT_SILU_GRAD, native.ACT_ADD
PRECISIONS = {"tf32": native.GEMM_TF32, "fp32": native.GEMM_FP32}

_THREAD = threading.local()


def current_precision() -> str:
    """The GEMM precision of the calling thread ("tf32" unless set)."""
    return getattr(_THREAD, "precision", "tf32")


@contextlib.contextmanager
def gemm_precision(precision: str):
    """Run the GEMMs of this thread at ``precision`` ("tf32" or "fp32") inside
    the block. Fused ops record the precision of their forward and re-enter it
    in their backward, which autograd runs on its own threads."""
    if precision not in PRECISIONS:
        raise NativeError(f"gemm precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
    before = current_precision()
    _THREAD.precision = precision
    try:
        yield
    finally:
        _THREAD.precision = before


def _operand(t: Tensor, name: str) -> Tensor:
    if t.dtype != torch.float32:
        raise NativeError(f"gemm: {name} must be float32, got {t.dtype}")
    if t.dim() != 2:
        raise NativeError(f"gemm: {name} must be 2-D, got {tuple(t.shape)}")
    if t.stride(1) != 1 or t.stride(0) % 4 != 0 or t.data_ptr() % 16 != 0 or t.stride(0) < t.shape[1]:
        t = t.contiguous()
        if t.shape[1] % 4 != 0:
            pitch = (t.shape[1] + 3) // 4 * 4
            padded = torch.zeros(t.shape[0], pitch, dtype=t.dtype, device=t.device)
            padded[:, : t.shape[1]] = t
            t = padded[:, : t.shape[1]]
    return t


def gemm(
    a: Tensor,
    b: Tensor,
    *,
    a_t: bool = False,
    b_t: bool = False,
    bias: Tensor | None = None,
    act: int = ACT_NONE,
    aux_in: Tensor | None = None,
    aux_out: Tensor | None = None,
    out: Tensor | None = None,
    accumulate: bool = False,
    alpha: float = 1.0,
    precision: str | None = None,
) -> Tensor:
    native.require_cuda(a, b, bias, aux_in, aux_out, out)
    a = _operand(a, "a")
    b = _operand(b, "b")
    m, k = (a.shape[1], a.shape[0]) if a_t else (a.shape[0], a.shape[1])
    n, kb = (b.shape[1], b.shape[0]) if b_t else (b.shape[0], b.shape[1])
    if k != kb:
        raise NativeError(f"gemm: inner dimensions differ ({k} vs {kb})")
    if out is None:
        if accumulate:
            raise NativeError("gemm: accumulate needs out")
        out = torch.empty(m, n, dtype=torch.float32, device=a.device)
    if out.shape != (m, n) or out.stride(1) != 1:
        raise NativeError(f"gemm: out must be ({m}, {n}) with unit column stride")
    if k == 0:
        if not accumulate:
            out.zero_()
        return out
    args = native.GemmArgs()
    args.m, args.n, args.k = m, n, k
    args.a, args.lda = a.data_ptr(), a.stride(0)
    args.b, args.ldb = b.data_ptr(), b.stride(0)
    args.c, args.ldc = out.data_ptr(), out.stride(0)
    if bias is not None:
        bias = bias.contiguous()
        args.bias = bias.data_ptr()
    auxes = [t for t in (aux_in, aux_out) if t is not None]
    for aux in auxes:
        if aux.shape != (m, n) or aux.stride(1) != 1 or aux.stride(0) != auxes[0].stride(0):
            raise NativeError(f"gemm: aux_in / aux_out must be ({m}, {n}) with unit column stride and one row pitch")
    if auxes:
        args.ld_aux = auxes[0].stride(0)
    args.aux_in = None if aux_in is None else aux_in.data_ptr()
    args.aux_out = None if aux_out is None else aux_out.data_ptr()
    args.a_mn_major, args.b_mn_major = int(a_t), int(b_t)
    args.act, args.accumulate, args.alpha = act, int(accumulate), float(alpha)
    precision = current_precision() if precision is None else precision
    if precision not in PRECISIONS:
        raise NativeError(f"gemm: precision must be one of {sorted(PRECISIONS)}, got {precision!r}")
    args.precision = PRECISIONS[precision]
    ws_bytes = native.lib().cg_gemm_workspace_bytes(ctypes.byref(args))
    workspace = None
    if ws_bytes > 0:
        workspace = torch.empty(ws_bytes // 4, dtype=torch.float32, device=a.device)
        args.workspace, args.workspace_bytes = workspace.data_ptr(), ws_bytes
    native.invoke("cg_gemm_tf32", ctypes.byref(args), native.stream_ptr(a.device), info=(m, n, k, precision))
    return out
