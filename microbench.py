"""
Microbenchmarks of the hot kernels, timed with CUDA events.

    python microbench.py attn [--n 4096] [--iters 10] [--precision fp32|tf32]
    python microbench.py pooled [--n 8280] [--iters 10] [--precision tf32|fp32]
    python microbench.py gemm M N K [--silu]

``attn``: the masked edge-attention microbenchmark: n atoms x 8 heads x 32
tokens x 32 dims, fp32, q/k/v ~ N(0, 1), bias ~ N(0, 0.1) per (n, h, i, j),
keys j >= c_n masked with c_n ~ U{8..32}; forward1, backward1 and backward2,
each against its algorithmic bytes (every operand read or written once), in
the fp32 (three-term tf32 split) or tf32 (one tf32 product) precision.
``pooled``: the envelope-pooled token attention of the 85M model's blocks:
n atoms x 12 heads x k = 30 tokens x 64 dims gathered from per-atom rows,
keys masked past c_n ~ U{8..30}, forward / backward1 / backward2.
``gemm``: one tcgen05 tf32 GEMM shape (bias, optionally the SiLU epilogue).
"""

from __future__ import annotations

import argparse
import json
import os
import sys

import torch

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

from create_graph_b200.edge_attn import (
    attn_backward1,
    attn_backward2,
    attn_forward1,
    pooled_attention_backward1,
    pooled_attention_backward2,
    pooled_attention_forward,
    pooled_attention_out,
)
from create_graph_b200.gemm import ACT_SILU, gemm


def attn_inputs(n: int, h: int = 8, s: int = 32, d: int = 32, seed: int = 0, device: str = "cuda"):
    gen = torch.Generator().manual_seed(seed)
    q, k, v = (torch.randn(n, h, s, d, generator=gen).to(device) for _ in range(3))
    bias = (0.1 * torch.randn(n, h, s, s, generator=gen)).to(device)
    counts = torch.randint(8, s + 1, (n,), generator=gen, dtype=torch.int32).to(device)
    g, hq, hk, hv = (torch.randn(n, h, s, d, generator=gen).to(device) for _ in range(4))
    hb = torch.randn(n, h, s, s, generator=gen).to(device)
    return q, k, v, bias, counts, g, hq, hk, hv, hb, d**-0.5


def attn_algorithmic_bytes(n: int, h: int = 8, s: int = 32, d: int = 32) -> dict[str, int]:
    t, tb, lse = n * h * s * d * 4, n * h * s * s * 4, n * h * s * 4
    return {
        "fwd1": 3 * t + tb + t + lse,
        "bwd1": 4 * t + tb + lse + 3 * t + tb,
        "bwd2": 7 * t + 2 * tb + lse + 4 * t + tb,
    }


def _time(fn, iters: int, batches: int = 3) -> float:
    """Milliseconds per call: the median over `batches` of `iters` back-to-back
    calls between two CUDA events. Calls are queued without synchronising, so
    the Python work that prepares each launch overlaps the previous kernel
    and the figure is the kernels' device time (timing calls one at a time
    would add that host time whenever it exceeds the queue)."""
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    per_call = []
    for _ in range(batches):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(iters):
            fn()
        b.record()
        torch.cuda.synchronize()
        per_call.append(a.elapsed_time(b) / iters)
    return sorted(per_call)[len(per_call) // 2]


def attn(n: int = 4096, iters: int = 10, hbm_gbs: float | None = None, which=("fwd1", "bwd1", "bwd2"),
         precision: str = "fp32") -> dict:
    """Median launch time and achieved GB/s of each kernel at (n, 8, 32, 32)."""
    q, k, v, bias, counts, g, hq, hk, hv, hb, scale = attn_inputs(n)
    kw = {"precision": precision}
    _, lse = attn_forward1(q, k, v, bias, scale, counts, **kw)
    fns = {
        "fwd1": lambda: attn_forward1(q, k, v, bias, scale, counts, **kw),
        "bwd1": lambda: attn_backward1(q, k, v, bias, lse, g, scale, counts, **kw),
        "bwd2": lambda: attn_backward2(q, k, v, bias, lse, g, scale, hq, hk, hv, hb, counts, **kw),
    }
    nbytes = attn_algorithmic_bytes(n)
    out = {}
    for name in which:
        ms = _time(fns[name], iters)
        gbs = nbytes[name] / (ms / 1e3) / 1e9
        out[name] = {"us": ms * 1e3, "bytes": nbytes[name], "gb_s": gbs}
        if hbm_gbs:
            out[name]["frac"] = gbs / hbm_gbs
    return out


def pooled_inputs(n: int, h: int = 12, k: int = 30, d: int = 64, seed: int = 0):
    gen = torch.Generator().manual_seed(seed)
    qkv = torch.randn(n, 3 * h * d, generator=gen)
    bias = 0.1 * torch.randn(n * k, h, generator=gen)
    env = torch.rand(n * k, generator=gen)
    counts = torch.randint(8, k + 1, (n,), generator=gen, dtype=torch.int32)
    index = torch.randint(0, n, (n, k), generator=gen, dtype=torch.int32)
    index[torch.arange(k)[None, :] >= counts[:, None]] = -1
    dm, hqkv = torch.randn(n, h * d, generator=gen), torch.randn(n, 3 * h * d, generator=gen)
    hb, he = torch.randn(n * k, h, generator=gen), torch.randn(n * k, generator=gen)
    cuda = [t.cuda() for t in (qkv, bias, env, index.view(-1), counts, dm, hqkv, hb, he)]
    return cuda, k, h


def pooled(n: int = 8280, iters: int = 10, precision: str = "tf32", heads: int = 12, k: int = 30, d: int = 64) -> dict:
    """Median launch time of the pooled attention kernels (default: the 85M model's shape)."""
    (qkv, bias, env, index, counts, dm, hqkv, hb, he), k, h = pooled_inputs(n, heads, k, d)
    args = (index, counts, k, h, 0.125, precision)
    _, lse, w = pooled_attention_forward(qkv, bias, env, *args)
    fns = {
        "fwd": lambda: pooled_attention_forward(qkv, bias, env, *args),
        "bwd1": lambda: pooled_attention_backward1(qkv, bias, env, lse, w, dm, *args),
        "bwd2": lambda: pooled_attention_backward2(qkv, bias, env, lse, w, dm, hqkv, hb, he, *args),
        "out": lambda: pooled_attention_out(qkv, w, index, counts, k, h),
    }
    return {name: {"us": _time(fn, iters) * 1e3} for name, fn in fns.items()}


def gemm_bench(m: int, n: int, k: int, silu: bool = False, iters: int = 20, a_mn: bool = False,
               b_mn: bool = False) -> dict:
    """One shape; a_mn / b_mn store A as (k, m) / B as (k, n) (the weight-gradient layouts)."""
    a = torch.randn(k, m, device="cuda") if a_mn else torch.randn(m, k, device="cuda")
    b = torch.randn(k, n, device="cuda") if b_mn else torch.randn(n, k, device="cuda")
    bias = torch.randn(n, device="cuda")
    kw = {"bias": bias, "a_t": a_mn, "b_t": b_mn}
    if silu:
        kw.update(act=ACT_SILU, aux_out=torch.empty(m, n, device="cuda"))
    ms = _time(lambda: gemm(a, b, **kw), iters)
    return {"shape": [m, n, k], "silu": silu, "a_mn": a_mn, "b_mn": b_mn, "us": ms * 1e3,
            "tflops": 2 * m * n * k / (ms / 1e3) / 1e12}


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    sub = parser.add_subparsers(dest="what", required=True)
    p_attn = sub.add_parser("attn")
    p_attn.add_argument("--n", type=int, default=4096)
    p_attn.add_argument("--iters", type=int, default=10)
    p_attn.add_argument("--precision", choices=("fp32", "tf32"), default="fp32")
    p_pool = sub.add_parser("pooled")
    p_pool.add_argument("--n", type=int, default=8280)
    p_pool.add_argument("--iters", type=int, default=10)
    p_pool.add_argument("--precision", choices=("fp32", "tf32"), default="tf32")
    p_pool.add_argument("--heads", type=int, default=12)
    p_pool.add_argument("--k", type=int, default=30)
    p_pool.add_argument("--d", type=int, default=64)
    p_gemm = sub.add_parser("gemm")
    p_gemm.add_argument("shape", type=int, nargs=3)
    p_gemm.add_argument("--silu", action="store_true")
    p_gemm.add_argument("--a-mn", action="store_true", help="A stored (k, m)")
    p_gemm.add_argument("--b-mn", action="store_true", help="B stored (k, n)")
    args = parser.parse_args()
    if args.what == "attn":
        print(json.dumps(attn(args.n, args.iters, precision=args.precision)))
    elif args.what == "pooled":
        print(json.dumps(pooled(args.n, args.iters, args.precision, args.heads, args.k, args.d)))
    else:
        print(json.dumps(gemm_bench(*args.shape, silu=args.silu, a_mn=args.a_mn, b_mn=args.b_mn)))


if __name__ == "__main__":
    main()
