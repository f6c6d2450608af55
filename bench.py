"""
Energy + force training-step throughput (atoms/s) of the 85M-parameter
edge-attention MLIP on B200s, data-parallel weak scaling.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

Workload: per rank ~8192 atoms as random systems of U{20..200} atoms at 0.1
atoms/A^3 (seed 1000 + rank), 12 blocks, hidden 768, 12 heads, FFN 3072,
128-Gaussian RBF, cutoff 6 A, k <= 30 neighbours, 50 species, tf32 GEMMs with
fp32 accumulation, CompileConfig(memory_budget=0.5, checkpoint=r"blocks\\.\\d+").
A step is one cg.create_graph call (energy + forces), the MSE loss on both and
loss.backward() (the parameter gradient through the force), one NCCL average
of the fp32 gradients for N > 1, and an AdamW update of the parameters (one
fused kernel; torch.optim.AdamW on the reference arm). Synthetic data,
random-init weights.

Rank 0 prints one JSON line. ``--impl reference`` times the reference's
algorithm for the same step (eager create_graph over torch CPU ops, the
oracle in oracle/step.py) on the host cores, on a bounded sample per step.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

ATOMS_PER_RANK = 8192
METRIC = "energy+force train-step atoms/s"
CONFIG_NAME = "allscaip_85m"


def env_rank():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            p = json.load(f)
        return p["hbm_gbs"], p["bf16_tflops"], p.get("bf16_tflops_sustained", p["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [line for line in out.splitlines() if line.strip()]

    def summary(self):
        sm, sm_max, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                sm_max = max(sm_max, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": sm_max or None,
            "reasons": sorted(reasons),
            "samples": len(sm),
        }


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------


def run_mine(args):
    import torch.distributed as dist

    import create_graph_b200 as cg
    from create_graph_b200 import mlip, native
    from create_graph_b200.ddp import FlatGradients
    from create_graph_b200.optim import FusedAdamW
    from create_graph_b200.graph import make_batch

    rank, world, local = env_rank()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=300))
    spec = mlip.SPECS[CONFIG_NAME]
    sizes = mlip.workload_sizes(CONFIG_NAME, seed=1000 + rank, atoms_target=args.atoms)
    pos_h, species_h, sys_ptr_h = mlip.synthetic_systems(sizes, spec.n_species, seed=1000 + rank)
    e_t_h, f_t_h = mlip.make_targets(len(sizes), pos_h.shape[0], seed=2000 + rank)
    n_atoms = pos_h.shape[0]

    torch.manual_seed(0)  # identical initial weights on every rank
    config = cg.CompileConfig(memory_budget=0.5, checkpoint=r"blocks\.\d+")
    model = mlip.MLIP(spec, config=config).to(dev)
    grads = FlatGradients(model.parameters(), world if world > 1 else None)
    opt = FusedAdamW(grads, **ADAMW)
    batch = make_batch(pos_h.to(dev), species_h.to(dev), sys_ptr_h.to(dev), spec.n_species)
    e_t, f_t = e_t_h.to(dev), f_t_h.to(dev)

    def step(b, et, ft):
        grads.zero()
        loss = mlip.train_step(model, b, et, ft)
        grads.allreduce()
        opt.step()
        return loss

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: int) -> int:
        if world == 1:
            return x
        t = torch.tensor([x], device=dev, dtype=torch.int64)
        dist.all_reduce(t)
        return int(t.item())

    for _ in range(args.warmup):
        step(batch, e_t, f_t)
    torch.cuda.synchronize()

    # ---- device-resident throughput ----
    torch.cuda.reset_peak_memory_stats(dev)
    launches0 = native.launch_count()
    with ClockSampler(local) as clocks:
        barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(args.steps):
            loss = step(batch, e_t, f_t)
        end.record()
        torch.cuda.synchronize()
        barrier()
    launches = native.launch_count() - launches0
    peak_gb = max_over_ranks(torch.cuda.max_memory_allocated(dev) / 1e9)
    ms = max_over_ranks(start.elapsed_time(end)) / args.steps
    total_atoms = sum_over_ranks(n_atoms)
    value = total_atoms / (ms / 1e3)

    # ---- end to end through the public API, host buffers each step ----
    pin = lambda t: t.pin_memory()  # noqa: E731
    host = [pin(t) for t in (pos_h, species_h, sys_ptr_h, e_t_h, f_t_h)]
    h2d = sum(t.numel() * t.element_size() for t in host)
    barrier()
    torch.cuda.synchronize()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        pos, species, sys_ptr, et, ft = (t.to(dev, non_blocking=True) for t in host)
        b = make_batch(pos, species, sys_ptr, spec.n_species)
        loss_host = step(b, et, ft).to("cpu")
    e_end.record()
    torch.cuda.synchronize()
    barrier()
    e_ms = max_over_ranks(e_start.elapsed_time(e_end)) / args.steps
    e2e = {
        "value": total_atoms / (e_ms / 1e3),
        "unit": "atoms/s",
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": loss_host.numel() * loss_host.element_size(),
    }

    # ---- kernel breakdown (instrumented steps after the timed region) ----
    kernels = kernel_breakdown(native, lambda: step(batch, e_t, f_t), dev)

    if rank == 0:
        hbm, bf16, bf16_sus, src = peaks()
        roofline = roofline_of(kernels, hbm, bf16, bf16_sus, src)
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "atoms/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms,
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32 (tf32 tensor-core products in the GEMMs and the edge attention, fp32 accumulation)",
            "data": "synthetic (seeded random systems, random-init weights)",
            "config": {
                "workload": f"{CONFIG_NAME}: ~{args.atoms} atoms/GPU as systems of U{{20..200}} atoms, "
                            "12 blocks, C 768, 12 heads, FFN 3072, 128 RBF, k<=30, memory_budget 0.5, "
                            "per-block checkpoint; step = energy + forces + loss.backward() + AdamW update",
                "atoms_per_step": total_atoms,
                "systems_rank0": len(sizes),
                "parallelism": f"dp{world}",
                "allreduce": (f"{len(grads.buckets)} buckets (<= 64 MiB) of the flat fp32 gradients, NCCL "
                              "all-reduce launched from backward hooks" if world > 1 else "none (1 rank)"),
                "l2": "working set of several GB per step (larger than L2)",
            },
            "e2e": e2e,
            "gpu_launches": launches,
            # torch.cuda.max_memory_allocated over the timed steps (max over ranks):
            # parameters, gradients, AdamW moments and the step's activations
            "peak_memory_gb": peak_gb,
            "roofline": roofline,
            # the GEMM entry point as a whole (every shape of the step) against the tf32 peak
            "roofline_gemm": (_gemm_roofline(kernels["cg_gemm_tf32"]["calls"], bf16_sus, src)
                              if "cg_gemm_tf32" in kernels else None),
            "kernels": {k: {"launches": v["launches"], "ms_per_step": v["ms"], "share": v["share"]}
                        for k, v in sorted(kernels.items(), key=lambda kv: -kv[1]["ms"])},
            "clocks": clocks.summary(),
            "loss": float(loss.item()),
        }
        # the metric's second part: edge-attention backward2 against its HBM roofline at the
        # microbenchmark shape (4096 atoms x 8 heads x 32 tokens x 32 dims, fp32 storage), in the
        # tf32 precision the model runs (headline) and the fp32 (three-term split) precision
        from create_graph_b200 import microbench

        line["edge_attn_bwd2"] = {"shape": "(4096, 8, 32, 32) fp32, keys masked past U{8..32}"}
        for prec in ("tf32", "fp32"):
            mb = microbench.attn(4096, iters=10, hbm_gbs=hbm, which=("bwd2",), precision=prec)["bwd2"]
            traffic = EDGE_BWD2_TRAFFIC_PER_ATOM * 4096 if prec == "tf32" else None
            entry = {"bound": "hbm", "achieved": mb["gb_s"], "peak": hbm, "unit": "GB/s",
                     "frac": mb["gb_s"] / hbm, "traffic": traffic, "algorithmic_bytes": mb["bytes"],
                     "us_per_launch": mb["us"], "peak_source": f"{src} hbm_gbs", "precision": prec}
            line["edge_attn_bwd2"]["roofline" if prec == "tf32" else "roofline_fp32"] = entry
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline(spec, sizes, pos_h, species_h, sys_ptr_h, e_t_h, f_t_h, model)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def kernel_breakdown(native, step, dev, n_steps=1):
    """Per entry point: launches, device time per step (CUDA events around each
    launch on its stream) and share of the instrumented step."""
    names = [n for n in native.exported_symbols() if n.startswith("cg_") and n not in
             ("cg_last_error", "cg_version", "cg_launch_count", "cg_device_error") and
             not n.endswith("_bytes") and not n.endswith("_workspace")]
    native.time_entry_points(names)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(n_steps):
        step()
    t1.record()
    torch.cuda.synchronize()
    total = t0.elapsed_time(t1) / n_steps
    out = {}
    for name in names:
        rec = native.TIMED.get(name, [])
        if not rec:
            continue
        ms = sum(a.elapsed_time(b) for a, b, _ in rec) / n_steps
        out[name] = {"launches": len(rec) // n_steps, "ms": ms, "share": ms / total, "calls": rec}
    native.time_entry_points(names, enable=False)
    return out


def attn_bytes(info, name):
    """Algorithmic bytes of one token-layout attention launch (each operand once)."""
    n, h, k, d = info
    t = n * k * h * d * 4       # one (n, k, C) fp32 tensor
    b = n * k * h * 4           # bias (n*k, h)
    lse = n * h * k * 4
    if name == "cg_edge_attn_fwd1":
        return 3 * t + b + t + lse
    if name == "cg_edge_attn_bwd1":
        return 3 * t + b + lse + t + 3 * t + b
    return 3 * t + b + lse + t + 3 * t + b + 3 * t + b + t


# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) per atom of one ncu
# capture of each kernel at a smaller size; traffic grows with the atoms a launch
# processes, so a launch's traffic is this figure times its atoms.
TRAFFIC_PER_ATOM = {
    "cg_pooled_attn_bwd1": (53.767680e6 + 329.964032e6) / 2048,  # 12 heads x 30 tokens x 64 dims, tf32
}
# the edge-attention backward2 microbenchmark kernel, 8 heads x 32 tokens x 32 dims, tf32
EDGE_BWD2_TRAFFIC_PER_ATOM = (303.211264e6 + 133.112064e6) / 1024


def pooled_attn_bytes(info, name):
    """Algorithmic bytes of one pooled-attention launch: every per-atom operand
    once (the gathered token rows are re-reads of the atom rows), plus the
    per-token [dq | dk] rows the backward kernels must write."""
    n, h, k, d = info
    C = h * d
    atom, key, tok = n * C * 4, n * k * h * 4, n * k * 4   # one (n, C), (n*k, h), (n*k) tensor
    stats = 2 * n * h * k * 4                              # lse and w
    if name == "cg_pooled_attn_fwd":
        return 3 * atom + key + tok + atom + stats
    dqk = 2 * n * k * C * 4
    if name == "cg_pooled_attn_bwd1":
        return 3 * atom + key + tok + stats + atom + dqk + 2 * key + tok
    return 6 * atom + 2 * key + 2 * tok + stats + atom + dqk + 2 * key + tok + atom


def _gemm_roofline(rec, bf16_sus, src, name="cg_gemm_tf32"):
    flops = sum(2 * m * n * k for _, _, (m, n, k) in rec)
    secs = sum(a.elapsed_time(b) for a, b, _ in rec) / 1e3
    achieved = flops / secs / 1e12
    peak = bf16_sus / 2
    return {"kernel": name, "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
            "frac": achieved / peak, "traffic": None, "peak_source": f"{src} bf16 sustained / 2 (dense tf32)"}


def roofline_of(kernels, hbm, bf16, bf16_sus, src):
    """Roofline of the dominant kernel: the one kernel with the most device time
    per step. The GEMM entry point runs a different kernel per shape (tile width,
    operand majors, split), so its launches compete shape by shape; the HBM-bound
    attention kernels are one kernel each."""
    if not kernels:
        return None
    candidates = {}
    for name, info in kernels.items():
        if name == "cg_gemm_tf32":
            shapes = {}
            for call in info["calls"]:
                shapes.setdefault(call[2], []).append(call)
            for shape, rec in shapes.items():
                candidates[("cg_gemm_tf32", shape)] = (sum(a.elapsed_time(b) for a, b, _ in rec), rec)
        else:
            candidates[(name, None)] = (info["ms"], info["calls"])
    (name, shape), (_, rec) = max(candidates.items(), key=lambda kv: kv[1][0])
    if name == "cg_gemm_tf32":
        return _gemm_roofline(rec, bf16_sus, src, name=f"cg_gemm_tf32 {shape}")
    if name.startswith("cg_edge_attn") or name.startswith("cg_pooled_attn"):
        count = attn_bytes if name.startswith("cg_edge_attn") else pooled_attn_bytes
        nbytes = sum(count(info, name) for _, _, info in rec)
        secs = sum(a.elapsed_time(b) for a, b, _ in rec) / 1e3
        achieved = nbytes / secs / 1e9
        traffic = None
        if name in TRAFFIC_PER_ATOM:
            traffic = TRAFFIC_PER_ATOM[name] * sum(info[0] for _, _, info in rec) / len(rec)
        return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic, "algorithmic_bytes": nbytes / len(rec),
                "peak_source": f"{src} hbm_gbs", "traffic_source": "ncu capture at 2048 atoms, scaled by atoms"}
    return {"kernel": name, "bound": "hbm", "achieved": None, "peak": hbm, "unit": "GB/s", "frac": None,
            "traffic": None}


# the optimizer update that closes every training step, on both arms
ADAMW = {"lr": 1e-4, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 1e-2}


def cpu_step(ostep, params, opt, spec, pos, species, sys_ptr, e_t, f_t):
    """One step of the reference algorithm on the host: the oracle's eager
    create_graph step, then torch.optim.AdamW on its gradients."""
    out = ostep.train_step(params, spec, pos, species, sys_ptr, e_t, f_t)
    for name, t in params.items():
        t.grad = out["grads"][name]
    opt.step()
    return out


def cpu_optimizer(params):
    return torch.optim.AdamW(list(params.values()), **ADAMW)


def cpu_baseline(spec, sizes, pos_h, species_h, sys_ptr_h, e_t_h, f_t_h, model, budget_s=20.0):
    """The oracle (reference algorithm, torch CPU, fp32) on a bounded sample:
    the first systems of rank 0's batch, about 10-30 s of CPU work."""
    from oracle import step as ostep

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    params = {n: p.detach().float().cpu().clone() for n, p in model.named_parameters()}
    opt = cpu_optimizer(params)
    sample, atoms = 0, 0
    while sample < len(sizes) and atoms < 160:
        atoms += sizes[sample]
        sample += 1
    sys_ptr = sys_ptr_h[: sample + 1].clone()
    pos, species = pos_h[:atoms], species_h[:atoms]
    e_t, f_t = e_t_h[:sample], f_t_h[:atoms]
    cpu_step(ostep, params, opt, spec, pos, species, sys_ptr, e_t, f_t)  # warm-up
    steps, t0 = 0, time.perf_counter()
    while True:
        cpu_step(ostep, params, opt, spec, pos, species, sys_ptr, e_t, f_t)
        steps += 1
        if time.perf_counter() - t0 > budget_s / 2 or steps >= 5:
            break
    secs = (time.perf_counter() - t0) / steps
    return {"value": atoms / secs, "unit": "atoms/s", "cores": threads, "kind": "port",
            "sample": f"{sample} systems, {atoms} atoms of rank 0's batch, {steps} timed steps (step + AdamW), "
                      "fp32 torch CPU"}


# ---------------------------------------------------------------------------
# the reference arm: the reference's algorithm on the host cores
# ---------------------------------------------------------------------------


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from create_graph_b200 import mlip
    from oracle import step as ostep

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    spec = mlip.SPECS[CONFIG_NAME]
    sizes = mlip.workload_sizes(CONFIG_NAME, seed=1000, atoms_target=args.atoms)
    pos_h, species_h, sys_ptr_h = mlip.synthetic_systems(sizes, spec.n_species, seed=1000)
    e_t_h, f_t_h = mlip.make_targets(len(sizes), pos_h.shape[0], seed=2000)
    torch.manual_seed(0)
    params = {n: p.detach().float() for n, p in mlip.reference_parameters(spec).items()}
    opt = cpu_optimizer(params)
    # each step: a bounded sample (the next few systems, ~160 atoms) of the workload
    starts = []
    b = 0
    while b < len(sizes):
        e = b
        atoms = 0
        while e < len(sizes) and atoms < 160:
            atoms += sizes[e]
            e += 1
        starts.append((b, e))
        b = e

    def sample_step(i):
        b0, b1 = starts[i % len(starts)]
        a0, a1 = int(sys_ptr_h[b0]), int(sys_ptr_h[b1])
        sys_ptr = sys_ptr_h[b0 : b1 + 1] - a0
        cpu_step(ostep, params, opt, spec, pos_h[a0:a1], species_h[a0:a1], sys_ptr, e_t_h[b0:b1], f_t_h[a0:a1])
        return a1 - a0

    for i in range(args.warmup):
        sample_step(i)
    atoms, t0 = 0, time.perf_counter()
    for i in range(args.steps):
        atoms += sample_step(args.warmup + i)
    secs = time.perf_counter() - t0
    value = atoms / secs
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "atoms/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": secs / args.steps * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded random systems, random-init weights)",
        "config": {
            "workload": f"{CONFIG_NAME}: the reference algorithm (eager create_graph over torch CPU ops, "
                        "then torch.optim.AdamW) on bounded samples of ~160 atoms of the same batch",
            "parallelism": "host cores",
        },
        "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} steps of ~160-atom samples, {atoms} atoms timed"},
        "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["mine", "reference"], default="mine")
    parser.add_argument("--atoms", type=int, default=ATOMS_PER_RANK, help="atoms per GPU")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    args = parser.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()
