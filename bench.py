"""
Energy + force training-step throughput (atoms/s) on B200s, data-parallel weak
scaling, for every named workload.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mine|reference]

Headline workload (``value``): the 85M-parameter edge-attention MLIP. Per rank
~8192 atoms as random systems of U{20..200} atoms at 0.1 atoms/A^3 (seed 1000 +
rank), 12 blocks, hidden 768, 12 heads, FFN 3072, 128-Gaussian RBF, cutoff 6 A,
k <= 30 neighbours, 50 species, tf32 GEMMs with fp32 accumulation,
CompileConfig(memory_budget=0.5, checkpoint=r"blocks\\.\\d+"). A step is one
cg.create_graph call (energy + forces), the MSE loss on both and
loss.backward() (the parameter gradient through the force), one NCCL average
of the fp32 gradients for N > 1, and an AdamW update of the parameters (one
fused kernel; torch.optim.AdamW on the CPU arms). Synthetic data, random-init
weights.

The other named workloads are reported under ``shapes`` in the same line:

- ``small_mlip``: 64 systems x 64 atoms per rank, 4 blocks, hidden 128, 4
  heads, 64 RBF, k <= 32, 10 species, fp32 (three-term tf32 products), the
  same step (data-parallel like the headline);
- ``mlp_step``: the examples/mlp.py-style per-atom MLP (4 molecules x 32 atoms
  per rank, 3 -> 64 -> 64 -> 1 SiLU, MSE on energy and forces), data-parallel;
- ``edge_attn``: the masked edge-attention op at 4096 atoms x 8 heads x 32
  tokens x 32 dims (keys masked past U{8..32}), forward1 / backward1 /
  backward2 on one GPU, tf32 and fp32 precision, each against its HBM
  roofline.

Rank 0 prints one JSON line. CPU baselines (rank 0, one GPU only) and the
``--impl reference`` arm run the reference's own code on the host cores when
oracle/_ref holds it (oracle/ref_build.py copies it there), else the oracle's
restatement (``kind`` says which), on bounded samples.
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
# ranks and timing
# ---------------------------------------------------------------------------


class Job:
    """The process group and device of this rank, with the collectives the
    timing needs (every rank calls them in the same order)."""

    def __init__(self):
        import torch.distributed as dist

        self.dist = dist
        self.rank, self.world, self.local = env_rank()
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta

            dist.init_process_group("nccl", device_id=self.dev, timeout=timedelta(seconds=300))

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, x: float) -> list[float]:
        """x from every rank, in rank order."""
        if self.world == 1:
            return [x]
        t = torch.tensor([x], device=self.dev, dtype=torch.float64)
        out = [torch.empty_like(t) for _ in range(self.world)]
        self.dist.all_gather(out, t)
        return [float(o.item()) for o in out]

    def sum(self, x: int) -> int:
        if self.world == 1:
            return x
        t = torch.tensor([x], device=self.dev, dtype=torch.int64)
        self.dist.all_reduce(t)
        return int(t.item())

    def timed(self, step, steps: int, per_rank: list | None = None) -> float:
        """ms per step of `steps` calls, CUDA events on this rank's stream,
        barrier + synchronize on both sides, max over ranks (every rank's own
        figure appended to per_rank when given)."""
        self.barrier()
        torch.cuda.synchronize()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            step()
        end.record()
        torch.cuda.synchronize()
        self.barrier()
        mine = start.elapsed_time(end) / steps
        everyone = self.gather(mine)
        if per_rank is not None:
            per_rank.extend(everyone)
        return max(everyone)

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


def kernel_breakdown(native, step, n_steps=1):
    """Per entry point: launches, device time per step (CUDA events around each
    launch on its stream) and share of the library's device time in the step
    (the instrumented step's wall time is host-bound, so it is no denominator)."""
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
        out[name] = {"launches": len(rec) // n_steps, "ms": ms, "calls": rec}
    device_ms = sum(v["ms"] for v in out.values()) or total
    for v in out.values():
        v["share"] = v["ms"] / device_ms
    native.time_entry_points(names, enable=False)
    return out


def kernel_table(kernels):
    return {k: {"launches": v["launches"], "ms_per_step": v["ms"], "share": v["share"]}
            for k, v in sorted(kernels.items(), key=lambda kv: -kv[1]["ms"])}


# ---------------------------------------------------------------------------
# rooflines
# ---------------------------------------------------------------------------


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
# capture of a kernel at a smaller size, for the (kernel, heads, tokens, dims)
# shape captured; traffic grows with the atoms a launch processes, so a launch's
# traffic is this figure times its atoms.
TRAFFIC_PER_ATOM = {
    ("cg_pooled_attn_bwd1", 12, 30, 64): (53.767680e6 + 329.964032e6) / 2048,  # tf32
    ("cg_pooled_attn_bwd2", 12, 30, 64): (127.4e6 + 346.0e6) / 2048,           # tf32
}
# the edge-attention backward2 microbenchmark kernel, 8 heads x 32 tokens x 32 dims, tf32
EDGE_BWD2_TRAFFIC_PER_ATOM = (303.211264e6 + 133.112064e6) / 1024


def pooled_attn_bytes(info, name):
    """Algorithmic bytes of one pooled-attention launch: every per-atom operand
    once (the gathered token rows are re-reads of the atom rows), plus the
    per-token [dq | dk] rows the backward kernels write."""
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


def gemm_roofline(rec, bf16_sus, src, name="cg_gemm_tf32"):
    """Achieved GEMM flops against the dense tf32 peak (half the measured bf16
    one); fp32-precision launches make three tf32 products per flop, so their
    peak is a third of it. frac = tensor time at peak / measured time."""
    tf32 = bf16_sus / 2
    flops = secs = at_peak = 0.0
    for a, b, info in rec:
        m, n, k = info[:3]
        f = 2.0 * m * n * k
        flops += f
        secs += a.elapsed_time(b) / 1e3
        at_peak += f / ((tf32 / 3 if len(info) > 3 and info[3] == "fp32" else tf32) * 1e12)
    achieved = flops / secs / 1e12
    frac = at_peak / secs
    return {"kernel": name, "bound": "tensor", "achieved": achieved, "peak": achieved / frac, "unit": "TFLOP/s",
            "frac": frac, "traffic": None,
            "peak_source": f"{src} bf16 sustained / 2 (dense tf32; / 3 for fp32-precision launches)"}


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
        return gemm_roofline(rec, bf16_sus, src, name=f"cg_gemm_tf32 {shape}")
    if name.startswith("cg_edge_attn") or name.startswith("cg_pooled_attn"):
        count = attn_bytes if name.startswith("cg_edge_attn") else pooled_attn_bytes
        nbytes = sum(count(info, name) for _, _, info in rec)
        secs = sum(a.elapsed_time(b) for a, b, _ in rec) / 1e3
        achieved = nbytes / secs / 1e9
        traffic = None
        key = (name, *rec[0][2][1:])
        if key in TRAFFIC_PER_ATOM:
            traffic = TRAFFIC_PER_ATOM[key] * sum(info[0] for _, _, info in rec) / len(rec)
        return {"kernel": name, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": achieved / hbm, "traffic": traffic, "algorithmic_bytes": nbytes / len(rec),
                "peak_source": f"{src} hbm_gbs",
                "traffic_source": "ncu capture at 2048 atoms, scaled by atoms" if traffic else None}
    return {"kernel": name, "bound": "hbm", "achieved": None, "peak": hbm, "unit": "GB/s", "frac": None,
            "traffic": None}


# ---------------------------------------------------------------------------
# the B200 arm
# ---------------------------------------------------------------------------

# the optimizer update that closes every training step, on every arm
ADAMW = {"lr": 1e-4, "betas": (0.9, 0.999), "eps": 1e-8, "weight_decay": 1e-2}


def headline_workload(job, atoms, config, captured: bool):
    """The 85M workload of one rank (its balanced share of the global pool of
    systems): model, gradient buffer, host inputs, their device buffers and
    the training step (CUDA graphs, or eager with the all-reduce overlapped)."""
    from create_graph_b200 import mlip
    from create_graph_b200.ddp import FlatGradients
    from create_graph_b200.graph import make_batch
    from create_graph_b200.optim import FusedAdamW

    spec = mlip.SPECS[CONFIG_NAME]
    sizes, pos_h, species_h, sys_ptr_h = mlip.sharded_workload(CONFIG_NAME, job.rank, job.world, atoms)
    e_t_h, f_t_h = mlip.make_targets(len(sizes), pos_h.shape[0], seed=2000 + job.rank)
    torch.manual_seed(0)  # identical initial weights on every rank
    model = mlip.MLIP(spec, config=config).to(job.dev)
    host = (pos_h, species_h, sys_ptr_h, e_t_h, f_t_h)
    bufs = [t.to(job.dev) for t in host]
    pos, species, sys_ptr, e_t, f_t = bufs
    if captured:
        def loss_fn():
            # index structures and neighbour lists rebuilt from the buffers on every replay
            batch = make_batch(pos, species, sys_ptr, spec.n_species, max_atoms=max(sizes))
            return mlip.train_step(model, batch, e_t, f_t)

        step, kernels, grads = captured_training(job, model, loss_fn)
        return spec, sizes, model, grads, host, bufs, step, kernels
    grads = FlatGradients(model.parameters(), job.world if job.world > 1 else None)
    opt = FusedAdamW(grads, **ADAMW)

    def step():
        grads.zero()
        batch = make_batch(pos, species, sys_ptr, spec.n_species)
        loss = mlip.train_step(model, batch, e_t, f_t)
        grads.allreduce()
        opt.step()
        return loss

    return spec, sizes, model, grads, host, bufs, step, None


def run_mine(args):
    import create_graph_b200 as cg
    from create_graph_b200 import native

    job = Job()
    hbm, bf16, bf16_sus, src = peaks()
    config = cg.CompileConfig(memory_budget=0.5, checkpoint=r"blocks\.\d+")
    captured = not args.eager
    spec, sizes, model, grads, host, bufs, step, kernels_per_step = headline_workload(job, args.atoms, config,
                                                                                      captured)
    n_atoms = host[0].shape[0]
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- device-resident throughput ----
    launches0 = native.launch_count()
    last, per_rank = {}, []
    with ClockSampler(job.local) as clocks:
        ms = job.timed(lambda: last.__setitem__("loss", step()), args.steps, per_rank)
    launches = kernels_per_step * args.steps if captured else native.launch_count() - launches0
    peak_gb = job.max(torch.cuda.max_memory_allocated(job.dev) / 1e9)
    total_atoms = job.sum(n_atoms)
    value = total_atoms / (ms / 1e3)

    # ---- end to end through the public API, host buffers each step ----
    pinned = [t.pin_memory() for t in host]
    h2d = sum(t.numel() * t.element_size() for t in pinned)

    def e2e_step():
        for dst, src in zip(bufs, pinned):
            dst.copy_(src, non_blocking=True)
        last["host_loss"] = step().to("cpu")

    e_ms = job.timed(e2e_step, args.steps)
    e2e = {
        "value": total_atoms / (e_ms / 1e3),
        "unit": "atoms/s",
        "h2d_bytes_per_step": h2d,
        "d2h_bytes_per_step": last["host_loss"].numel() * last["host_loss"].element_size(),
    }

    # ---- the gradient average's own device time, per step (max over ranks) ----
    allreduce_ms = None
    if job.world > 1 and captured:
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        job.barrier()
        torch.cuda.synchronize()
        a0.record()
        for _ in range(3):
            grads.allreduce()
        a1.record()
        torch.cuda.synchronize()
        allreduce_ms = job.max(a0.elapsed_time(a1) / 3)

    # ---- kernel breakdown (one instrumented eager step after the timed region) ----
    from create_graph_b200 import mlip
    from create_graph_b200.graph import make_batch

    pos, species, sys_ptr, e_t, f_t = bufs
    kernels = kernel_breakdown(native, lambda: mlip.train_step(
        model, make_batch(pos, species, sys_ptr, spec.n_species, max_atoms=max(sizes)), e_t, f_t))
    shapes = {} if args.headline_only else other_shapes(job, args, hbm, bf16, bf16_sus, src)
    if job.rank == 0:
        line = {
            "metric": METRIC,
            "value": value,
            "unit": "atoms/s",
            "n_gpus": job.world,
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
                            "per-block checkpoint; step = neighbour lists + energy + forces + loss.backward() "
                            "+ AdamW update",
                "atoms_per_step": total_atoms,
                "systems_rank0": len(sizes),
                "sharding": "one global pool of systems, least-loaded assignment by atoms (equal work per rank)",
                "parallelism": f"dp{job.world}",
                "execution": ("CUDA graphs: create_graph + loss.backward() captured as one graph, the AdamW "
                              "update as another" if captured else "eager, all-reduce buckets overlapped with "
                              "backward"),
                "allreduce": ("none (1 rank)" if job.world == 1 else
                              "NCCL average of the flat fp32 gradients between the two graphs" if captured else
                              f"{len(grads.buckets)} buckets (<= 64 MiB) of the flat fp32 gradients, NCCL "
                              "all-reduce launched from backward hooks"),
                "l2": "working set of several GB per step (larger than L2)",
            },
            "e2e": e2e,
            "gpu_launches": launches,
            "per_rank_ms_per_step": per_rank,
            "allreduce_ms_per_step": allreduce_ms,
            # torch.cuda.max_memory_allocated since the start of the run (max over ranks):
            # parameters, gradients, AdamW moments and the step's activations (a
            # captured graph's buffers are allocated during its warm-up and capture)
            "peak_memory_gb": peak_gb,
            "roofline": roofline_of(kernels, hbm, bf16, bf16_sus, src),
            # the GEMM entry point as a whole (every shape of the step) against the tf32 peak
            "roofline_gemm": (gemm_roofline(kernels["cg_gemm_tf32"]["calls"], bf16_sus, src)
                              if "cg_gemm_tf32" in kernels else None),
            "kernels": kernel_table(kernels),
            "kernels_note": "per-kernel device times from one eager step, CUDA events around each launch; share of the library kernels' summed device time",
            "clocks": clocks.summary(),
            "loss": float(last["loss"].item()),
        }
        if "edge_attn" in shapes:
            # the metric's second part, kept at the top level: edge-attention backward2
            # against its HBM roofline at the microbenchmark shape
            line["edge_attn_bwd2"] = {"shape": shapes["edge_attn"]["shape"],
                                      "roofline": shapes["edge_attn"]["tf32"]["bwd2"]["roofline"],
                                      "roofline_fp32": shapes["edge_attn"]["fp32"]["bwd2"]["roofline"]}
        line["shapes"] = shapes
        if job.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_mlip(spec, sizes, host, model, budget_s=20.0)
            for name, fn in (("small_mlip", cpu_small_mlip), ("mlp_step", cpu_mlp), ("edge_attn", cpu_edge_attn)):
                if name in shapes:
                    shapes[name]["cpu_baseline"] = fn()
        print(json.dumps(line), flush=True)
    job.close()


def other_shapes(job, args, hbm, bf16, bf16_sus, src) -> dict:
    """The other named workloads (every rank runs the data-parallel ones)."""
    shapes = {
        "small_mlip": bench_small_mlip(job, args, hbm, bf16, bf16_sus, src),
        "mlp_step": bench_mlp(job, args, hbm, bf16, bf16_sus, src),
    }
    if job.rank == 0:
        shapes["edge_attn"] = bench_edge_attn(hbm, src)
    return shapes


def captured_training(job, model, loss_fn):
    """A training step of static shapes as two CUDA graphs (create_graph +
    loss.backward(), then the fused AdamW update) with the gradient average
    between them: (step, library kernels per step)."""
    from create_graph_b200.ddp import FlatGradients
    from create_graph_b200.graphs import CapturedStep
    from create_graph_b200.optim import FusedAdamW

    grads = FlatGradients(model.parameters(), job.world if job.world > 1 else None, overlap=False)
    opt = FusedAdamW(grads, **ADAMW)

    def backward():
        grads.zero()
        return loss_fn()

    first, second = CapturedStep(backward), CapturedStep(opt.step)

    def step():
        loss = first()
        grads.allreduce()
        second()
        return loss

    return step, first.kernels + second.kernels, grads


def bench_small_mlip(job, args, hbm, bf16, bf16_sus, src) -> dict:
    from create_graph_b200 import mlip, native
    from create_graph_b200.graph import make_batch

    spec = mlip.SMALL_MLIP
    sizes = mlip.workload_sizes("small_mlip")
    pos, species, sys_ptr = (t.to(job.dev) for t in mlip.synthetic_systems(sizes, spec.n_species,
                                                                          seed=1000 + job.rank))
    e_t, f_t = (t.to(job.dev) for t in mlip.make_targets(len(sizes), pos.shape[0], seed=2000 + job.rank))
    torch.manual_seed(0)
    model = mlip.MLIP(spec).to(job.dev)

    def loss_fn():
        # the batch's index structures and neighbour lists are rebuilt from the
        # position buffer on every replay
        batch = make_batch(pos, species, sys_ptr, spec.n_species, max_atoms=max(sizes))
        return mlip.train_step(model, batch, e_t, f_t)

    step, kernels, _ = captured_training(job, model, loss_fn)
    for _ in range(args.warmup):
        step()
    steps = max(args.steps, 20)
    ms = job.timed(step, steps)
    atoms = job.sum(pos.shape[0])
    eager_kernels = kernel_breakdown(native, lambda: mlip.train_step(
        model, make_batch(pos, species, sys_ptr, spec.n_species, max_atoms=max(sizes)), e_t, f_t))
    return {
        "metric": METRIC, "value": atoms / (ms / 1e3), "unit": "atoms/s", "ms_per_step": ms,
        "config": {"workload": "small_mlip: 64 systems x 64 atoms per GPU, 4 blocks, C 128, 4 heads, FFN 512, "
                               "64 RBF, k<=32, 10 species, fp32 (three-term tf32 products); step = neighbour lists "
                               "+ energy + forces + loss.backward() + AdamW update, captured as CUDA graphs",
                   "atoms_per_step": atoms, "parallelism": f"dp{job.world}"},
        "gpu_launches_per_step": kernels,
        "roofline": roofline_of(eager_kernels, hbm, bf16, bf16_sus, src),
        "roofline_gemm": (gemm_roofline(eager_kernels["cg_gemm_tf32"]["calls"], bf16_sus, src)
                          if "cg_gemm_tf32" in eager_kernels else None),
        "kernels": kernel_table(eager_kernels),
        "kernels_note": "per-kernel times from one eager step (CUDA events per launch); the timed steps replay graphs",
    }


def bench_mlp(job, args, hbm, bf16, bf16_sus, src) -> dict:
    from create_graph_b200 import mlp, native

    spec = mlp.MLPSpec()
    torch.manual_seed(0)
    model = mlp.MLPModel(spec).to(job.dev)
    pos, e_t, f_t = (t.to(job.dev) for t in mlp.synthetic_batch(spec, seed=job.rank))
    batch = {"pos": pos, "molecules": mlp.molecules_csr(spec, job.dev)}
    step, kernels, _ = captured_training(job, model, lambda: mlp.train_step(model, batch, e_t, f_t))
    for _ in range(max(args.warmup, 3)):
        step()
    steps = max(args.steps, 200)
    ms = job.timed(step, steps)
    atoms = job.sum(spec.n_mol * spec.n_atom)
    eager_kernels = kernel_breakdown(native, lambda: mlp.train_step(model, batch, e_t, f_t))
    return {
        "metric": METRIC, "value": atoms / (ms / 1e3), "unit": "atoms/s", "ms_per_step": ms,
        "config": {"workload": "mlp_step: 4 molecules x 32 atoms per GPU, per-atom MLP 3 -> 64 -> 64 -> 1 SiLU, "
                               "E = per-molecule sum, MSE(E) + MSE(F); step = energy + forces + loss.backward() "
                               "+ AdamW update (tf32 GEMMs), captured as CUDA graphs",
                   "atoms_per_step": atoms, "parallelism": f"dp{job.world}"},
        "gpu_launches_per_step": kernels,
        "roofline": roofline_of(eager_kernels, hbm, bf16, bf16_sus, src),
        "note": "latency bound: a few dozen kernels of a few microseconds each",
        "kernels": kernel_table(eager_kernels),
        "kernels_note": "per-kernel times from one eager step (CUDA events per launch); the timed steps replay graphs",
    }


def bench_edge_attn(hbm, src) -> dict:
    """forward1 / backward1 / backward2 at (4096, 8, 32, 32), both precisions."""
    import microbench

    out = {"shape": "(4096, 8, 32, 32) fp32, keys masked past U{8..32}"}
    for prec in ("tf32", "fp32"):
        mb = microbench.attn(4096, iters=10, hbm_gbs=hbm, which=("fwd1", "bwd1", "bwd2"), precision=prec)
        out[prec] = {}
        for name, r in mb.items():
            traffic = EDGE_BWD2_TRAFFIC_PER_ATOM * 4096 if (prec, name) == ("tf32", "bwd2") else None
            out[prec][name] = {
                "us_per_launch": r["us"], "atoms_per_s": 4096 / (r["us"] / 1e6),
                "roofline": {"bound": "hbm", "achieved": r["gb_s"], "peak": hbm, "unit": "GB/s",
                             "frac": r["gb_s"] / hbm, "traffic": traffic, "algorithmic_bytes": r["bytes"],
                             "us_per_launch": r["us"], "peak_source": f"{src} hbm_gbs", "precision": prec},
            }
    return out


# ---------------------------------------------------------------------------
# CPU legs: the reference's own code (oracle/_ref) or the oracle's restatement
# ---------------------------------------------------------------------------


def cpu_optimizer(params):
    return torch.optim.AdamW(list(params.values()), **ADAMW)


class CpuMlipStep:
    """One step of the reference's path on the host cores: neighbour lists
    (oracle/neighbors.py), the reference's cg.create_graph(exact=True) on the
    model's energy function (or, without oracle/_ref, the oracle's own eager
    step), the MSE loss and torch.optim.AdamW."""

    def __init__(self, spec, params):
        from oracle import ref

        self.spec, self.params = spec, params
        self.opt = cpu_optimizer(params)
        loaded = ref.load()
        if loaded is not None:
            self.kind = "reference"
            self.ref_cg = loaded[0]
            self.model = ref.energy_model(self.ref_cg, params, spec)
            self.opt = torch.optim.AdamW(list(self.model.parameters()), **ADAMW)
            self.label = "the reference's cg.create_graph(exact=True) (oracle/_ref)"
        else:
            self.kind = "port"
            self.label = "the oracle's eager create_graph restatement (oracle/step.py)"

    def __call__(self, pos, species, sys_ptr, e_t, f_t):
        import numpy as np

        from oracle import neighbors as onb
        from oracle import step as ostep

        if self.kind == "port":
            out = ostep.train_step(self.params, self.spec, pos, species, sys_ptr, e_t, f_t)
            for name, t in self.params.items():
                t.grad = out["grads"][name]
            self.opt.step()
            return
        nbr, counts, _, _ = onb.neighbor_list(pos.numpy(), np.asarray(sys_ptr), self.spec.cutoff, self.spec.k)
        batch = {"pos": pos, "species": species, "sys_ptr": sys_ptr, "nbr": torch.from_numpy(nbr),
                 "counts": torch.from_numpy(counts)}
        self.model.zero_grad()
        res, grads = self.ref_cg.create_graph(self.model, batch, exact=True)
        loss = (res["energy"] - e_t).square().mean() + (-grads["pos"] - f_t).square().mean()
        loss.backward()
        self.opt.step()


def _cpu_threads() -> int:
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    return threads


def _sample_ranges(sizes, atoms_per_sample):
    """Consecutive system ranges of ~atoms_per_sample atoms each."""
    out, b = [], 0
    while b < len(sizes):
        e, atoms = b, 0
        while e < len(sizes) and atoms < atoms_per_sample:
            atoms += sizes[e]
            e += 1
        out.append((b, e))
        b = e
    return out


def _time_cpu_samples(runner, host, ranges, warmup, steps, budget_s):
    """Run `warmup` then `steps` samples (cycling through `ranges`); with steps
    = 0, as many as fit in budget_s (at most 8). Returns (atoms, samples, s)."""
    pos_h, species_h, sys_ptr_h, e_t_h, f_t_h = host

    def one(i):
        b0, b1 = ranges[i % len(ranges)]
        a0, a1 = int(sys_ptr_h[b0]), int(sys_ptr_h[b1])
        runner(pos_h[a0:a1], species_h[a0:a1], sys_ptr_h[b0 : b1 + 1] - a0, e_t_h[b0:b1], f_t_h[a0:a1])
        return a1 - a0

    for i in range(warmup):
        one(i)
    atoms, n, t0 = 0, 0, time.perf_counter()
    while True:
        atoms += one(warmup + n)
        n += 1
        if steps > 0 and n >= steps:
            break
        if steps == 0 and (n >= 8 or time.perf_counter() - t0 > budget_s):
            break
    return atoms, n, time.perf_counter() - t0


def cpu_baseline_mlip(spec, sizes, host, model, budget_s=20.0, atoms_per_sample=160):
    threads = _cpu_threads()
    params = {n: p.detach().float().cpu().clone() for n, p in model.named_parameters()}
    runner = CpuMlipStep(spec, params)
    atoms, n, secs = _time_cpu_samples(runner, host, _sample_ranges(sizes, atoms_per_sample)[:1], 1, 0, budget_s / 2)
    return {"value": atoms / secs, "unit": "atoms/s", "cores": threads, "kind": runner.kind,
            "sample": f"{n} timed steps of the first ~{atoms_per_sample} atoms of rank 0's batch (step + AdamW), "
                      f"fp32 torch CPU, {runner.label}"}


def cpu_small_mlip():
    from create_graph_b200 import mlip

    spec = mlip.SMALL_MLIP
    threads = _cpu_threads()
    sizes = mlip.workload_sizes("small_mlip")
    pos, species, sys_ptr = mlip.synthetic_systems(sizes, spec.n_species, seed=1000)
    e_t, f_t = mlip.make_targets(len(sizes), pos.shape[0], seed=2000)
    torch.manual_seed(0)
    params = {n: t.float() for n, t in mlip.reference_parameters(spec).items()}
    runner = CpuMlipStep(spec, params)
    atoms, n, secs = _time_cpu_samples(runner, (pos, species, sys_ptr, e_t, f_t), _sample_ranges(sizes, 512), 1,
                                       0, 10.0)
    return {"value": atoms / secs, "unit": "atoms/s", "cores": threads, "kind": runner.kind,
            "sample": f"{n} timed steps of 8 of the 64 systems (512 atoms each) (step + AdamW), fp32 torch CPU, "
                      f"{runner.label}"}


def cpu_mlp():
    from create_graph_b200 import mlp
    from oracle import ref

    threads = _cpu_threads()
    spec = mlp.MLPSpec()
    pos, e_t, f_t = mlp.synthetic_batch(spec, seed=0)
    mol = torch.arange(spec.n_mol * spec.n_atom) // spec.n_atom
    loaded = ref.load()
    torch.manual_seed(0)
    if loaded is not None:
        ref_cg, kind, label = loaded[0], "reference", "the reference's cg.create_graph (exact=True, oracle/_ref)"
        model = ref.mlp_model(ref_cg, spec.hidden, spec.n_mol, spec.n_atom)
    else:
        from torch import nn

        ref_cg, kind, label = None, "port", "eager autograd.grad(create_graph=True) in torch (oracle restatement)"
        model = nn.Sequential(nn.Linear(3, spec.hidden), nn.SiLU(), nn.Linear(spec.hidden, spec.hidden), nn.SiLU(),
                              nn.Linear(spec.hidden, 1))
    opt = torch.optim.AdamW(list(model.parameters()), **ADAMW)

    def step():
        opt.zero_grad()
        if ref_cg is not None:
            out, grads = ref_cg.create_graph(model, {"pos": pos, "mol": mol}, exact=True)
            energy, g = out["energy"], grads["pos"]
        else:
            x = pos.detach().requires_grad_(True)
            p3 = x.view(spec.n_mol, spec.n_atom, 3)
            centred = (p3 - p3.mean(dim=1, keepdim=True)).view(-1, 3)
            energy = torch.zeros(spec.n_mol).index_add(0, mol, model(centred)[:, 0])
            (g,) = torch.autograd.grad(energy.sum(), x, create_graph=True)
        loss = (energy - e_t).square().mean() + (-g - f_t).square().mean()
        loss.backward()
        opt.step()

    for _ in range(5):
        step()
    n, t0 = 0, time.perf_counter()
    while n < 2000 and time.perf_counter() - t0 < 5.0:
        step()
        n += 1
    secs = time.perf_counter() - t0
    atoms = n * spec.n_mol * spec.n_atom
    return {"value": atoms / secs, "unit": "atoms/s", "cores": threads, "kind": kind,
            "sample": f"{n} steps of the whole 128-atom batch (step + AdamW), fp32 torch CPU, {label}"}


def cpu_edge_attn(n_sample=512):
    """The reference's EdgeAttention op (or the oracle's numpy restatement) on
    n_sample of the 4096 atoms, fp32, per kernel; atoms/s = n_sample / time."""
    import microbench
    from oracle import ref

    threads = _cpu_threads()
    q, k, v, bias, counts, g, hq, hk, hv, hb, scale = microbench.attn_inputs(n_sample, device="cpu")
    keymask = torch.arange(q.shape[2])[None, :] >= counts[:, None].long()
    bias = bias.masked_fill(keymask[:, None, None, :], -torch.inf)
    hb = torch.where(torch.isfinite(bias), hb, torch.zeros_like(hb))
    loaded = ref.load()
    if loaded is not None:
        op, kind, label = loaded[1], "reference", "the reference's EdgeAttention op (oracle/_ref)"
        _, lse = op.op(q, k, v, bias, scale)
        fns = {
            "fwd1": lambda: op.op(q, k, v, bias, scale),
            "bwd1": lambda: op.backward1_op(q, k, v, bias, lse, g, scale),
            "bwd2": lambda: op.backward2_op(q, k, v, bias, lse, g, scale, hq, hk, hv, hb),
        }
    else:
        from oracle import edge_attn as oattn

        a = [t.double().numpy() for t in (q, k, v, bias)]
        kind, label = "port", "the oracle's numpy restatement (oracle/edge_attn.py, float64)"
        fns = {
            "fwd1": lambda: oattn.forward1(*a, scale),
            "bwd1": lambda: oattn.backward1(*a, g.double().numpy(), scale),
            "bwd2": lambda: oattn.backward2(*a, g.double().numpy(), scale,
                                            *(t.double().numpy() for t in (hq, hk, hv, hb))),
        }
    out = {"unit": "atoms/s", "cores": threads, "kind": kind,
           "sample": f"{n_sample} of the 4096 atoms (8 heads x 32 x 32), fp32, best of 2, {label}"}
    for name, fn in fns.items():
        best = None
        for _ in range(2):
            t0 = time.perf_counter()
            fn()
            dt = time.perf_counter() - t0
            best = dt if best is None else min(best, dt)
        out[name] = {"value": n_sample / best, "seconds_per_sample": best}
    out["value"] = out["bwd2"]["value"]
    return out


# ---------------------------------------------------------------------------
# the reference arm: the reference's path on the host cores
# ---------------------------------------------------------------------------


def run_reference(args):
    rank, world, _ = env_rank()
    if rank != 0:
        return
    from create_graph_b200 import mlip

    threads = _cpu_threads()
    spec = mlip.SPECS[CONFIG_NAME]
    sizes, pos, species, sys_ptr = mlip.sharded_workload(CONFIG_NAME, 0, 1, args.atoms)
    host = (pos, species, sys_ptr, *mlip.make_targets(len(sizes), pos.shape[0], seed=2000))
    torch.manual_seed(0)
    params = {n: p.detach().float() for n, p in mlip.reference_parameters(spec).items()}
    runner = CpuMlipStep(spec, params)
    # each step: a bounded sample (the next few systems, ~160 atoms) of the workload
    atoms, n, secs = _time_cpu_samples(runner, host, _sample_ranges(sizes, 160), args.warmup, args.steps, 0.0)
    value = atoms / secs
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": "atoms/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": secs / n * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded random systems, random-init weights)",
        "config": {
            "workload": f"{CONFIG_NAME}: {runner.label}, then torch.optim.AdamW, on bounded samples of "
                        "~160 atoms of the same batch",
            "parallelism": "host cores",
        },
        "cpu_baseline": {"value": value, "unit": "atoms/s", "cores": threads, "kind": runner.kind,
                         "sample": f"{n} steps of ~160-atom samples, {atoms} atoms timed"},
        "e2e": {"value": value, "unit": "atoms/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=5)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["mine", "reference"], default="mine")
    parser.add_argument("--atoms", type=int, default=ATOMS_PER_RANK, help="atoms per GPU (headline workload)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--headline-only", action="store_true", help="skip the other named workloads")
    parser.add_argument("--eager", action="store_true",
                        help="run the headline step eagerly (all-reduce buckets overlapped with backward)")
    args = parser.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_mine(args)


if __name__ == "__main__":
    main()
