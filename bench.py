#!/usr/bin/env python
"""Headline benchmark: FlashCart potential energy + forces + stress at 27,648 atoms.

Workload (the MD-scale inference step): a seeded 27,648-atom water-like periodic box (9,216 H2O,
24 x 24 x 16 jittered lattice, 74.52 x 74.52 x 49.68 A), r_max 5 A (~1.49 M edges), the
reference architecture with 128 channels, hidden and edge ranks <= 3, 2 interaction
layers, correlation 3, random-init weights (torch.manual_seed(0)), float32. One step =
``FlashCartPotential.predict(graph, compute_forces=True, compute_stress=True)``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

With N > 1 (torchrun, one rank per GPU) the one cell is split by atom-domain
decomposition (``flashcart_b200.domain``: 2x1x1, 2x2x1, 2x2x2 domains); each rank
evaluates the edges of the atoms it owns and exchanges ghost positions and layer
features with its neighbours over NCCL, energy and virial are summed over ranks
("scaling": "strong", value = 27,648 atoms / step time). The timed region is bracketed
by a barrier and a device synchronise on each rank and the max over ranks is reported. ``--impl reference``
times the CPU reference port (the oracle) on the host cores instead.
"""

from __future__ import annotations

import argparse
import datetime
import json
import os
import re
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "atom-steps/s (E+F+stress) at 27,648 atoms"
UNIT = "atom-steps/s"
WORKLOAD = ("MD-scale inference: 27,648-atom water box (24x24x16 H2O lattice, r_max 5 A), FlashCart C=128, l<=3, "
            "2 interactions, correlation 3, E+F+stress per step")
FALLBACK_HBM_GBS = 6650.0


def _args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--cpu-atoms", type=int, choices=sorted(CPU_BOXES), default=192,
                    help="atoms of the CPU sample (same density as the 27,648-atom box; the per-atom rate is the reported "
                         "figure, the 27,648-atom box itself does not fit host RAM in the reference py path)")
    ap.add_argument("--op-case", choices=["conv", "gemm", "linear_bf16", "dense"], default=None,
                    help="run one small operator case (for ncu captures) instead of the benchmark")
    ap.add_argument("--allreduce", choices=["buckets", "flat"], default="buckets",
                    help="data-parallel training: gradient all-reduce in buckets during the backward, or one "
                         "flat all-reduce after it")
    ap.add_argument("--config", type=int, choices=[1, 2, 3, 4], default=3,
                    help="3: the headline E+F+S step; 1: the isolated TP convolution microbenchmark; "
                         "2: edge expansion + equivariant linear map (one GPU, one JSON line); "
                         "4: data-parallel training (32 molecules per GPU, energy + force loss, Muon)")
    return ap.parse_args()


def _dist_env():
    return int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)), int(os.environ.get("LOCAL_RANK", 0))


# --------------------------------------------------------------------------------- inputs


def build_graph(seed: int, device):
    from flashcart_b200.data import neighbors, synthetic

    s = synthetic.water_box(24, 24, 16, seed=seed)
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0,
                                     device=str(device) if torch.cuda.is_available() else "cpu")
    g = synthetic.graph_from_structure(s, ei, sh, device=device, dtype=torch.float32)
    return g, ei.shape[1] / len(s["positions"])


def build_model(avg_neighbors: float, device):
    from flashcart_b200.model.flashcart import FlashCartPotential
    from flashcart_b200.model.presets import water_model_kwargs

    torch.manual_seed(0)
    return FlashCartPotential(**water_model_kwargs("cfg3arch", avg_neighbors)).to(device)


# --------------------------------------------------------------------------------- clocks


class ClockSampler:
    """SM clock and throttle reasons sampled during the timed region.

    NVML (read-only queries) polled every 10 ms from a thread, so a timed region of a few
    tens of milliseconds (8 ranks) still gets samples; the first sample is taken when the
    sampler starts, i.e. at the start of the timed region. Where NVML cannot be loaded,
    ``nvidia-smi -lms 200`` in a subprocess (which misses regions shorter than 200 ms)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
    NAMES = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, local_rank: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        idx = local_rank
        if vis:
            parts = [p.strip() for p in vis.split(",")]
            if local_rank < len(parts) and parts[local_rank].isdigit():
                idx = int(parts[local_rank])
        self.idx = idx
        self.proc = None
        self.file = None
        self.thread = None
        self.samples = []  # (sm_mhz, max_mhz, reasons)
        self.source = None

    def _nvml_handle(self):
        try:
            import pynvml
            pynvml.nvmlInit()
            return pynvml, pynvml.nvmlDeviceGetHandleByIndex(self.idx)
        except Exception:  # NVML missing or no such device: fall back to nvidia-smi
            return None, None

    def _nvml_sample(self, nv, h):
        sm = nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM)
        mx = nv.nvmlDeviceGetMaxClockInfo(h, nv.NVML_CLOCK_SM)
        bits = nv.nvmlDeviceGetCurrentClocksEventReasons(h)
        flags = (nv.nvmlClocksEventReasonHwSlowdown, nv.nvmlClocksEventReasonHwThermalSlowdown,
                 nv.nvmlClocksEventReasonSwThermalSlowdown, nv.nvmlClocksEventReasonSwPowerCap)
        self.samples.append((float(sm), float(mx), {n for n, f in zip(self.NAMES, flags) if bits & f}))

    def start(self):
        import threading

        nv, h = self._nvml_handle()
        if nv is not None:
            self.source = "nvml"
            self._stop = threading.Event()
            try:
                self._nvml_sample(nv, h)
            except Exception:
                nv = None
        if nv is not None:
            def poll():
                while not self._stop.wait(0.010):
                    try:
                        self._nvml_sample(nv, h)
                    except Exception:
                        return

            self.thread = threading.Thread(target=poll, daemon=True)
            self.thread.start()
            return
        self.source = "nvidia-smi"
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, ValueError):
            self.proc = None

    def _read_smi(self):
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.file.flush()
        self.file.seek(0)
        rows = [r.split(",") for r in self.file.read().strip().splitlines() if r.strip()]
        os.unlink(self.file.name)
        for r in rows:
            r = [c.strip() for c in r]
            if len(r) < 9:
                continue
            try:
                sm, mx = float(r[1]), float(r[2])
            except ValueError:
                continue
            self.samples.append((sm, mx, {n for n, v in zip(self.NAMES, r[5:9]) if v.lower() == "active"}))

    def stop(self):
        if self.thread is not None:
            self._stop.set()
            self.thread.join(timeout=5)
        elif self.proc is not None:
            self._read_smi()
        if not self.samples:
            return None
        reasons = set().union(*(r for _, _, r in self.samples))
        return {"sm_mhz": statistics.median(s for s, _, _ in self.samples),
                "sm_max_mhz": max(m for _, m, _ in self.samples), "reasons": sorted(reasons),
                "samples": len(self.samples), "source": self.source}


# --------------------------------------------------------------------------------- helpers


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def _count_own_launches(step, graph) -> int:
    """Kernels of this library's shared object launched by one step, counted from the CUDA
    activity trace of one extra (untimed) step."""
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step(graph)
        torch.cuda.synchronize()
    own = re.compile(r"(^|[^A-Za-z_])(fc::|tma::)|sig_[0-9]{3}[ns]::")
    n = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and own.search(ev.name):
            n += 1
    return n


def _replay_difference(eager, replayed) -> float:
    """Largest relative difference (to each output's largest magnitude, at least 1) between
    the energy, forces and stress of an eager step and of a graph replay."""
    worst = 0.0
    for k in ("energy", "forces", "stress"):
        a, b = replayed[k].double(), eager[k].double()
        worst = max(worst, (a - b).abs().max().item() / max(1.0, b.abs().max().item()))
    return worst


def _profile_traffic(kernel: str):
    """DRAM bytes per launch of a kernel from the committed ncu summaries (profiles/*.md)."""
    pat = re.compile(r"traffic_bytes_per_launch\[" + re.escape(kernel) + r"\]\s*[:=]\s*([0-9.eE+]+)")
    d = os.path.join(ROOT, "profiles")
    if not os.path.isdir(d):
        return None
    for fn in sorted(os.listdir(d)):
        if fn.endswith((".md", ".txt")):
            m = pat.search(open(os.path.join(d, fn)).read())
            if m:
                return float(m.group(1))
    return None


# water boxes of the CPU sample: molecules per lattice axis at the benchmark box's spacing and seed.
# The float32 oracle port peaks near 20 MB of host memory per atom (31 GB at 1,536 atoms),
# so 3,072 atoms does not fit a 62 GB host and is not offered.
CPU_BOXES = {192: (4, 4, 4), 1536: (8, 8, 8)}


def cpu_reference_sample(steps: int, warmup: int, min_seconds: float = 0.0, atoms: int = 192):
    """The oracle port of the potential on the host cores: a water box of ``atoms`` atoms
    (192 by default), the 128-channel rank <= 3 architecture of the benchmark."""
    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.model.flashcart import FlashCartPotential
    from flashcart_b200.model.presets import water_model_kwargs
    from oracle import model_oracle

    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    s = synthetic.water_box(*CPU_BOXES[atoms], seed=0)
    ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0)
    avg = ei.shape[1] / len(s["positions"])
    cfg = water_model_kwargs("cfg3arch", avg)
    torch.manual_seed(0)
    sd = FlashCartPotential(**cfg).state_dict()
    g = synthetic.graph_from_structure(s, ei, sh, device="cpu", dtype=torch.float32)
    for _ in range(warmup):
        model_oracle.predict(sd, cfg, g)
    n_done, t0 = 0, time.perf_counter()
    while n_done < steps or (time.perf_counter() - t0) < min_seconds:
        model_oracle.predict(sd, cfg, g)
        n_done += 1
    dt = time.perf_counter() - t0
    n_atoms = len(s["positions"])
    rec = {"value": n_atoms * n_done / dt, "unit": UNIT, "cores": cores, "kind": "port",
           "sample": f"{n_done} E+F+S steps of a {n_atoms}-atom water box ({ei.shape[1]} edges) with the 128-channel, "
                     f"rank <= 3 architecture, float32, oracle port (torch CPU) on {cores} threads; per-atom rate"}
    # how the port's speed compares with the reference's own PyTorch path (measured where the
    # reference source is available, oracle/time_port_vs_reference.py)
    cmp_path = os.path.join(ROOT, "oracle", "port_vs_reference_cpu.json")
    if os.path.exists(cmp_path):
        with open(cmp_path) as f:
            rec["port_vs_reference_py"] = json.load(f)
    return rec, dt / n_done


# --------------------------------------------------------------------------------- arms


def run_reference(args):
    rank, world, _ = _dist_env()
    if rank != 0:
        return
    base, ms = cpu_reference_sample(args.steps, args.warmup, atoms=args.cpu_atoms)
    line = {
        "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": base["sample"], "parallelism": "host cores"},
        "impl": "reference", "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_b200(args):
    import torch.distributed as dist

    from flashcart_b200 import ops

    rank, world, local = _dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    # one periodic cell; with N > 1 GPUs it is split by atom-domain decomposition
    graph, avg = build_graph(seed=0, device=dev)
    n_atoms = graph["positions"].shape[0]
    n_edges = graph["edge_index"].shape[1]
    model = build_model(avg, dev)
    plan = None
    if world > 1:
        from flashcart_b200.domain import build_plans

        plan = build_plans(graph["positions"].cpu(), graph["cell"][0].cpu(), graph["edge_index"].cpu(),
                           graph["shifts"].cpu(), world)[rank].to(dev)

    def step(g):
        if world > 1:
            return model.predict_domain(g, plan, compute_forces=True, compute_stress=True)
        return model.predict(g, compute_forces=True, compute_stress=True)

    graph = dict(graph)
    graph["use_shifts"] = True  # periodic cell: no device read of pbc inside the (captured) step
    for _ in range(max(args.warmup, 0)):
        step(graph)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    # pass 1 (eager launches): per-operator CUDA events for the roofline and the kernel breakdown
    timer = ops.KernelTimer()
    ops.set_kernel_timer(timer)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        out = step(graph)
    e1.record()
    torch.cuda.synchronize()
    ops.set_kernel_timer(None)
    eager_ms = e0.elapsed_time(e1) / args.steps
    ops.check_device_status(dev)
    own_per_step = _count_own_launches(step, graph)

    # pass 2 (headline): the same step captured once as a CUDA graph and replayed
    from flashcart_b200.graphs import GraphedStep

    if world > 1:
        dist.barrier()
    graphed = GraphedStep(step, graph, warmup=2)
    for _ in range(3):
        replayed = graphed()
    torch.cuda.synchronize()
    # the timed path must give the eager step's result (same inputs; atomics make float32
    # agree to rounding, not bit for bit)
    replay_rel = _replay_difference(out, replayed)
    if world > 1:  # every rank takes the same decision
        r = torch.tensor([replay_rel], device=dev, dtype=torch.float64)
        dist.all_reduce(r, op=dist.ReduceOp.MAX)
        replay_rel = float(r[0])
    if replay_rel > 1e-5:
        raise RuntimeError(f"graph replay differs from the eager step: max relative difference {replay_rel:.3e}")
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    torch.cuda.cudart().cudaProfilerStart()  # lets `ncu --profile-from-start off` capture exactly this region
    e0.record()
    for _ in range(args.steps):
        out = graphed()
    e1.record()
    torch.cuda.synchronize()
    torch.cuda.cudart().cudaProfilerStop()
    ms = e0.elapsed_time(e1) / args.steps
    clock_info = clocks.stop()
    ops.check_device_status(dev)
    if world > 1:
        dist.barrier()

    # end to end: inputs from pinned host memory into the graph's static buffers, replay,
    # results back to pinned host memory, every step
    keys = ["positions", "cell", "atom_types", "edge_index", "shifts", "batch"]
    if world > 1:
        keys = ["positions", "cell", "atom_types"]  # the rank's edges and exchange lists travel with its plan
    host = {k: graph[k].cpu().pin_memory() for k in keys}
    h2d = sum(t.numel() * t.element_size() for t in host.values())
    plan_pairs = []
    if plan is not None:
        for dev_t in (plan.owned, plan.ghosts, plan.edge_index, plan.shifts, *plan.send_idx, *plan.recv_pos):
            plan_pairs.append((dev_t, dev_t.cpu().pin_memory()))
        h2d += sum(h.numel() * h.element_size() for _, h in plan_pairs)
    out_host = {k: torch.empty(out[k].shape, dtype=out[k].dtype, pin_memory=True) for k in ("energy", "forces",
                                                                                             "stress")}
    d2h = sum(t.numel() * t.element_size() for t in out_host.values())
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(args.steps):
        for d_t, h_t in plan_pairs:
            d_t.copy_(h_t, non_blocking=True)
        o = graphed({k: v for k, v in host.items()})
        for k in out_host:
            out_host[k].copy_(o[k], non_blocking=True)
    a1.record()
    torch.cuda.synchronize()
    e2e_ms = a0.elapsed_time(a1) / args.steps

    # roofline of the dominant kernel (largest total device time in the timed region). The
    # halo collective is not a candidate: its eager-pass time includes the wait for the
    # slowest rank (ranks drift apart in eager mode), so it is timed on its own below.
    durs = timer.durations_ms()
    nbytes = timer.bytes_per_call()
    top = max((k for k in durs if not k.startswith("halo")), key=lambda k: sum(durs[k]))
    avg_ms = sum(durs[top]) / len(durs[top])
    bytes_per_launch = sum(nbytes[top]) / len(nbytes[top])
    peak, peak_src = _peaks()
    achieved = bytes_per_launch / (avg_ms * 1e-3) / 1e9
    traffic = _profile_traffic(top)
    share = sum(durs[top]) / (eager_ms * args.steps)

    t = torch.tensor([ms, e2e_ms, eager_ms], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, e2e_max, eager_max = float(t[0]), float(t[1]), float(t[2])
    ranks = None
    if world > 1:
        # what limits the scaling: per-rank step time (graphed), halo time (eager pass: pack,
        # NCCL all-to-all, unpack, forward and backward) and each rank's share of the edges
        halo_ms = sum(sum(v) for k, v in durs.items() if k.startswith("halo")) / args.steps
        alone_ms = _halo_alone_ms(plan, graph_feature_width(model), dev)
        mine = torch.tensor([ms, eager_ms, halo_ms, float(plan.edge_index.shape[1]), float(plan.n_own),
                             float(plan.n_ghost), alone_ms], device=dev, dtype=torch.float64)
        every = [torch.zeros_like(mine) for _ in range(world)]
        dist.all_gather(every, mine)
        every = torch.stack(every).cpu()
        ranks = {"step_ms": [round(float(v), 3) for v in every[:, 0]],
                 "eager_ms": [round(float(v), 3) for v in every[:, 1]],
                 "halo_ms_per_step": [round(float(v), 3) for v in every[:, 2]],
                 "halo_exchange_alone_ms": [round(float(v), 4) for v in every[:, 6]],
                 "edges": [int(v) for v in every[:, 3]], "owned_atoms": [int(v) for v in every[:, 4]],
                 "ghost_atoms": [int(v) for v in every[:, 5]],
                 "edge_imbalance_max_over_min": float(every[:, 3].max() / every[:, 3].min())}
    graphed.release()
    cpu_base = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu_base, _ = cpu_reference_sample(steps=1, warmup=1, min_seconds=10.0)
    if rank == 0:
        value = n_atoms / (ms_max * 1e-3)
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "atoms": n_atoms, "edges": n_edges,
                       "l2": "inputs larger than L2 (per-edge path weights of layer 2: "
                             f"{n_edges * 23 * 128 * 4 / 1e9:.1f} GB)",
                       "execution": "whole step captured as one CUDA graph and replayed; roofline and "
                                    "kernel breakdown from an eager pass of the same steps",
                       "eager_ms_per_step": eager_max,
                       "replay_vs_eager_max_rel": replay_rel,
                       "parallelism": (f"atom-domain decomposition {'x'.join(map(str, plan.grid))} of the one cell, "
                                       f"halo exchange over NCCL (all-to-all), x{world}") if plan is not None
                       else "one cell on one GPU"},
            "roofline": {"bound": "hbm", "kernel": top, "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "peak_source": f"{peak_src} (hbm_gbs)",
                         "bytes_per_launch": bytes_per_launch, "ms_per_launch": avg_ms,
                         "share_of_step": share},
            "cpu_baseline": cpu_base,
            "e2e": {"value": n_atoms / (e2e_max * 1e-3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": own_per_step * args.steps,
            "clocks": clock_info,
            "kernels_ms_per_step": {k: sum(v) / args.steps for k, v in sorted(durs.items(),
                                                                               key=lambda kv: -sum(kv[1]))},
        }
        if ranks is not None:
            line["ranks"] = ranks
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def graph_feature_width(model) -> int:
    """Width of the node features that the halo exchange moves between interaction layers."""
    return int(model.node_dim)


def _halo_alone_ms(plan, width: int, dev, reps: int = 20) -> float:
    """One forward halo exchange (pack, NCCL all-to-all, unpack) of a layer's node features
    (owned rows x width floats), timed on its own after a barrier: the per-exchange cost
    without the rank skew that the eager pass adds. Every rank runs the same exchanges."""
    import torch.distributed as dist

    from flashcart_b200.domain import ghost_rows_from_owners

    x = torch.randn(plan.n_own, width, device=dev)
    out = x.new_empty((plan.n_ghost, width))
    for _ in range(3):
        ghost_rows_from_owners(x, plan, out=out)
    torch.cuda.synchronize()
    dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        ghost_rows_from_owners(x, plan, out=out)
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def run_op_case(case: str):
    """Small single-operator cases with the benchmark's shapes, sized for ncu captures (a few GB):
    ``conv``: conv products (3,3)->3 and (0,3)->3, C=128, forward + backward, on a 3,456-atom water
    box; ``gemm``: the radial-MLP output layer 64 -> 23*128 and its input gradient on 200,000 rows;
    ``linear_bf16``: the bf16 storage path of o3.LinearLayer(3, 3, 128, 128) on 400,000 rows;
    ``dense``: the product layers' node-level product (3,3)->3, C=128, shared frozen weights,
    forward + input gradients on the benchmark's 27,648 rows."""
    from flashcart_b200 import o3
    from flashcart_b200.data import neighbors, synthetic
    from flashcart_b200.nn.layers import LinearLayer

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    if case == "conv":
        s = synthetic.water_box(12, 12, 8, seed=0)
        ei, sh = neighbors.neighbor_list(s["positions"], s["cell"], s["pbc"], 5.0, device="cuda")
        pos = torch.as_tensor(s["positions"], device=dev, dtype=torch.float32)
        ei = torch.as_tensor(ei, device=dev)
        cell = torch.as_tensor(s["cell"], device=dev, dtype=torch.float32)
        vec = pos[ei[1]] - pos[ei[0]] + torch.as_tensor(sh, device=dev, dtype=torch.float32) @ cell
        x2 = o3.Irreps(3)(vec)
        n, c = pos.shape[0], 128
        for (l1, l2, lo) in [(3, 3, 3), (0, 3, 3)]:
            tp = o3.TensorProduct(l1, l2, lo, c, 1)
            in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g)
            w = torch.randn(ei.shape[1], tp.n_total_paths * c, device=dev, generator=g)
            out = tp(in1, x2, w, ei[0], ei[1])
            torch.ops.flashcart.tp_bwd(torch.randn_like(out), in1, x2, w, ei[0], ei[1], l1, l2, lo, c, 1, False,
                                       False, tp._in1_offs, tp._in2_offs, tp._out_sizes, tp._n_paths_per_l,
                                       tp.n_total_paths, False, l1 > 0, True, True)
    elif case == "dense":
        tp = o3.TensorProduct(3, 3, 3, 128, 128, shared_weights=True)
        n = 27_648
        in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g, requires_grad=True)
        in2 = torch.randn(n, tp.in2_dim, device=dev, generator=g, requires_grad=True)
        w = torch.randn(tp.n_total_paths * 128, device=dev, generator=g)
        out = tp(in1, in2, w)
        torch.autograd.grad(out, [in1, in2], torch.randn_like(out))
    elif case == "linear_bf16":
        lin = o3.LinearLayer(3, 3, 128, 128, weight_scale=1.0).to(dev)
        x = torch.randn(400_000, 16 * 128, device=dev, generator=g).to(torch.bfloat16)
        with torch.no_grad():
            lin(x)
    else:
        lay = LinearLayer(64, 23 * 128).to(dev)
        for p_ in lay.parameters():
            p_.requires_grad_(False)
        h = torch.randn(200_000, 64, device=dev, generator=g, requires_grad=True)
        out = lay(h)
        torch.autograd.grad(out, [h], torch.randn_like(out))
    torch.cuda.synchronize()
    from flashcart_b200.ops import check_device_status
    check_device_status(dev)
    print(json.dumps({"op_case": case, "ok": True}))


def _event_ms(fn, reps: int, warmup: int) -> float:
    for _ in range(max(warmup, 1)):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(reps):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / reps


def _roof(nbytes: int, ms: float, peak: float, peak_src: str, traffic=None):
    ach = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s", "frac": ach / peak, "traffic": traffic,
            "peak_source": f"{peak_src} (hbm_gbs)", "bytes_per_launch": nbytes, "ms_per_launch": ms}


def run_config1(args):
    """Isolated tensor-product microbenchmark: TensorProduct(2, 2, 2, 64, 1) convolution, E = 2^20 edges over
    N = 2^16 nodes (receiver-sorted uniform indices), unit-vector moments scaled by
    N(0,1) radial weights as in2, N(0,1) node features and path weights, forward and
    backward with respect to in1, in2 and the weights; fp32."""
    from flashcart_b200 import o3, ops

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    n, e, c = 65536, 1048576, 64
    idx_i = torch.sort(torch.randint(0, n, (e,), device=dev, generator=g)).values
    idx_j = torch.randint(0, n, (e,), device=dev, generator=g)
    u = torch.randn(e, 3, device=dev, generator=g)
    in2 = (o3.Irreps(2).forward_normalized(u / u.norm(dim=-1, keepdim=True))
           * torch.randn(e, 1, device=dev, generator=g)).contiguous()
    tp = o3.TensorProduct(2, 2, 2, c, 1)
    in1 = torch.randn(n, tp.in1_dim, device=dev, generator=g)
    w = torch.randn(e, tp.n_total_paths * c, device=dev, generator=g)
    a = (idx_i, idx_j, 2, 2, 2, c, 1, False, False, tp._in1_offs, tp._in2_offs, tp._out_sizes, tp._n_paths_per_l,
         tp.n_total_paths, False)
    out = torch.ops.flashcart.tp_fwd(in1, in2, w, *a)
    gout = torch.randn_like(out)
    fwd = lambda: torch.ops.flashcart.tp_fwd(in1, in2, w, *a)
    bwd = lambda: torch.ops.flashcart.tp_bwd(gout, in1, in2, w, *a, True, True, True)
    reps = max(args.steps, 1)
    fwd_ms, bwd_ms = _event_ms(fwd, reps, args.warmup), _event_ms(bwd, reps, args.warmup)
    ops.check_device_status(dev)
    idx = 8 * (2 * e + n + 1)
    fwd_b = 4 * (in1.numel() + in2.numel() + w.numel() + out.numel()) + idx
    bwd_b = 4 * (gout.numel() + 2 * in1.numel() + 2 * in2.numel() + 2 * w.numel()) + idx
    peak, src = _peaks()
    ms = fwd_ms + bwd_ms
    print(json.dumps({
        "metric": "TP convolution (2,2)->2 forward + backward, E=2^20, N=2^16, C=64",
        "value": e / (ms * 1e-3), "unit": "edges/s", "n_gpus": 1, "steps": reps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": "f32", "data": "synthetic",
        "config": {"workload": "isolated TP convolution microbenchmark", "edges": e, "nodes": n, "channels": c, "paths": tp.n_total_paths,
                   "l2": "inputs larger than L2 (weights 2.9 GB)"},
        "roofline": {"fwd": _roof(fwd_b, fwd_ms, peak, src), "bwd": _roof(bwd_b, bwd_ms, peak, src)},
    }), flush=True)


def run_config2(args):
    """Edge expansion + equivariant linear map: 2,000,000 edge vectors uniform in a 5 A ball; moments T^l(r^),
    l <= 3, times h = Linear(8 -> 128)(Bessel(8, 5 A)(r) * cutoff_6(r)) laid out as
    (E, 2048), then o3.LinearLayer(3, 3, 128, 128) with Xavier-normal weights and
    weight_scale 1 (3xTF32 tensor-core path); forward, fp32."""
    from flashcart_b200 import o3, ops
    from flashcart_b200.nn.layers import LinearLayer
    from flashcart_b200.nn.radial import BesselBasis, PolynomialCutoff

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    e, C = 2_000_000, 128
    d = torch.randn(e, 3, device=dev, generator=g)
    d = d / d.norm(dim=-1, keepdim=True)
    r = 5.0 * torch.rand(e, device=dev, generator=g) ** (1.0 / 3.0)
    v = d * r.unsqueeze(-1)
    v = v[v.norm(dim=-1) >= 1e-4].contiguous()
    e = v.shape[0]
    torch.manual_seed(0)
    lay = LinearLayer(8, C).to(dev)
    lin = o3.LinearLayer(3, 3, C, C, weight_scale=1.0).to(dev)
    with torch.no_grad():
        for wl in lin.weight:
            wl.normal_(0.0, (2.0 / (C + C)) ** 0.5)
    basis, cut, irr = BesselBasis(8, 5.0).to(dev), PolynomialCutoff(5.0, 6).to(dev), o3.Irreps(3)
    sizes = [(2 * l + 1) for l in range(4)]

    def expand():
        rr = v.norm(dim=-1)
        T = irr.forward_normalized(v / rr.unsqueeze(-1))
        h = lay(basis(rr) * cut(rr).unsqueeze(-1))
        blocks = torch.split(T, sizes, dim=1)
        return torch.cat([(b.unsqueeze(-1) * h.unsqueeze(1)).reshape(e, -1) for b in blocks], dim=-1)

    # fused: Y_l = T_l (x) (h W_l^T) -- one 128 -> 4 x 128 GEMM on h, then one pass writing Y
    wcat = LinearLayer(C, 4 * C, weight_scale=1.0).to(dev)
    with torch.no_grad():
        wcat.weight.copy_(torch.cat([wl for wl in lin.weight], dim=0))

    def fused():
        rr = v.norm(dim=-1)
        T = irr.forward_normalized(v / rr.unsqueeze(-1))
        u = wcat(lay(basis(rr) * cut(rr).unsqueeze(-1)))
        return ops.edge_expand_fwd(T, u.view(e, 4, C), 3, C, True)

    with torch.no_grad():
        x = expand()
        reps = max(args.steps, 1)
        exp_ms = _event_ms(expand, reps, args.warmup)
        lin_ms = _event_ms(lambda: lin(x), reps, args.warmup)
        y_ref = lin(x)
        # bf16 storage path of the same map: bf16 in / out, fp32 accumulation on tcgen05
        x_bf = x.to(torch.bfloat16)
        del x
        bf16_ms = _event_ms(lambda: lin(x_bf), reps, args.warmup)
        bf16_rel = ((lin(x_bf).float() - y_ref).abs().max() / y_ref.abs().max()).item()
        del x_bf
        y = fused()
        rel = ((y - y_ref).abs().max() / y_ref.abs().max()).item()
        del y, y_ref
        torch.cuda.empty_cache()
        fused_ms = _event_ms(fused, reps, args.warmup)
    ops.check_device_status(dev)
    peak, src = _peaks()
    ms = exp_ms + lin_ms
    xb = e * 16 * C * 4
    print(json.dumps({
        "metric": "edge expansion + equivariant linear map 128->128, l<=3, 2,000,000 edges",
        "value": e / (ms * 1e-3), "unit": "edges/s", "n_gpus": 1, "steps": reps, "warmup": args.warmup,
        "ms_per_step": ms, "higher_is_better": True, "dtype": "f32 (linear map: 3xTF32 tensor cores)",
        "data": "synthetic", "config": {"workload": "edge expansion + equivariant linear map", "edges": e, "channels": C,
                                         "expansion": "unfused reference composition (torch) writing (E, 2048)"},
        "roofline": {"expansion": _roof(e * 12 + xb, exp_ms, peak, src), "linear": _roof(2 * xb, lin_ms, peak, src)},
        "linear_bf16": {"ms": bf16_ms, "how": "x, W, y in bf16, tcgen05 kind::f16 with fp32 accumulation",
                        "max_rel_diff_vs_fp32": bf16_rel, "roofline": _roof(xb, bf16_ms, peak, src)},
        "fused": {"ms_per_step": fused_ms, "value": e / (fused_ms * 1e-3), "unit": "edges/s",
                  "how": "Y_l = T_l (x) (h W_l^T): GEMM 128 -> 4 x 128 (3xTF32) on h, fc_edge_expand_fwd writes Y",
                  "max_rel_diff_vs_unfused": rel,
                  "roofline": _roof(e * 12 + xb, fused_ms, peak, src)},
    }), flush=True)


def run_config4(args):
    """Data-parallel training. Per GPU and step 32 seeded random-walk
    molecules (20-60 atoms, H/C/N/O 50/30/10/10, seed 1000 rank + step); labels from a
    random-init teacher (config-0 architecture, elements H/C/N/O, seed 1); the student
    (seed 0) takes the energy-per-atom + force MSE with forces from create_graph=True (the
    operators' double backward), one flat NCCL all-reduce of the gradients, then AdamW +
    Muon (Newton-Schulz on the tensor cores). Batches and labels are built before the
    timed region; value = molecules (and atoms) of all ranks / max-over-ranks step time."""
    import torch.distributed as dist

    from flashcart_b200 import ops, training
    from flashcart_b200.model.flashcart import FlashCartPotential

    rank, world, local = _dist_env()
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    kw = dict(elements=training.ELEMENTS, r_max=5.0, n_hidden_feats=64, l_max_hidden_feats=2, l_max_edge_attrs=2,
              n_radial=8, n_interactions=2, correlation=3, layer_norm=True, nonlinearity=True,
              gate_activation="sigmoid", radial_mapping="cosine", path_reduced_product=False,
              fit_atomic_shifts=False, atomic_shifts=[0.0] * 4)
    n_steps = max(args.warmup, 0) + max(args.steps, 1)
    graphs = [training.batch_graph(training.synthetic_molecules(32, rank=rank, step=st), 5.0, dev)
              for st in range(n_steps)]
    avg = graphs[0]["edge_index"].shape[1] / graphs[0]["positions"].shape[0]  # mean degree of the first batch
    torch.manual_seed(1)
    teacher = FlashCartPotential(**kw, avg_neighbors=avg).to(dev)
    torch.manual_seed(0)
    student = FlashCartPotential(**kw, avg_neighbors=avg).to(dev)
    opts = training.make_optimizer(student)
    buckets = training.GradientBuckets(student) if (world > 1 and args.allreduce == "buckets") else None
    batches = []
    for g in graphs:
        lab = teacher.predict(g, compute_forces=True)
        batches.append((g, lab["energy"].detach(), lab["forces"].detach()))
    n_atoms = [int(b[0]["positions"].shape[0]) for b in batches]
    for st in range(args.warmup):
        training.train_step(student, *batches[st], opts, buckets=buckets)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for st in range(args.warmup, n_steps):
        loss = training.train_step(student, *batches[st], opts, buckets=buckets)
    e1.record()
    torch.cuda.synchronize()
    ops.check_device_status(dev)
    ms = e0.elapsed_time(e1) / max(args.steps, 1)
    t = torch.tensor([ms, float(sum(n_atoms[args.warmup:]))], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t[0:1], op=dist.ReduceOp.MAX)
        dist.all_reduce(t[1:2], op=dist.ReduceOp.SUM)
    ms_max, atoms = float(t[0]), float(t[1])
    if rank == 0:
        mols_per_s = 32 * world / (ms_max * 1e-3)
        print(json.dumps({
            "metric": "DP training structures/s (32 molecules of 20-60 atoms per GPU, E+F loss, Muon)",
            "value": mols_per_s, "unit": "structures/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "weak", "dtype": "f32", "data": "synthetic",
            "atom_steps_per_s": atoms / max(args.steps, 1) / (ms_max * 1e-3), "final_loss": float(loss),
            "config": {"workload": "data-parallel training", "molecules_per_gpu": 32, "parallelism": f"dp{world}",
                       "allreduce": args.allreduce if world > 1 else "none",
                       "model": "64 channels, ranks <= 2 (the 192-atom CPU run's architecture), elements H/C/N/O"},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = _args()
    if args.config == 4:
        run_config4(args)
    elif args.config == 1:
        run_config1(args)
    elif args.config == 2:
        run_config2(args)
    elif args.op_case is not None:
        run_op_case(args.op_case)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
