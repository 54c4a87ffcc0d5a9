#!/usr/bin/env python
"""Benchmark: forward edges/s of WignerDBasis + EquivariantEdgewiseLinear
(benchmark config 2) on B200, with roofline, clocks, end-to-end and CPU baseline.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the headline benchmark configuration): in/out Repr(lvals=[0..4], mult=64), N = 20000
nodes uniform in a 60 A cube, 32-nearest-neighbour graph (src over the neighbours
of dst), E = 640000, node features (N, 64, 25) ~ N(0, 1) gathered to edges by
src, directions = dst - src, num_bins = 100 over [0, 10], float32, seed 1.
Synthetic data (the reference benchmarks on random graphs too); module weights
random-init with torch.manual_seed(1).

One step = P, Q = WignerDBasis(directions); out = layer(P, Q, x[src], distances),
with the layer's radial mix on the tensor cores (--mix bf16x3, the default: every
operand split into two bf16 terms, float32-level accuracy; --mix bf16: the bf16-mix
path; --mix fp32: CUDA-core float32), inputs resident in HBM (4.1 GB of edge features per step >> 126 MB L2, so no
flush is needed).  Under torchrun (N > 1) every rank runs its own independent
graph (seed 1 + rank): data-parallel, no collective on the data path, weak scaling.

--impl reference times the reference algorithm on the host cores: the CPU
restatement in oracle/ (batched matrix_exp basis, bmm, block-diagonal mix, bmm;
the reference has no CPU kernel of its own), on a bounded sample of the same
workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "flash-eq_b200"))

import torch  # noqa: E402

LVALS = [0, 1, 2, 3, 4]
MULT = 64
N_NODES = 20000
K_NN = 32
BOX = 60.0
NUM_BINS = 100
MAX_DIST = 10.0
SEED = 1

# One metric string per workload, printed by both arms (ours and --impl reference), so the
# two lines can be compared directly.
METRIC_CONFIG2 = "edges/sec (WignerDBasis + EquivariantEdgewiseLinear fwd)"
METRIC_BLOCK = "edges/sec (EquivariantTransformerBlock fwd)"


# ---------------------------------------------------------------------------
# Workload
# ---------------------------------------------------------------------------
def knn_graph(coords: torch.Tensor, k: int, chunk: int = 4096):
    """src -> dst: src ranges over the k nearest neighbours (no self) of each dst."""
    n = coords.shape[0]
    nbrs = []
    for s in range(0, n, chunk):
        d = torch.cdist(coords[s:s + chunk], coords)
        idx = torch.arange(s, min(n, s + chunk), device=coords.device)
        d[torch.arange(len(idx), device=coords.device), idx] = float("inf")
        nbrs.append(d.topk(k, dim=1, largest=False).indices)
    nbr = torch.cat(nbrs)
    dst = torch.arange(n, device=coords.device).repeat_interleave(k)
    return nbr.reshape(-1), dst


def make_workload(seed: int, device, n_nodes: int = N_NODES):
    """Nodes uniform in a cube of side BOX * (n_nodes / N_NODES)^(1/3) (constant density)."""
    g = torch.Generator().manual_seed(seed)
    coords = torch.rand(n_nodes, 3, generator=g) * (BOX * (n_nodes / N_NODES) ** (1.0 / 3.0))
    x = torch.randn(n_nodes, MULT, sum(2 * l + 1 for l in LVALS), generator=g)
    coords_d = coords.to(device)
    src, dst = knn_graph(coords_d, K_NN)
    return {"coords": coords, "x": x, "coords_d": coords_d, "x_d": x.to(device), "src": src, "dst": dst}


def build_modules(device):
    import flash_eq as fe

    torch.manual_seed(SEED)
    r = fe.Repr(LVALS, mult=MULT)
    layer = fe.EquivariantEdgewiseLinear(r, r, num_bins=NUM_BINS, min_dist=0.0, max_dist=MAX_DIST).to(device)
    layer.eval()
    basis = fe.WignerDBasis([r, r]).to(device)
    return layer, basis


def per_edge_work():
    """Algorithmic bytes and flops per edge (fp32 I/O) of the edgewise linear."""
    d = sum(2 * l + 1 for l in LVALS)
    byts = MULT * d * 4 * 2 + 16
    mix = 0
    for m in range(max(LVALS) + 1):
        n = sum(1 for l in LVALS if l >= m)
        mix += 2 * MULT * MULT * n * n * (1 if m == 0 else 4)
    rot = 2 * 2 * MULT * sum((2 * l + 1) ** 2 for l in LVALS)
    table_bytes = (NUM_BINS + 1) * MULT * MULT * sum(2 * min(a, b) + 1 for a in LVALS for b in LVALS) * 4
    return byts, mix, rot, table_bytes


# ---------------------------------------------------------------------------
# Clocks sampler (nvidia-smi during the timed region)
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu_index = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu_index)],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
        except (OSError, ValueError):
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        mhz, mx, reasons, power = [], None, set(), []
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                mhz.append(float(parts[1]))
                mx = float(parts[2])
                power.append(float(parts[3]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(mhz), "power_w_max": max(power) if power else None}


def measured_sustained():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            return float(json.load(fh)["bf16_tflops_sustained"])
    except (OSError, KeyError, ValueError):
        return None


def profiled_traffic(stage: str, E: int):
    """DRAM bytes (read + write) of one step's launches of `stage`, from the committed ncu
    summary profiles/<stage>_config2.md ("dram_bytes_per_edge: X"), scaled to E edges."""
    path = os.path.join(ROOT, "profiles", f"{stage}_config2.md")
    try:
        with open(path) as fh:
            for ln in fh:
                if ln.strip().startswith("dram_bytes_per_edge:"):
                    return float(ln.split(":", 1)[1]) * E
    except (OSError, ValueError):
        pass
    return None


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as fh:
            pk = json.load(fh)
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, 1590.0, "fallback"


# ---------------------------------------------------------------------------
# CPU baseline: the reference algorithm on the host cores (oracle port)
# ---------------------------------------------------------------------------
def cpu_reference_setup(sample_edges: int):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle as orc

    wl = _cpu_workload()
    layer, _ = build_modules("cpu")
    with torch.no_grad():
        table = layer.radial_weights()
    p1, p2 = layer.radial_weights.binning_params()
    src, dst = wl["src"], wl["dst"]
    sel = torch.arange(min(sample_edges, src.numel()))
    vec = wl["coords"][dst[sel]] - wl["coords"][src[sel]]
    ef = wl["x"][src[sel]]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    def step():
        dist = vec.norm(dim=-1)
        P = orc.wigner_basis(vec, LVALS)
        return orc.edgewise_fwd(P, P, ef, dist, table, LVALS, LVALS, layer.solid_harmonic_scale, p1, p2,
                                NUM_BINS, False, nthreads=threads)

    return step, int(sel.numel()), threads


def parity_rows(dist: torch.Tensor, p1: float, p2: float, num_bins: int, n_rows: int = 16384, seed: int = 0):
    """A fixed sample of edge ids for the parity check of a timed output: up to 48 edges of
    every distance bin present, up to 2048 of the most populated bin, the rest drawn
    uniformly (seeded), n_rows in all, sorted.  Linear bins, as the workload uses."""
    dist = dist.detach().float().cpu()
    E = dist.numel()
    lo = ((dist - p1) * p2).clamp(0.0, float(num_bins)).floor().long().clamp(max=num_bins - 1)
    order = torch.argsort(lo, stable=True)
    counts = torch.bincount(lo, minlength=num_bins)
    starts = torch.cumsum(counts, 0) - counts
    picks = []
    for b in torch.nonzero(counts).flatten().tolist():
        picks.append(order[starts[b]:starts[b] + min(48, int(counts[b]))])
    top = int(torch.argmax(counts))
    picks.append(order[starts[top]:starts[top] + min(2048, int(counts[top]))])
    sel = torch.unique(torch.cat(picks))
    if sel.numel() < min(n_rows, E):
        taken = torch.zeros(E, dtype=torch.bool)
        taken[sel] = True
        rest = torch.randperm(E, generator=torch.Generator().manual_seed(seed))
        rest = rest[~taken[rest]][: min(n_rows, E) - sel.numel()]
        sel = torch.cat([sel, rest])
    return torch.sort(sel).values, int((counts > 0).sum())


def parity_vs_oracle(y_rows, f_rows, vec_rows, dist_rows, table, lvals, sh_scale, p1, p2, num_bins):
    """Relative L2 error of output rows y_rows against the CPU restatement of the reference
    path (matrix_exp basis, bmm, block-diagonal mix, bmm) in float64 on the same rows."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle as orc

    P = orc.wigner_basis(vec_rows.double().cpu(), lvals)
    ref = orc.edgewise_fwd(P, P, f_rows.double().cpu(), dist_rows.double().cpu(), table.double().cpu(), lvals,
                           lvals, sh_scale, p1, p2, num_bins, False)
    return float((y_rows.double().cpu() - ref).norm() / ref.norm())


_CPU_WL = {}


def _cpu_workload():
    if "wl" not in _CPU_WL:
        _CPU_WL["wl"] = make_workload(SEED, "cpu")
    return _CPU_WL["wl"]


def cpu_model():
    try:
        with open("/proc/cpuinfo") as fh:
            for ln in fh:
                if ln.startswith("model name"):
                    return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def time_cpu(step, n, reps):
    step()
    t0 = time.perf_counter()
    for _ in range(reps):
        step()
    return (time.perf_counter() - t0) / reps


def pick_cpu_sample(target_s: float = 2.0):
    """Size the per-step sample so one step takes about target_s seconds."""
    step, n, threads = cpu_reference_setup(256)
    t = time_cpu(step, n, 1)
    per_edge = t / n
    return max(256, min(640000, int(target_s / max(per_edge, 1e-9)))), threads


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    sample, threads = pick_cpu_sample(2.0)
    step, n, threads = cpu_reference_setup(sample)
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    value = n / dt
    line = {
        "metric": METRIC_CONFIG2, "impl": "reference", "value": value, "unit": "edges/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": config_block(args.gpus),
        "cpu_baseline": {"value": value, "unit": "edges/s", "cores": threads, "kind": "port",
                         "sample": f"{n} edges of the config-2 workload per step (CPU: {cpu_model()})"},
        "e2e": {"value": value, "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def config_block(n_gpus, n_nodes=N_NODES):
    if LVALS != [0, 1, 2, 3, 4]:
        return {"workload": f"variant: config-2 graph (N={n_nodes}) with Repr({LVALS}, {MULT}) in and out",
                "edges_per_gpu": n_nodes * K_NN, "global_edges": n_nodes * K_NN * n_gpus}
    if n_nodes != N_NODES:
        return {"workload": f"profiling case: config-2 shapes with N={n_nodes} nodes, E={n_nodes * K_NN}",
                "edges_per_gpu": n_nodes * K_NN, "global_edges": n_nodes * K_NN * n_gpus}
    return {"workload": "config2: WignerDBasis + EquivariantEdgewiseLinear forward, Repr([0,1,2,3,4],64) -> same, "
                        "N=20000 uniform 60A cube, 32-NN, E=640000 per GPU, 100 bins over [0,10]",
            "edges_per_gpu": N_NODES * K_NN, "global_edges": N_NODES * K_NN * n_gpus,
            "parallelism": f"dp{n_gpus} (independent graph per GPU)",
            "l2": "no flush: 4.1 GB of edge features read per step >> 126 MB L2"}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    pg = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        # communicator set-up lines (rank, device, transport) in the log, even where the
        # environment asks only for the version line
        if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
            os.environ["NCCL_DEBUG"] = "INFO"
        os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
        pg = dist
    return world, rank, local, pg


def barrier(pg):
    if pg is not None:
        pg.barrier()
    torch.cuda.synchronize()


def max_over_ranks(pg, v: float) -> float:
    if pg is None:
        return v
    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    pg.all_reduce(t, op=pg.ReduceOp.MAX)
    return float(t.item())


def gpu_index_for(local: int) -> int:
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    if vis:
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        if local < len(ids) and ids[local].isdigit():
            return int(ids[local])
    return local


def run_ours(args):
    world, rank, local, pg = dist_setup(args)
    dev = torch.device("cuda", local)
    from flash_eq.cuda import _lib

    lib = _lib.load()
    wl = make_workload(SEED + rank, dev, args.nodes)
    layer, basis = build_modules(dev)
    layer.mix_precision = args.mix
    src, dst, x, coords = wl["src"], wl["dst"], wl["x_d"], wl["coords_d"]
    E = src.numel()
    vec = coords[dst] - coords[src]
    dist_e = vec.norm(dim=-1)

    def step():
        with torch.no_grad():
            P, Q = basis(vec)
            return layer(P, Q, x[src], dist_e)

    # nvidia-smi takes ~0.1 s to its first sample: started before the warm-up, it covers the
    # (short) timed region too
    clk = ClockSampler(gpu_index_for(local))
    clk.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # the step replayed as one CUDA graph, as the block workload does (the library's ops are
    # stream-ordered and allocate through torch's caching allocator): the same kernels without
    # the host's launch gaps; the eager step is timed too and reported as ms_eager
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step()
    torch.cuda.current_stream().wait_stream(side)
    cg = torch.cuda.CUDAGraph()
    n_cap = lib.feq_launch_count()
    with torch.cuda.graph(cg):
        step()
    per_replay = lib.feq_launch_count() - n_cap
    for _ in range(args.warmup):
        cg.replay()

    def timed(fn, steps):
        barrier(pg)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier(pg)
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        barrier(pg)
        return max_over_ranks(pg, t0.elapsed_time(t1) / steps)

    torch.cuda.profiler.start()      # lets `ncu --profile-from-start off` capture just the timed steps
    ms = timed(cg.replay, args.steps)
    torch.cuda.profiler.stop()
    launches = per_replay * args.steps
    clocks = clk.stop()
    # eager steps warmed up again first: the graph's private memory pool was filled since the
    # last eager step, and the first eager steps after it pay the allocator's new segments
    for _ in range(3):
        step()
    ms_eager = timed(step, max(3, args.steps // 4))
    del cg
    value = E * world / (ms / 1e3)

    # --- per-stage device times: CUDA events the library records on the stream each
    # stage is launched on, over a few extra steps after the timed region
    from flash_eq.cuda import ops as feq_ops

    prof_steps = 3
    feq_ops.profile_enable(True)
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    stages = feq_ops.profile_read()
    feq_ops.profile_enable(False)
    byts, mix_flops, rot_flops, table_bytes = per_edge_work()
    d = sum(2 * l + 1 for l in LVALS)
    nsplit = 2 if args.mix == "bf16x3" else 1
    tensor_mult = {"bf16x3": 6, "bf16": 2}.get(args.mix, 0)     # bf16 MMAs per algorithmic MAC
    stage_bytes = {                                                # algorithmic bytes per edge
        "basis": d * d * 4 + 12,
        "rotate_in": MULT * d * 4 + 28 + 4 + MULT * d * 2 * nsplit,
        "rotate_out": MULT * d * 4 * 2 + 24,
        "tc_mix": MULT * d * 2 * nsplit + MULT * d * 4 + 4,
        "sep_edgewise": byts,                                      # the fused path's own bytes
    }
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    tc_sustained = measured_sustained() or tc_peak
    per_step = {k: {"ms": v[0] / prof_steps, "launches": v[1] // prof_steps} for k, v in stages.items()}
    dom = max(per_step, key=lambda k: per_step[k]["ms"]) if per_step else None
    roofline = None
    if dom == "tc_mix":
        t = per_step[dom]["ms"] / 1e3
        alg = E * mix_flops / t / 1e12
        exe = alg * tensor_mult
        roofline = {"bound": "tensor", "achieved": alg, "peak": tc_sustained, "unit": "TFLOP/s",
                    "frac": alg / tc_sustained, "traffic": profiled_traffic("tc_mix", E),
                    "traffic_source": "committed ncu summary profiles/tc_mix_config2.md (DRAM bytes per edge, "
                                      "scaled to E); not measured in this run",
                    "kernel": f"tc_mix ({per_step[dom]['launches']} launches per step, one per m-block), "
                              f"CUDA events on its stream, {prof_steps} steps",
                    "peak_kind": "measured bf16 sustained (MEASURED_PEAKS.json)",
                    "executed_tflops": exe, "executed_frac": exe / tc_sustained,
                    "note": f"achieved counts the algorithmic mix FLOPs; the {args.mix} formulation executes "
                            f"{tensor_mult} bf16 MMA FLOPs per algorithmic FLOP (two neighbouring bins"
                            + (", 3-term hi/lo split" if args.mix == "bf16x3" else "") + ")"}
    elif dom == "sep_edgewise":
        t = per_step[dom]["ms"] / 1e3
        gbs = E * byts / t / 1e9
        es = 16 if d <= 16 else 32
        exe = E * 4 * MULT * es * MULT * 2 * {"bf16x3": 3, "bf16": 1}.get(args.mix, 0) / t / 1e12
        roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                    "traffic": profiled_traffic("sep_edgewise", E), "kernel": f"sep_edgewise (one launch per step: gather rows in, rotation, "
                                              f"separable mix on tcgen05, rotation back, rows out), CUDA events on "
                                              f"its stream, {prof_steps} steps",
                    "peak_kind": f"{peak_kind} HBM copy bandwidth (MEASURED_PEAKS.json)",
                    "bytes_per_edge": byts,
                    "traffic_source": "committed ncu summary profiles/sep_edgewise_config2.md (DRAM bytes per edge of a "
                                      "small case of this workload, scaled to E); not measured in this run",
                    "alg_mix_tflops": E * mix_flops / t / 1e12,
                    "executed_tensor_tflops": exe, "executed_tensor_frac": exe / tc_sustained}
    elif dom is not None:
        t = per_step[dom]["ms"] / 1e3
        gbs = E * stage_bytes.get(dom, 0) / t / 1e9
        roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                    "traffic": profiled_traffic(dom, E), "kernel": dom, "peak_kind": peak_kind,
                    "traffic_source": f"committed ncu summary profiles/{dom}_config2.md (DRAM bytes per edge, "
                                      "scaled to E); not measured in this run"}
    for k, v in per_step.items():
        if k in stage_bytes and k != "tc_mix":
            v["hbm_gbs"] = E * stage_bytes[k] / (v["ms"] / 1e3) / 1e9
    if "tc_mix" in per_step:
        per_step["tc_mix"]["alg_tflops"] = E * mix_flops / (per_step["tc_mix"]["ms"] / 1e3) / 1e12
    step_gbs = value / world * byts / 1e9
    step_roofline = {"bound": "hbm", "achieved": step_gbs, "peak": hbm_peak, "unit": "GB/s",
                     "frac": step_gbs / hbm_peak, "bytes_per_edge": byts,
                     "note": "whole step against the fused-path algorithmic bytes per edge "
                             "(input row + output row + 16 B, fp32)"}

    # --- parity of the timed computation: one more step, a fixed row sample (every distance
    # bin present, the most populated bin) against the float64 CPU restatement (oracle)
    parity = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        with torch.no_grad():
            y = step()
        rw = layer.radial_weights
        p1, p2 = rw.binning_params()
        sel, nbins = parity_rows(dist_e, p1, p2, rw.num_bins)
        sel_d = sel.to(dev)
        with torch.no_grad():
            table = rw()
        err = parity_vs_oracle(y[sel_d], x[src[sel_d]], vec[sel_d], dist_e[sel_d], table, LVALS,
                               layer.solid_harmonic_scale, p1, p2, rw.num_bins)
        tol = 2e-2 if args.mix == "bf16" else 1e-4
        parity = {"rel_l2": err, "tolerance": tol, "ok": err < tol, "rows": int(sel.numel()),
                  "bins_covered": nbins, "against": "CPU restatement of the reference path in float64 "
                                                   "(oracle/), same inputs, one step's output"}
        del y

    # --- end to end through the public API from pinned host buffers
    e2e = run_e2e(args, wl, layer, basis, dev, pg, world) if args.e2e_steps > 0 else None

    result = None
    if rank == 0:
        result = {
            "metric": METRIC_CONFIG2, "value": value, "unit": "edges/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "ms_eager": ms_eager,
            "timing": "CUDA-graph replay of the step (ms_eager: the same step launched eagerly)",
            "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16" if args.mix == "bf16" else "f32",
            "data": "synthetic", "config": config_block(world, args.nodes),
            "roofline": roofline,
            "step_roofline": step_roofline,
            "stages_ms_per_step": per_step,
            "mix": args.mix,
            "clocks": clocks,
            "e2e": e2e,
            "gpu_launches": int(launches),
        }
        if world == 1 and not args.no_cpu_baseline:
            result["parity"] = parity
        if world == 1 and not args.no_cpu_baseline and args.nodes == N_NODES:
            try:
                sample, threads = pick_cpu_sample(3.0)
                cstep, n, threads = cpu_reference_setup(sample)
                dt = time_cpu(cstep, n, 3)
                result["cpu_baseline"] = {"value": n / dt, "unit": "edges/s", "cores": threads, "kind": "port",
                                          "sample": f"{n} edges of the same workload, 3 reps "
                                                    f"(CPU: {cpu_model()})"}
            except Exception as exc:  # the baseline must not hide the GPU number
                result["cpu_baseline"] = {"value": None, "error": repr(exc)}
    if world > 1 and not args.no_config5:
        # the scaling run of this default workload exercises no collective (independent graphs);
        # the same run also measures config 5 (one graph, dst-range partition, NCCL halo
        # exchange per layer) at this GPU count, with its exchange time and stage table
        del wl, x, src, coords, vec, dist_e
        torch.cuda.empty_cache()
        rec5 = giant_measure(args, world, rank, local, pg, GIANT_NODES, 10, 3, 0)
        if rank == 0:
            result["config5_partitioned"] = rec5
    if rank == 0:
        print(json.dumps(result), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def run_e2e(args, wl, layer, basis, dev, pg, world):
    """Same step through the public API with host buffers: H2D of the step's
    inputs from pinned memory and D2H of the full output, inside the timed region."""
    x_h = wl["x"].pin_memory()
    c_h = wl["coords"].pin_memory()
    s_h, d_h = wl["src"].cpu().pin_memory(), wl["dst"].cpu().pin_memory()
    E = s_h.numel()
    d_out = sum(2 * l + 1 for l in LVALS)
    out_h = torch.empty(E, MULT, d_out, pin_memory=True)

    # The edges go through in chunks so the device->host copy of one chunk's output (on a
    # second stream) overlaps the computation of the next.
    n_chunks = max(1, args.e2e_chunks)
    bounds = [E * i // n_chunks for i in range(n_chunks + 1)]
    copy_stream = torch.cuda.Stream(device=dev)

    def step():
        x = x_h.to(dev, non_blocking=True)
        c = c_h.to(dev, non_blocking=True)
        s, d = s_h.to(dev, non_blocking=True), d_h.to(dev, non_blocking=True)
        for a, b in zip(bounds[:-1], bounds[1:]):
            with torch.no_grad():
                v = c[d[a:b]] - c[s[a:b]]
                P, Q = basis(v)
                y = layer(P, Q, x[s[a:b]], v.norm(dim=-1))
            done = torch.cuda.Event()
            done.record()
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(done)
                out_h[a:b].copy_(y, non_blocking=True)
                y.record_stream(copy_stream)
        torch.cuda.current_stream().wait_stream(copy_stream)

    steps = args.e2e_steps
    step()
    barrier(pg)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    barrier(pg)
    ms = max_over_ranks(pg, t0.elapsed_time(t1) / steps)
    h2d = x_h.numel() * 4 + c_h.numel() * 4 + s_h.numel() * 8 + d_h.numel() * 8
    return {"value": E * world / (ms / 1e3), "unit": "edges/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": out_h.numel() * 4, "ms_per_step": ms, "steps": steps, "chunks": n_chunks}


# Published single-layer numbers of the reference (fwd + bwd + Adam, float32, H100, C = 32,
# 64 bins): (lmax, edges) -> ms per step, README.md:281-290 of hmblair/flash-eq.
PUBLISHED_TRAIN_MS = {(1, 32000): 5.3, (2, 32000): 11.5, (4, 5000): 7.1, (6, 5000): 14.7, (4, 20000): 21.5,
                      (6, 20000): 50.6, (4, 50000): 50.1, (6, 50000): 123.5, (4, 128000): 125.6,
                      (6, 128000): 309.7}


def run_train(args):
    """The reference's published single-layer training step (its benchmarks/compare_all.py
    harness, restated): EquivariantEdgewiseLinear(Repr(0..L, 32)), 64 bins over [0, 10],
    random unit directions, U[0, 10] distances, MSE to a random target, Adam."""
    import flash_eq as fe

    world, rank, local, pg = dist_setup(args)
    dev = torch.device("cuda", local)
    lmax, E, C = args.lmax, args.edges, 32
    torch.manual_seed(SEED + rank)
    r = fe.Repr(list(range(lmax + 1)), mult=C)
    layer = fe.EquivariantEdgewiseLinear(r, r, num_bins=64, min_dist=0.0, max_dist=10.0).to(dev)
    layer.mix_precision = args.mix if args.mix != "fp32" else "bf16x3"
    basis = fe.WignerDBasis([r, r]).to(dev)
    opt = torch.optim.Adam(layer.parameters(), lr=1e-4)
    g = torch.Generator(device=dev).manual_seed(SEED + rank)
    feats = torch.randn(E, C, r.dim(), device=dev, generator=g).requires_grad_()
    dirs = torch.randn(E, 3, device=dev, generator=g)
    dirs = dirs / dirs.norm(dim=-1, keepdim=True)
    dists = torch.rand(E, device=dev, generator=g) * 10.0
    target = torch.randn(E, C, r.dim(), device=dev, generator=g)
    P, Q = basis(dirs)

    def step():
        opt.zero_grad()
        out = layer(P, Q, feats, dists)
        loss = ((out - target) ** 2).mean()
        loss.backward()
        opt.step()

    for _ in range(args.warmup):
        step()
    barrier(pg)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    barrier(pg)
    ms = max_over_ranks(pg, t0.elapsed_time(t1) / args.steps)
    if rank == 0:
        pub = PUBLISHED_TRAIN_MS.get((lmax, E))
        print(json.dumps({
            "metric": "edges/sec (fwd+bwd+Adam, EquivariantEdgewiseLinear)", "value": E * world / (ms / 1e3),
            "unit": "edges/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "mix": layer.mix_precision,
            "config": {"workload": f"reference single-layer training step: Repr(0..{lmax}, 32), E={E}, 64 bins",
                       "edges_per_gpu": E},
            "published_reference_ms_h100": pub,
            "note": "published number is the reference on an H100 (README), context only"}), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# benchmark config 3: EquivariantTransformerBlock forward on batched small graphs
# ---------------------------------------------------------------------------
BLOCK_GRAPHS, BLOCK_NODES, BLOCK_RADIUS, BLOCK_HEADS, BLOCK_SEED = 256, 30, 5.0, 8, 2


def make_block_workload(seed, device):
    """256 molecule-like graphs of 30 nodes, coordinates N(0, 1.5^2) per axis, all directed
    pairs within 5 A (no self loops), features (N, 64, 9) ~ N(0, 1): benchmark config 3."""
    g = torch.Generator().manual_seed(seed)
    coords = torch.randn(BLOCK_GRAPHS, BLOCK_NODES, 3, generator=g) * 1.5
    x = torch.randn(BLOCK_GRAPHS * BLOCK_NODES, 64, 9, generator=g)
    # squared distance as the float32 expression (dx*dx + dy*dy) + dz*dz against r*r, the
    # cut-off Graph.radius applies on the GPU (same edge set bit for bit)
    dv = coords[:, None, :, :] - coords[:, :, None, :]                 # [g, a, b] = x_b - x_a
    d2 = (dv[..., 0] * dv[..., 0] + dv[..., 1] * dv[..., 1]) + dv[..., 2] * dv[..., 2]
    r2 = torch.tensor(BLOCK_RADIUS, dtype=torch.float32) * torch.tensor(BLOCK_RADIUS, dtype=torch.float32)
    mask = (d2 < r2) & ~torch.eye(BLOCK_NODES, dtype=torch.bool)[None]
    gi, a, b = torch.nonzero(mask, as_tuple=True)
    src, dst = gi * BLOCK_NODES + a, gi * BLOCK_NODES + b     # src -> dst within each graph
    return {"coords": coords.reshape(-1, 3), "x": x, "src": src, "dst": dst}


def build_block(device):
    import flash_eq as fe

    torch.manual_seed(BLOCK_SEED)
    r = fe.Repr([0, 1, 2], mult=64)
    blk = fe.EquivariantTransformerBlock(r, r, num_heads=BLOCK_HEADS, max_dist=MAX_DIST).to(device).eval()
    return blk, fe.WignerDBasis([r]).to(device), r


def block_step_fn(blk, basis, graph, coords, x):
    def step():
        with torch.no_grad():
            vec = coords[graph.src] - coords[graph.dst]           # src - dst (transformer.py:406)
            P = basis.lazy(vec)[0]
            return blk(P, P, x, vec.norm(dim=-1), graph)
    return step


def cpu_block_setup(n_graphs):
    """The reference algorithm of the block on the host cores: the module's node-level parts
    in PyTorch and the attention layer restated with the oracle (matrix_exp basis, bmm,
    block-diagonal mix, bmm, scatter softmax, scatter pooling), on n_graphs graphs."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle as orc
    import flash_eq as fe

    wl = make_block_workload(BLOCK_SEED, "cpu")
    blk, _, r = build_block("cpu")
    lv = [0, 1, 2]
    nn_ = n_graphs * BLOCK_NODES
    keep = wl["dst"] < nn_
    src, dst = wl["src"][keep], wl["dst"][keep]
    coords, x = wl["coords"][:nn_], wl["x"][:nn_]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    att = blk.attn

    def attention(P, Q, xin, dist, graph, edge_features=None):
        E = src.numel()
        qk = att.linear_qk(att.norm_qk(xin))
        Qe = qk[:, :64][dst].reshape(E, BLOCK_HEADS, -1)
        Ke = qk[:, 64:][src].reshape(E, BLOCK_HEADS, -1)
        rw = att.linear_v.radial_weights
        p1, p2 = rw.binning_params()
        V = orc.edgewise_fwd(P, P, xin[src], dist, rw(), lv, lv, att.linear_v.solid_harmonic_scale, p1, p2,
                             rw.num_bins, rw.log, nthreads=threads)
        w = orc.edge_attention(Qe, Ke, V, dst, nn_, att.attention.log_scale.exp(), BLOCK_HEADS)
        return orc.pool(w, dst, nn_, "sum")

    att.forward = attention
    graph = fe.Graph(src=src, dst=dst, num_nodes=nn_)

    def step():
        with torch.no_grad():
            vec = coords[src] - coords[dst]
            P = orc.wigner_basis(vec, lv)
            return blk(P, P, x, vec.norm(dim=-1), graph)

    return step, int(src.numel()), threads


def oracle_attention_forward(att, lv_in, lv_out, threads):
    """EquivariantAttention.forward (reference attention.py:271-314) on the host cores, with
    the edgewise V through the CPU restatement of the reference path (oracle/): node-level
    QK projection in PyTorch, bmm / block-diagonal mix / bmm, scatter softmax, scatter pool."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle as orc

    def forward(P, Q, xin, dist, graph, edge_features=None):
        src, dst, N = graph.src, graph.dst, graph.num_nodes
        mult, H = att.in_repr.mult, att.num_heads
        qk = att.linear_qk(att.norm_qk(xin))
        E = src.numel()
        Qe = qk[:, :mult][dst].reshape(E, H, -1)
        Ke = qk[:, mult:][src].reshape(E, H, -1)
        lv = att.linear_v
        rw = lv.radial_weights
        p1, p2 = rw.binning_params()
        f = xin[src] if edge_features is None else xin[src] + edge_features
        V = orc.edgewise_fwd(P, Q, f, dist, rw(), lv_in, lv_out, lv.solid_harmonic_scale, p1, p2, rw.num_bins,
                             rw.log, nthreads=threads)
        w = orc.edge_attention(Qe, Ke, V, dst, N, att.attention.log_scale.exp(), H, dist,
                               att.attention.distance_decay_scale)
        return orc.pool(w, dst, N, att.pool.reduce)

    return forward


def shard_graphs(graph_of_edge: torch.Tensor, n_graphs: int, world: int, rank: int):
    """Contiguous graph-id range [g0, g1) of this rank: one batch split across the ranks with
    boundaries on the cumulative edge count (about E / world edges per rank)."""
    from flash_eq.partition import dst_range_bounds

    b = dst_range_bounds(graph_of_edge, n_graphs, world)
    return int(b[rank]), int(b[rank + 1])


def run_block(args):
    """One step = the block forward (basis handles from the edge vectors, attention with the
    edgewise V, gated MLP) on the whole batch; data-parallel by graph batch under torchrun."""
    import flash_eq as fe

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        step, n, threads = cpu_block_setup(8)
        for _ in range(max(1, args.warmup)):
            step()
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        dt = (time.perf_counter() - t0) / args.steps
        print(json.dumps({
            "metric": METRIC_BLOCK, "impl": "reference", "value": n / dt,
            "unit": "edges/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": block_config(args.gpus, int(make_block_workload(BLOCK_SEED, "cpu")["src"].numel())),
            "cpu_baseline": {"value": n / dt, "unit": "edges/s", "cores": threads, "kind": "port",
                             "sample": f"8 of the 256 graphs ({n} edges) per step (CPU: {cpu_model()})"},
            "e2e": {"value": n / dt, "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return 0
    world, rank, local, pg = dist_setup(args)
    dev = torch.device("cuda", local)
    from flash_eq.cuda import _lib
    from flash_eq.cuda import ops as feq_ops

    lib = _lib.load()
    wl = make_block_workload(BLOCK_SEED, dev)
    E_total = int(wl["src"].numel())
    if world > 1:        # one batch, contiguous graph ranges balanced by edge count
        g0, g1 = shard_graphs(wl["dst"] // BLOCK_NODES, BLOCK_GRAPHS, world, rank)
        n0, n1 = g0 * BLOCK_NODES, g1 * BLOCK_NODES
        keep = (wl["dst"] >= n0) & (wl["dst"] < n1)
        wl = {"coords": wl["coords"][n0:n1], "x": wl["x"][n0:n1], "src": wl["src"][keep] - n0,
              "dst": wl["dst"][keep] - n0}
    blk, basis, r = build_block(dev)
    for m in blk.modules():
        if isinstance(m, fe.EquivariantEdgewiseLinear):
            m.mix_precision = args.mix
    N = wl["x"].shape[0]
    graph = fe.Graph(src=wl["src"].to(dev), dst=wl["dst"].to(dev), num_nodes=N)
    coords, x = wl["coords"].to(dev), wl["x"].to(dev)
    E = graph.num_edges
    eager = block_step_fn(blk, basis, graph, coords, x)
    for _ in range(max(3, args.warmup)):
        eager()
    torch.cuda.synchronize()
    # the whole forward replayed as one CUDA graph (the library's ops are stream-ordered and
    # allocate through torch's caching allocator, so the step captures as is)
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            eager()
    torch.cuda.current_stream().wait_stream(side)
    cg = torch.cuda.CUDAGraph()
    n_cap = lib.feq_launch_count()
    with torch.cuda.graph(cg):
        out_static = eager()
    per_replay = lib.feq_launch_count() - n_cap      # the library's kernels in one captured step
    step = cg.replay

    def timed(fn, steps):
        barrier(pg)
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            fn()
        t1.record()
        barrier(pg)
        return max_over_ranks(pg, t0.elapsed_time(t1) / steps)

    clk = ClockSampler(gpu_index_for(local))      # started before the warm-up (see run_ours)
    clk.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.profiler.start()      # lets `ncu --profile-from-start off` capture just the timed steps
    ms = timed(step, args.steps)
    torch.cuda.profiler.stop()
    launches = per_replay * args.steps
    clocks = clk.stop()
    for _ in range(3):                # eager steps warmed up again after the graph replays
        eager()
    ms_eager = timed(eager, max(3, args.steps // 4))
    value = E_total / (ms / 1e3)
    # per-stage device times of the library's kernels (eager steps, events on their streams)
    prof_steps = 3
    feq_ops.profile_enable(True)
    for _ in range(prof_steps):
        eager()
    torch.cuda.synchronize()
    stages = {k: {"ms": v[0] / prof_steps, "launches": v[1] // prof_steps} for k, v in feq_ops.profile_read().items()}
    feq_ops.profile_enable(False)
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    # algorithmic bytes per edge of the edge stages (fp32 rows C * d = 576 floats; bf16 A)
    row = 64 * 9 * 4
    nsplit = 2 if args.mix == "bf16x3" else 1
    stage_bytes = {"rotate_in": row + 32 + 64 * 9 * 2 * nsplit, "rotate_out": 2 * row + 24,
                   "tc_mix": 64 * 9 * 2 * nsplit + row + 4, "attn_pool": row + 16,
                   "sep_edgewise": 2 * row + 16}
    for k, v in stages.items():
        if k in stage_bytes:
            v["hbm_gbs"] = E * stage_bytes[k] / (v["ms"] / 1e3) / 1e9
    dom = max((k for k in stages if k in stage_bytes), key=lambda k: stages[k]["ms"], default=None)
    roofline = None
    if dom is not None:
        gbs = stages[dom]["hbm_gbs"]
        roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                    "traffic": None, "kernel": f"{dom} (largest edge stage; CUDA events on its stream)",
                    "peak_kind": peak_kind, "bytes_per_edge": stage_bytes[dom]}
    e2e = None
    if args.e2e_steps > 0:
        x_h, c_h = wl["x"].pin_memory(), wl["coords"].pin_memory()
        s_h, d_h = wl["src"].pin_memory(), wl["dst"].pin_memory()
        out_h = torch.empty(N, 64, 9, pin_memory=True)

        def e2e_step():
            xd, cd = x_h.to(dev, non_blocking=True), c_h.to(dev, non_blocking=True)
            g = fe.Graph(src=s_h.to(dev, non_blocking=True), dst=d_h.to(dev, non_blocking=True), num_nodes=N)
            out_h.copy_(block_step_fn(blk, basis, g, cd, xd)(), non_blocking=True)

        e2e_step()
        ms_e = timed(e2e_step, args.e2e_steps)
        e2e = {"value": E_total / (ms_e / 1e3), "unit": "edges/s",
               "h2d_bytes_per_step": (x_h.numel() + c_h.numel()) * 4 + (s_h.numel() + d_h.numel()) * 8,
               "d2h_bytes_per_step": out_h.numel() * 4, "ms_per_step": ms_e, "steps": args.e2e_steps,
               "note": "eager steps through the public API (Graph built per step: its dst sort and "
                       "validation included)"}
    if rank == 0:
        result = {
            "metric": METRIC_BLOCK, "value": value, "unit": "edges/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16" if args.mix == "bf16" else "f32", "data": "synthetic",
            "config": block_config(world, E_total), "edges_rank0": E, "roofline": roofline,
            "stages_ms_per_step": stages,
            "eager_ms_per_step": ms_eager, "mix": args.mix, "clocks": clocks, "e2e": e2e,
            "gpu_launches": int(launches), "note": "value: the step replayed as one CUDA graph; "
                                                   "eager_ms_per_step: the same step launched op by op"}
        if world == 1 and not args.no_cpu_baseline:
            try:
                cstep, n, threads = cpu_block_setup(8)
                cstep()
                t0 = time.perf_counter()
                for _ in range(2):
                    cstep()
                dt = (time.perf_counter() - t0) / 2
                result["cpu_baseline"] = {"value": n / dt, "unit": "edges/s", "cores": threads, "kind": "port",
                                          "sample": f"8 of the 256 graphs ({n} edges), 2 reps (CPU: {cpu_model()})"}
            except Exception as exc:  # the baseline must not hide the GPU number
                result["cpu_baseline"] = {"value": None, "error": repr(exc)}
        print(json.dumps(result), flush=True)
    del cg
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


def block_config(n_gpus, E_total):
    return {"workload": "config3: EquivariantTransformerBlock forward, Repr([0,1,2],64) -> same, 8 heads, "
                        "256 graphs x 30 nodes, coords N(0,1.5^2), all pairs within 5 A, 100 bins over [0,10]",
            "global_edges": E_total,
            "parallelism": f"dp{n_gpus}: the one batch split by contiguous graph ranges balanced by edge count"
                           if n_gpus > 1 else "one GPU",
            "l2": "no flush: 0.9 GB of edge rows (V) written and read per step >> 126 MB L2"}


# ---------------------------------------------------------------------------
# benchmark config 4: the full 6-layer EquivariantTransformer on 4096 graphs of 50 nodes
# ---------------------------------------------------------------------------
MODEL_GRAPHS, MODEL_NODES, MODEL_K, MODEL_HEADS, MODEL_LAYERS, MODEL_SEED = 4096, 50, 16, 8, 6, 3
# Out Repr([0], 8) stands in for the configured Repr([0], 1): the reference itself rejects 8
# heads on out mult 1 (attention.py:233-236); 8 is the smallest mult the 8 heads accept.
MODEL_OUT_MULT = 8
METRIC_MODEL = "edges/sec (6-layer EquivariantTransformer fwd)"


def make_model_workload(seed, device, n_graphs=MODEL_GRAPHS):
    """4096 graphs of 50 nodes, coordinates N(0, 2^2) per axis, 16-NN within each graph
    (src over the neighbours of dst), node features (N, 32, 4) ~ N(0, 1): benchmark config 4."""
    g = torch.Generator().manual_seed(seed)
    coords = torch.randn(n_graphs, MODEL_NODES, 3, generator=g) * 2.0
    x = torch.randn(n_graphs * MODEL_NODES, 32, 4, generator=g)
    c = coords.to(device)
    d = torch.cdist(c, c)
    d.diagonal(dim1=1, dim2=2).fill_(float("inf"))
    nbr = d.topk(MODEL_K, dim=2, largest=False).indices                     # (G, 50, 16)
    base = (torch.arange(n_graphs, device=c.device) * MODEL_NODES).view(-1, 1, 1)
    src = (nbr + base).reshape(-1)
    dst = (torch.arange(MODEL_NODES, device=c.device).view(1, -1, 1) + base).expand(-1, -1, MODEL_K).reshape(-1)
    return {"coords": coords.reshape(-1, 3), "x": x, "src": src.cpu(), "dst": dst.cpu()}


def build_model(device):
    import flash_eq as fe

    torch.manual_seed(MODEL_SEED)
    model = fe.EquivariantTransformer(fe.Repr([0, 1], 32), fe.Repr([0, 1, 2, 3], 128), fe.Repr([0], MODEL_OUT_MULT),
                                      num_layers=MODEL_LAYERS, num_heads=MODEL_HEADS, max_dist=MAX_DIST)
    return model.to(device).eval()


def model_config(n_gpus, E_total):
    return {"workload": "config4: 6-layer EquivariantTransformer forward, in Repr([0,1],32), hidden "
                        "Repr([0,1,2,3],128), out Repr([0],8) (out mult 8 for the configured 1: 8 heads must divide "
                        "it, attention.py:233-236), 8 heads, 4096 graphs x 50 nodes, coords N(0,2^2), 16-NN per "
                        "graph, 100 bins over [0,10]",
            "global_edges": E_total,
            "parallelism": f"dp{n_gpus}: the one batch split by contiguous graph ranges balanced by edge count"
                           if n_gpus > 1 else "one GPU",
            "l2": "no flush: 27 GB of edge rows (V) per hidden layer >> 126 MB L2"}


def cpu_model_setup(n_graphs):
    """The reference algorithm of the model on the host cores for the first n_graphs graphs:
    node-level modules in PyTorch, every attention layer through oracle_attention_forward,
    the basis by the oracle's matrix_exp (wigner.py:144-240)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import feq_oracle as orc
    import flash_eq as fe

    wl = make_model_workload(MODEL_SEED, "cpu", n_graphs=n_graphs)
    model = build_model("cpu")
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lv = {"in": [0, 1], "hid": [0, 1, 2, 3], "out": [0]}
    for i, blk in enumerate(model.layers):
        a = lv["in"] if i == 0 else lv["hid"]
        b = lv["out"] if i == MODEL_LAYERS - 1 else lv["hid"]
        blk.attn.forward = oracle_attention_forward(blk.attn, a, b, threads)
    model.basis.lazy = lambda vec: [orc.wigner_basis(vec, lv[k]) for k in ("in", "hid", "out")]
    graph = fe.Graph(src=wl["src"], dst=wl["dst"], num_nodes=n_graphs * MODEL_NODES)
    coords, x = wl["coords"], wl["x"]

    def step():
        with torch.no_grad():
            return model(coords, x, graph)

    return step, int(wl["src"].numel()), threads


def run_model(args):
    """One step = the 6-layer model forward over the batch (basis once, 6 blocks, final norm);
    under torchrun the one batch is split by contiguous graph ranges (no collective)."""
    import flash_eq as fe

    E_total = MODEL_GRAPHS * MODEL_NODES * MODEL_K
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return 0
        step, n, threads = cpu_model_setup(2)
        step()
        t0 = time.perf_counter()
        for _ in range(max(1, args.steps)):
            step()
        dt = (time.perf_counter() - t0) / max(1, args.steps)
        print(json.dumps({
            "metric": METRIC_MODEL, "impl": "reference", "value": n / dt, "unit": "edges/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt * 1e3, "higher_is_better": True,
            "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": model_config(args.gpus, E_total),
            "cpu_baseline": {"value": n / dt, "unit": "edges/s", "cores": threads, "kind": "port",
                             "sample": f"2 of the 4096 graphs ({n} edges) per step (CPU: {cpu_model()})"},
            "e2e": {"value": n / dt, "unit": "edges/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
            flush=True)
        return 0
    world, rank, local, pg = dist_setup(args)
    dev = torch.device("cuda", local)
    from flash_eq.cuda import _lib
    from flash_eq.cuda import ops as feq_ops

    lib = _lib.load()
    wl = make_model_workload(MODEL_SEED, dev)
    g0, g1 = shard_graphs(wl["dst"] // MODEL_NODES, MODEL_GRAPHS, world, rank) if world > 1 else (0, MODEL_GRAPHS)
    n0, n1 = g0 * MODEL_NODES, g1 * MODEL_NODES
    keep = (wl["dst"] >= n0) & (wl["dst"] < n1)
    src, dst = (wl["src"][keep] - n0).to(dev), (wl["dst"][keep] - n0).to(dev)
    coords, x = wl["coords"][n0:n1].to(dev), wl["x"][n0:n1].to(dev)
    graph = fe.Graph(src=src, dst=dst, num_nodes=n1 - n0)
    E = graph.num_edges
    model = build_model(dev)
    for m in model.modules():
        if isinstance(m, fe.EquivariantEdgewiseLinear):
            m.mix_precision = args.mix

    def step():
        with torch.no_grad():
            return model(coords, x, graph)

    clk = ClockSampler(gpu_index_for(local))      # started before the warm-up (see run_ours)
    clk.start()
    for _ in range(max(3, args.warmup)):
        step()
    barrier(pg)
    n_l0 = lib.feq_launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(pg)
    t0.record()
    for _ in range(args.steps):
        step()
    t1.record()
    barrier(pg)
    launches = lib.feq_launch_count() - n_l0
    clocks = clk.stop()
    ms = max_over_ranks(pg, t0.elapsed_time(t1) / args.steps)
    value = E_total / (ms / 1e3)
    feq_ops.profile_enable(True)
    step()
    torch.cuda.synchronize()
    stages = {k: {"ms": v[0], "launches": v[1]} for k, v in feq_ops.profile_read().items()}
    feq_ops.profile_enable(False)
    hbm_peak, _, peak_kind = measured_peaks()
    tc_sustained = measured_sustained() or 1430.0
    # the hidden -> hidden edgewise linears (4 of 6) dominate: C = 128, L <= 3
    d_h = 16
    mix_flops_h = 2 * 128 * 128 * sum((sum(1 for l in range(4) if l >= m)) ** 2 * (1 if m == 0 else 4)
                                      for m in range(4))
    roofline = None
    if "tc_mix" in stages:
        t = stages["tc_mix"]["ms"] / 1e3
        alg = 4 * E * mix_flops_h / t / 1e12     # lower bound: the 4 hidden -> hidden layers' mix FLOPs
        roofline = {"bound": "tensor", "achieved": alg, "peak": tc_sustained, "unit": "TFLOP/s",
                    "frac": alg / tc_sustained, "traffic": None,
                    "kernel": f"tc_mix ({stages['tc_mix']['launches']} launches per step), CUDA events on its stream",
                    "peak_kind": "measured bf16 sustained (MEASURED_PEAKS.json)",
                    "note": "achieved counts only the 4 hidden->hidden layers' algorithmic mix FLOPs "
                            f"({mix_flops_h / 1e6:.2f} MFLOP/edge) against the time of all 6 layers' mixes"}
    e2e = None
    if args.e2e_steps > 0:
        x_h, c_h = wl["x"][n0:n1].pin_memory(), wl["coords"][n0:n1].pin_memory()
        s_h, d_h_ = (wl["src"][keep] - n0).pin_memory(), (wl["dst"][keep] - n0).pin_memory()
        out_h = torch.empty(n1 - n0, MODEL_OUT_MULT, 1, pin_memory=True)

        def e2e_step():
            xd, cd = x_h.to(dev, non_blocking=True), c_h.to(dev, non_blocking=True)
            g = fe.Graph(src=s_h.to(dev, non_blocking=True), dst=d_h_.to(dev, non_blocking=True), num_nodes=n1 - n0)
            with torch.no_grad():
                out_h.copy_(model(cd, xd, g), non_blocking=True)

        e2e_step()
        barrier(pg)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record()
        barrier(pg)
        ms_e = max_over_ranks(pg, e0.elapsed_time(e1) / args.e2e_steps)
        e2e = {"value": E_total / (ms_e / 1e3), "unit": "edges/s",
               "h2d_bytes_per_step": (x_h.numel() + c_h.numel()) * 4 + (s_h.numel() + d_h_.numel()) * 8,
               "d2h_bytes_per_step": out_h.numel() * 4, "ms_per_step": ms_e, "steps": args.e2e_steps}
    if rank == 0:
        result = {
            "metric": METRIC_MODEL, "value": value, "unit": "edges/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "strong" if world > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16" if args.mix == "bf16" else "f32", "data": "synthetic",
            "config": model_config(world, E_total), "edges_rank0": E, "roofline": roofline,
            "stages_ms_per_step": stages, "mix": args.mix, "clocks": clocks, "e2e": e2e,
            "gpu_launches": int(launches), "memory_gb_rank0": torch.cuda.max_memory_allocated(dev) / 1e9}
        if world == 1 and not args.no_cpu_baseline:
            try:
                cstep, n, threads = cpu_model_setup(2)
                cstep()
                t0c = time.perf_counter()
                cstep()
                dt = time.perf_counter() - t0c
                result["cpu_baseline"] = {"value": n / dt, "unit": "edges/s", "cores": threads, "kind": "port",
                                          "sample": f"2 of the 4096 graphs ({n} edges), 1 rep (CPU: {cpu_model()})"}
            except Exception as exc:  # the baseline must not hide the GPU number
                result["cpu_baseline"] = {"value": None, "error": repr(exc)}
        print(json.dumps(result), flush=True)
    if pg is not None:
        pg.barrier()
        pg.destroy_process_group()
    return 0


# ---------------------------------------------------------------------------
# Config 5: one giant graph, dst-range partitioned across the ranks
# ---------------------------------------------------------------------------
GIANT_NODES = 1_000_000
GIANT_K = 16
GIANT_SEED = 4
GIANT_STEP = 3.8


def make_walk(n: int, seed: int) -> torch.Tensor:
    """3-D random walk: n positions, isotropic steps of GIANT_STEP A (seeded, CPU)."""
    g = torch.Generator().manual_seed(seed)
    steps = torch.randn(n, 3, generator=g)
    return torch.cumsum(GIANT_STEP * steps / steps.norm(dim=1, keepdim=True), 0)


def giant_measure(args, world, rank, local, pg, n, steps, warmup, e2e_steps):
    """Config 5 on the ranks of pg: build the graph (GPU kNN), partition it by dst range, time
    `steps` forward steps of the 2-layer transformer (max over ranks), then a few profiled
    steps: per-stage device times (rank 0), the per-layer NCCL exchanges (CUDA events around
    each all_to_all_single, max over ranks) and every rank's halo size.  Returns rank 0's
    record (other ranks: None)."""
    import flash_eq as fe
    from flash_eq import partition as fpart
    from flash_eq.cuda import _lib
    from flash_eq.cuda import ops as feq_ops
    from flash_eq.partition import partition_graph

    dev = torch.device("cuda", local)
    lib = _lib.load()
    coords = make_walk(n, GIANT_SEED)
    coords_d = coords.to(dev)
    t_build = time.perf_counter()
    graph = fe.Graph.knn(coords_d, GIANT_K)
    part = partition_graph(graph, world, rank) if world > 1 else graph
    torch.cuda.synchronize()
    t_build = time.perf_counter() - t_build
    r = fe.Repr([0, 1, 2], 64)
    torch.manual_seed(GIANT_SEED)
    model = fe.EquivariantTransformer(r, r, r, num_layers=2, num_heads=8, max_dist=MAX_DIST).to(dev).eval()
    for m in model.modules():
        if isinstance(m, fe.EquivariantEdgewiseLinear):
            m.mix_precision = args.mix
    x = torch.randn(n, 64, 9, generator=torch.Generator().manual_seed(GIANT_SEED + 1))
    lo, hi = (part.node_start, part.node_end) if world > 1 else (0, n)
    x_own = x[lo:hi].to(dev)
    E_total, E_rank = graph.num_edges, part.num_edges
    del graph

    def step():
        with torch.no_grad():
            return model(coords_d, x_own, part)

    clk = ClockSampler(gpu_index_for(local))      # started before the warm-up (see run_ours)
    clk.start()
    for _ in range(max(3, warmup)):
        step()
    barrier(pg)
    n0 = lib.feq_launch_count()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(pg)
    t0.record()
    for _ in range(steps):
        step()
    t1.record()
    barrier(pg)
    launches = lib.feq_launch_count() - n0
    clocks = clk.stop()
    ms = max_over_ranks(pg, t0.elapsed_time(t1) / steps)
    value = E_total / (ms / 1e3)
    # profiled steps: library stages (rank 0) and the exchanges (every rank)
    feq_ops.profile_enable(True)
    fpart.EXCHANGE_EVENTS = [] if world > 1 else None
    prof_steps = 2
    for _ in range(prof_steps):
        step()
    torch.cuda.synchronize()
    stages = {k: {"ms": v[0] / prof_steps, "launches": v[1] // prof_steps} for k, v in feq_ops.profile_read().items()}
    feq_ops.profile_enable(False)
    exchange = None
    if world > 1:
        ev = fpart.EXCHANGE_EVENTS
        fpart.EXCHANGE_EVENTS = None
        per = [a.elapsed_time(b) for a, b in ev]
        k = len(per) // prof_steps
        ex_ms = max_over_ranks(pg, sum(per) / prof_steps)
        halos = torch.zeros(world, dtype=torch.float64, device=dev)
        halos[rank] = part.num_halo
        owned = torch.zeros(world, dtype=torch.float64, device=dev)
        owned[rank] = hi - lo
        pg.all_reduce(halos)
        pg.all_reduce(owned)
        exchange = {"ms_per_step_max_rank": ex_ms, "exchanges_per_step": k,
                    "ms_each_rank0": [round(v, 4) for v in per[:k]],
                    "halo_rows_per_rank": [int(v) for v in halos.tolist()],
                    "owned_rows_per_rank": [int(v) for v in owned.tolist()],
                    "bytes_per_exchange_rank0": int(part.num_halo) * 64 * 9 * 4}
    hbm_peak, _, peak_kind = measured_peaks()
    row = 64 * 9 * 4
    nsplit = 2 if args.mix == "bf16x3" else 1
    stage_bytes = {"rotate_in": row + 32 + 64 * 9 * 2 * nsplit, "rotate_out": 2 * row + 24,
                   "attn_pool": row + 16, "sep_edgewise": 2 * row + 16}
    for k_, v in stages.items():
        if k_ in stage_bytes:
            v["hbm_gbs"] = 2 * E_rank * stage_bytes[k_] / (v["ms"] / 1e3) / 1e9     # 2 layers per step
    dom = max((k_ for k_ in stages if k_ in stage_bytes), key=lambda k_: stages[k_]["ms"], default=None)
    roofline = None
    if dom is not None:
        gbs = stages[dom]["hbm_gbs"]
        roofline = {"bound": "hbm", "achieved": gbs, "peak": hbm_peak, "unit": "GB/s", "frac": gbs / hbm_peak,
                    "traffic": None, "kernel": f"{dom} (largest HBM-bound edge stage, rank 0; CUDA events on its stream)",
                    "peak_kind": peak_kind, "bytes_per_edge": stage_bytes[dom]}
    lib_ms = sum(v["ms"] for v in stages.values())
    e2e = None
    if e2e_steps > 0:
        x_h = x[lo:hi].pin_memory()
        out_h = torch.empty(hi - lo, 64, 9, pin_memory=True)

        def e2e_step():
            xd = x_h.to(dev, non_blocking=True)
            with torch.no_grad():
                out_h.copy_(model(coords_d, xd, part), non_blocking=True)

        e2e_step()
        barrier(pg)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        barrier(pg)
        ms_e = max_over_ranks(pg, e0.elapsed_time(e1) / e2e_steps)
        e2e = {"value": E_total / (ms_e / 1e3), "unit": "edges/s", "h2d_bytes_per_step": x_h.numel() * 4,
               "d2h_bytes_per_step": out_h.numel() * 4, "ms_per_step": ms_e, "steps": e2e_steps,
               "note": "per rank: owned node features in from pinned host memory, owned outputs back; the "
                       "graph and its partition stay resident (built once)"}
    rec = None
    if rank == 0:
        largest = max(stages.items(), key=lambda kv: kv[1]["ms"]) if stages else None
        rec = {
            "metric": "edges/sec (2-layer EquivariantTransformer fwd, dst-range partitioned, device-timed)",
            "value": value, "unit": "edges/s", "n_gpus": world, "steps": steps, "warmup": warmup,
            "ms_per_step": ms, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": "bf16" if args.mix == "bf16" else "f32", "data": "synthetic",
            "config": {"workload": f"config5: 3-D random walk of {n} nodes (3.8 A isotropic steps, seed 4), "
                                   f"16-NN graph built on the GPU (Graph.knn), E={E_total}; 2-layer "
                                   "EquivariantTransformer, Repr([0,1,2],64) in/hidden/out, 8 heads, max_dist 10",
                       "global_edges": E_total, "edges_rank0": E_rank, "owned_rows_rank0": hi - lo,
                       "halo_rows_rank0": part.num_halo if world > 1 else 0,
                       "parallelism": f"dst-range partition over {world} GPU(s), NCCL halo exchange "
                                      "(all_to_all_single) of the src-side rows per layer" if world > 1
                                      else "whole graph on one GPU",
                       "graph_build_s": t_build,
                       "l2": f"no flush: {E_rank * row / 1e9:.1f} GB of edge rows per layer >> 126 MB L2"},
            "roofline": roofline, "stages_ms_per_step_rank0": stages, "exchange": exchange,
            "step_breakdown_rank0_ms": {"library_kernels": lib_ms,
                                        "nccl_exchange": exchange["ms_per_step_max_rank"] if exchange else 0.0,
                                        "other (torch glue: radial net, residual adds, LayerScale, gathers)": max(0.0, ms - lib_ms - (
                                            exchange["ms_per_step_max_rank"] if exchange else 0.0)),
                                        "largest_library_stage": largest[0] if largest else None},
            "mix": args.mix, "clocks": clocks, "e2e": e2e, "gpu_launches": int(launches),
            "memory_gb_rank0": torch.cuda.max_memory_allocated(dev) / 1e9}
    del model, part, coords_d, x_own
    torch.cuda.empty_cache()
    return rec


def run_giant(args):
    """One step = the 2-layer EquivariantTransformer forward over the rank's dst range of the
    1 M-node graph; per layer the rank's halo rows come from their owners (NCCL all-to-all).
    Graph built once (GPU kNN) and partitioned before the timed region; strong scaling."""
    n = args.nodes if args.nodes != N_NODES else GIANT_NODES
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "config 5 has no CPU arm: the oracle port of the "
                              "2-layer transformer over 16 M edges takes hours on the host cores; the block "
                              "workload carries the transformer CPU baseline"}), flush=True)
        return 0
    # 16 M edge rows per layer: let the caching allocator grow segments instead of
    # fragmenting across the per-layer edge tensors (read at the first CUDA use)
    os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    world, rank, local, pg = dist_setup(args)
    rec = giant_measure(args, world, rank, local, pg, n, args.steps, args.warmup, args.e2e_steps)
    if rank == 0:
        print(json.dumps(rec), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


# Published PatchedConvSE3 forward times of the reference (FULL fuse, C = 32, 500 bins, one
# ConvSE3 layer, NVIDIA H100): (L, edges) -> (SE(3)-T ms, patched ms), README.md:371-380.
PUBLISHED_PATCH_MS = {(2, 4096): (0.71, 1.03), (2, 16384): (2.20, 2.41), (2, 65536): (8.87, 7.70),
                      (3, 4096): (1.48, 1.42), (3, 16384): (5.42, 3.86), (3, 65536): (21.80, 13.39)}


def run_patch(args):
    """The reference's patch benchmark shapes through flash_eq.patch.PatchedConvSE3: one
    convolution forward (gather, rotation, 500-bin mix with sh_scale = 0, rotation back,
    edge -> node sum), C = 32, L = 2 / 3, 4K / 16K / 65K edges on a random graph of E / 16
    nodes; a synthetic converted table (the NVIDIA model is not part of this build)."""
    import flash_eq as fe
    from types import SimpleNamespace

    from flash_eq.patch import PatchedConvSE3

    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference patch path needs NVIDIA's "
                              "SE(3)-Transformer and DGL (not in this image); its published H100 times are "
                              "carried in the line as context"}), flush=True)
        return 0
    world, rank, local, pg = dist_setup(args)
    dev = torch.device("cuda", local)
    rows = []
    for L in (2, 3):
        for E in (4096, 16384, 65536):
            C, nb, N = 32, 500, E // 16
            gen = torch.Generator().manual_seed(1000 * L + E)
            lv = list(range(L + 1))
            rin = fe.Repr(lv, mult=C)
            pr = fe.ProductRepr(rin, rin)
            table = (torch.randn(nb + 1, C, C, pr.nreps(), generator=gen) * 0.05).to(dev)
            conv = SimpleNamespace(pool=True, fiber_in=SimpleNamespace(degrees=lv),
                                   fiber_out=SimpleNamespace(degrees=lv), self_interaction=False)
            mod = PatchedConvSE3(conv, table, pr, rin, rin, nb, 0.0, 10.0)
            mod.mix_precision = args.mix
            node = {str(d): torch.randn(N, C, 2 * d + 1, generator=gen).to(dev) for d in lv}
            src = torch.randint(0, N, (E,), generator=gen).to(dev)
            dst = torch.randint(0, N, (E,), generator=gen).to(dev)
            rel = (torch.randn(E, 3, generator=gen) * 3.0).to(dev)

            class G:
                def edges(self):
                    return src, dst

                def num_nodes(self):
                    return N

            graph = G()
            basis_mod = fe.WignerDBasis([fe.Repr(lv)]).to(dev)

            def step():
                with torch.no_grad():
                    dist = rel.norm(dim=-1)
                    (M,) = basis_mod(rel / dist[:, None])
                    return mod(node, {}, graph, {"_P": M, "_Q": M, "_distances": dist})

            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record()
            for _ in range(args.steps):
                step()
            t1.record()
            torch.cuda.synchronize()
            ms = t0.elapsed_time(t1) / args.steps
            se3t, patched = PUBLISHED_PATCH_MS[(L, E)]
            rows.append({"L": L, "edges": E, "ms": ms, "edges_per_s": E / (ms / 1e3),
                         "published_h100_patched_ms": patched, "published_h100_se3t_ms": se3t})
    if rank == 0:
        last = rows[-1]
        print(json.dumps({
            "metric": "edges/sec (PatchedConvSE3 fwd, L=3, 65K edges)", "value": last["edges_per_s"],
            "unit": "edges/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": last["ms"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "bf16" if args.mix == "bf16" else "f32", "data": "synthetic",
            "config": {"workload": "patch: one PatchedConvSE3 forward (FULL fuse, C=32, 500 bins, sh_scale 0, "
                                   "edge->node sum) on a random graph of E/16 nodes, synthetic table; step includes "
                                   "the WignerDBasis of the edge directions"},
            "table": rows, "mix": args.mix,
            "note": "published numbers: the reference on an NVIDIA H100 (README), context only"}), flush=True)
    if pg is not None:
        pg.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-config5", action="store_true",
                    help="at N > 1, skip the config-5 (partitioned giant graph) record of the default run")
    ap.add_argument("--nodes", type=int, default=N_NODES,
                    help="graph size (default: the config-2 size); smaller values only for profiling captures")
    ap.add_argument("--e2e-steps", type=int, default=3)
    ap.add_argument("--e2e-chunks", type=int, default=8,
                    help="edge chunks per end-to-end step (output copy of one overlaps compute of the next)")
    ap.add_argument("--workload", choices=["config2", "block", "model", "train", "giant", "patch"],
                    default="config2",
                    help="config2: the metric (default); block: benchmark config 3 (transformer block "
                         "forward); model: benchmark config 4 (6-layer transformer forward on 4096 graphs); "
                         "train: the reference's published single-layer fwd+bwd+Adam step "
                         "(--lmax, --edges); giant: benchmark config 5 (1 M-node graph, dst-range "
                         "partitioned across the ranks, strong scaling)")
    ap.add_argument("--edges", type=int, default=None)
    ap.add_argument("--lmax", type=int, default=4,
                    help="degrees 0..lmax in and out (default 4 = config 2); other values are variants, not the metric")
    ap.add_argument("--mix", choices=["fp32", "bf16x3", "bf16"], default="bf16x3",
                    help="radial-mix arithmetic: fp32 CUDA cores, bf16x3 / bf16 tensor cores")
    args = ap.parse_args()
    global LVALS
    LVALS = list(range(args.lmax + 1))
    if args.workload == "train":
        if args.lmax == 4 and args.edges is None:
            args.edges = 128000
        args.edges = args.edges or 32000
        return run_train(args)
    if args.workload == "block":
        return run_block(args)
    if args.workload == "model":
        return run_model(args)
    if args.workload == "patch":
        return run_patch(args)
    if args.workload == "giant":
        return run_giant(args)
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
