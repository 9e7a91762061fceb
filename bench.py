"""Benchmark: energy + forces throughput (atom-steps/s) of the uma-s-shaped model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl flash|reference] [--gemm f16x3|tf32x3|tf32]

Workload: bulk fcc Cu 10x10x10 conventional supercell, 4,000
atoms, displacements N(0, 0.05 A), cutoff 6 A, <= 30 neighbours (120,000 edges), random
uma-s-shaped weights (lmax=mmax=2, C=128, 4 layers, B=64, seed 0). A step is one energy
+ forces evaluation (forward + backward of the whole backbone + energy head) on a new set
of MD-like positions with the cached graph. Timing: CUDA events per step on the launching
stream, L2 flushed (256 MB write) before every step outside the timed events, max over
ranks. ``value`` has the positions already in HBM; ``e2e`` copies them from pinned host
memory and the energy and forces back inside the timed region, through the public API
(``Predictor(ZeroAllocBackbone(backbone), head)``).

With N > 1 GPUs (torchrun, one process per GPU) the system is bulk Cu 10 x 10 x (10 N), 4,000
atoms per GPU (weak scaling; N = 1 is config 3), split into N slabs with a per-layer halo
exchange over NCCL (``flash_uma_b200.partition``). ``--impl reference`` times the CPU
restatement of the reference implementation (the oracle) on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "atom-steps/s (energy+forces) uma-s-shaped"
UNIT = "atom-steps/s"

# algorithmic HBM bytes of one call of each entry point (fp32, minimum traffic: every
# per-edge / per-node tensor read or written once)
def alg_bytes(name, N, E, C, B, M_rows=None, D=None):
    # the *_f16x3 variants move the same bytes (a split output has the fp32 footprint)
    name = name[: -len("_f16x3")] if name.endswith("_f16x3") and name != "fuma_linear_f16x3" else name
    f = 4
    if name == "fuma_gather_fwd":
        return E * (f * 34 + f * 12 * C + 8 + f * 18 * C) + N * f * 9 * C
    if name == "fuma_gather_bwd":
        return E * (f * 18 * C + f * 12 * C + f * 34 + 16 + f * 12 * C + f * 34) + N * f * 9 * C * 2
    if name == "fuma_rotate_scatter_fwd":
        return E * (f * 9 * C + f * 34 + f + 4) + N * 2 * f * 9 * C + 4 * (N + 1)
    if name == "fuma_rotate_scatter_bwd":
        return E * (f * 9 * C * 2 + f * 34 * 2 + f * 2 + 4) + N * f * 9 * C
    if name == "fuma_gating_fwd":
        return E * f * 20 * C
    if name == "fuma_gating_bwd":
        return E * f * 31 * C
    if name == "fuma_init_scatter_fwd":
        return E * (f * 3 * C + f * 34 + f + 4) + N * f * 9 * C
    if name == "fuma_init_scatter_bwd":
        return E * (f * 6 * C + f * 68 + f * 2 + 4) + N * f * 9 * C
    if name == "fuma_geometry_fwd":
        return E * (f * (B + 2 * C) + f * 34 + f + 12 + 16) + N * 20
    if name == "fuma_geometry_bwd":
        return E * (f * B + f * 34 + f + 12 + 16 + 12) + N * 12
    if name == "fuma_edge_vec_to_nodes":
        return E * (2 * 12 + 8) + N * 12
    if name == "fuma_ln_silu_fwd":
        return M_rows * (2 * f * D + 8)
    if name == "fuma_ln_silu_bwd":
        return M_rows * (3 * f * D + 8)
    return None


# dense FLOPs of the model's GEMMs per edge and layer: radial 2*(K_in*H + H*H + H*12C), conv1
# 2*70C^2, conv2 2*29C^2 in the forward; the input-gradient GEMMs of the backward have the same
# count, except that with gauss_only the first radial layer's gradient covers only the B
# Gaussian columns (the fused path: the embedding columns do not depend on positions)
def gemm_flops_per_step(E, C, B, L, H=None, gauss_only=True, N_atomwise=0):
    """``N_atomwise``: atoms whose gated atom-wise block runs on the same GEMM kernel (the fp16
    modes): its scalar MLP and two per-degree maps, 40 N C H forward and 40 N C H for the input
    gradients per layer (the stacked-degree GEMMs also compute two unused degree blocks, which
    are not counted)."""
    H = H or C
    rad_layer = 2 * ((B + 2 * C) * H + H * H + H * 12 * C)
    rad_init = 2 * ((B + 2 * C) * H + H * H + H * 3 * C)
    so2 = 2 * 70 * C * C + 2 * 29 * C * C
    fwd = E * (L * (rad_layer + so2) + rad_init)
    bwd = fwd - (E * (L + 1) * 2 * 2 * C * H if gauss_only else 0)
    return fwd + bwd + 80 * N_atomwise * C * H * L


GEMM_OPS = ("fuma_linear_f16x3", "fuma_linear", "fuma_linear_f16")


def gemm_mode(mode, bf16):
    """Tensor-pipe products per fp32 product, the pipe's peak (TF/s) and labels of a GEMM mode."""
    if mode == "f16x3":
        return {"passes": 3, "peak": bf16, "pipe": "fp16", "op": "fuma_linear_f16x3",
                "kernel": "fuma_linear_f16x3 (gemm_f16x3_kernel)", "label": "tcgen05 f16x3 (fp16 split, fp32-level)",
                "peak_note": "dense fp16 = measured dense bf16 rate"}
    if mode == "f16":
        return {"passes": 1, "peak": bf16, "pipe": "fp16", "op": "fuma_linear_f16",
                "kernel": "fuma_linear_f16 (gemm_f16x3_kernel, single product)",
                "label": "tcgen05 f16 (single fp16 product, TF32 accuracy class)",
                "peak_note": "dense fp16 = measured dense bf16 rate"}
    return {"passes": 3 if mode == "tf32x3" else 1, "peak": bf16 / 2, "pipe": "tf32", "op": "fuma_linear",
            "kernel": "fuma_linear (gemm_tf32_kernel)",
            "label": "tcgen05 3xTF32 (fp32-level)" if mode == "tf32x3" else "tcgen05 TF32 (single pass)",
            "peak_note": "dense TF32 taken as half the measured dense bf16 rate"}


def gemm_summary(per_op, E, C, B, L, mode, N=0):
    """Dense-contraction share of one step (from the probe pass): fp32-equivalent FLOP rate and the
    tensor-pipe rate (3 products per fp32 product in the split modes)."""
    g = gemm_mode(mode, 0.0)
    ms = per_op.get(g["op"])
    if not ms:
        return None
    f16 = mode in ("f16x3", "f16")
    flops = gemm_flops_per_step(E, C, B, L, gauss_only=f16, N_atomwise=N if f16 else 0)
    return {"flops_per_step": flops, "ms_per_step": ms, "tflops_fp32_equiv": flops / (ms * 1e-3) / 1e12,
            "tflops_pipe": g["passes"] * flops / (ms * 1e-3) / 1e12, "pipe": g["pipe"], "passes": g["passes"]}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.index), "-lms", "200"], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        loaded = [s for s in sm if mx and s > 0.5 * max(mx)] or sm
        return {"sm_mhz": statistics.median(loaded) if loaded else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def build_problem(device, gemm: str, system=None):
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import config3_system, to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    system = system or config3_system()
    data = to_graph([system])
    off = SyntheticESCNMDBackbone(seed=0).to(device)
    head = make_energy_head(128, 128, seed=1).to(device)
    pred = Predictor(ZeroAllocBackbone(off, gemm=gemm), head)
    return system, data, pred


def md_positions(pos0: torch.Tensor, count: int, seed: int = 0):
    """MD-like position sequence: small random displacements (0.01 A rms) around pos0."""
    g = torch.Generator().manual_seed(seed)
    return [pos0 + 0.01 * torch.randn(pos0.shape, generator=g) for _ in range(count)]


def workload_system(workload: str, world: int):
    """(system, stress, scaling, label) of a bench workload at ``world`` GPUs.

    default: config 3 at N = 1, weak scaling beyond (bulk fcc Cu 10 x 10 x 10N, 4,000 atoms
             per GPU, split into N slabs with per-layer halo exchange);
    config4: the ~10k-atom water box with energy + forces + stress (1 and 2 GPUs);
    config5: bulk fcc Cu 30 x 30 x 28 (100,800 atoms) at every N (strong scaling)."""
    from flash_uma_b200.systems import bulk_fcc, config3_system, config4_system, config5_system
    if workload == "config5":
        return config5_system(), False, "strong", "bulk_cu_100800 (BASELINE config 5), E+F per step"
    if workload == "config4":
        return config4_system(), True, "strong", "water box 3,333 H2O (BASELINE config 4), E+F+S per step"
    if world == 1:
        return config3_system(), False, "weak", "bulk_cu_4000 (BASELINE config 3), E+F per step"
    return (bulk_fcc(10, 10, 10 * world, jitter=0.05, seed=0, name=f"bulk_cu_{4000 * world}"), False, "weak",
            f"bulk Cu 10x10x{10 * world} (4000 atoms per GPU, weak scaling of config 3), E+F per step")


def build_partitioned(device, gemm: str, world: int, rank: int, system=None, stress: bool = False):
    """N > 1 GPUs: the system split into N slabs along its long axis with a per-layer halo
    exchange of node embeddings over NCCL (flash_uma_b200.partition)."""
    from flash_uma_b200.partition import PartitionedModel, make_plan
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    data = to_graph([system])
    off = SyntheticESCNMDBackbone(seed=0).to(device)
    head = make_energy_head(128, 128, seed=1).to(device)
    bb = ZeroAllocBackbone(off, gemm=gemm)
    plan = make_plan(system.positions, system.cell, data.edge_index.numpy(), world, rank)
    pm = PartitionedModel(bb.ce, plan, device)
    d = data.to(device)
    csd = bb.csd_embedding(d.charge, d.spin).float().detach()

    fixed = (d.atomic_numbers, d.batch, d.cell_offsets, d.cell[0], csd)
    csd_sys = dict(charge=d.charge, spin=d.spin, natoms=d.natoms)

    def step(pos):
        out = pm.energy_forces(head, pos, *fixed, stress=stress, **csd_sys)
        return dict(zip(("energy", "forces", "stress"), out))

    def make_graph(pos0, capture_hook=None):
        """The step captured as one CUDA graph with its NCCL collectives (every rank calls this)."""
        from flash_uma_b200.partition import GraphedPartitionedStep
        g = GraphedPartitionedStep(pm, head, pos0, *fixed, stress=stress, capture_hook=capture_hook, **csd_sys)

        class Step:
            def __call__(self, pos):
                return dict(zip(("energy", "forces", "stress"), g(pos)))

            def release(self):
                g.release()
        return Step()

    return system, data, step, plan, make_graph


def run_flash(args, rank, world, device):
    from flash_uma_b200 import _native
    _native.load()
    C, B, L = 128, 64, 4
    K, W = args.steps, args.warmup
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    system, with_stress, scaling, label = workload_system(args.workload, world)
    if world > 1:
        system, data_cpu, step, plan, make_graph = build_partitioned(device, args.gemm, world, rank, system,
                                                                      with_stress)
        N, E = data_cpu.pos.shape[0], data_cpu.edge_index.shape[1]
        pos_seq = [p.to(device) for p in md_positions(data_cpu.pos, K + W, seed=0)]
    else:
        plan = None
        system, data_cpu, pred = build_problem(device, args.gemm, system)
        N, E = data_cpu.pos.shape[0], data_cpu.edge_index.shape[1]
        data = data_cpu.to(device)
        pos_seq = [p.to(device) for p in md_positions(data_cpu.pos, K + W, seed=rank)]

        import dataclasses

        def step(pos):
            return pred(dataclasses.replace(data, pos=pos), stress=with_stress)

    # ---- which of our kernels dominates: one probe pass with every entry point timed
    probe = _native.LaunchProbe(timed=list(_native.KERNELS_PER_CALL))
    for w in range(W):
        step(pos_seq[w])
    torch.cuda.synchronize()
    _native.set_probe(probe)
    res0 = step(pos_seq[0])
    torch.cuda.synchronize()
    _native.set_probe(None)
    # results at the first position, for the parity check against the reference's Triton path
    check0 = (res0["energy"].detach().clone(), res0["forces"].detach().clone())
    del res0
    per_op = {n: sum(probe.times_ms(n)) for n in probe.events}
    probe_counts = dict(probe.counts)
    dominant = max(per_op, key=per_op.get)
    launches_per_step = probe.launches

    graphed = args.graph
    gstep = None
    if graphed:
        # the whole step (graph build, forward, backward; with N > 1 also the NCCL halo exchanges
        # and all-reduces) as one CUDA graph. The probe is active during the capture: it counts
        # the launches of one step and records event nodes around the dominant kernel's
        # launches, whose elapsed times then read the last replay.
        gprobe = _native.LaunchProbe(timed=[dominant], external=True)
        hook = lambda on: _native.set_probe(gprobe if on else None)   # noqa: E731
        if world > 1:
            # captured collectives do not communicate, so a capture that fails on one rank leaves
            # the others consistent: all ranks agree on graph or eager with one all-reduce
            try:
                gstep = make_graph(pos_seq[0], capture_hook=hook)
            except Exception as exc:   # noqa: BLE001 - reported, then the eager step is used
                print(f"rank {rank}: CUDA-graph capture of the partitioned step failed ({exc}); "
                      "falling back to eager launches", file=sys.stderr, flush=True)
                gstep = None
            ok = torch.tensor([0 if gstep is None else 1], device=device)
            torch.distributed.all_reduce(ok, op=torch.distributed.ReduceOp.MIN)
            if int(ok.item()) == 0:
                if gstep is not None:
                    gstep.release()
                gstep, graphed = None, False
        else:
            from flash_uma_b200.predict import GraphedStep
            gstep = GraphedStep(pred, dataclasses.replace(data, pos=pos_seq[0]), stress=with_stress,
                                capture_hook=hook)
        if graphed:
            graph_launches = gprobe.launches
            step = gstep
    # ---- timed region 1: inputs resident in HBM. Launch counting covers every timed step; the
    # dominant kernel's launches are bracketed with CUDA events in the last timed step only
    # (pre-created events), so the instrumentation does not slow the other steps.
    probe = _native.LaunchProbe(timed=[dominant], pool=4 * probe_counts.get(dominant, 1) + 8)
    probe.timing = False
    sampler = ClockSampler(device.index if device.index is not None else 0)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    sampler.start()
    _native.set_probe(probe)
    evs = []
    for k in range(K):
        flush.zero_()
        probe.timing = k == K - 1
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        torch.cuda.nvtx.range_push("fuma_step")
        res = step(pos_seq[W + k])
        torch.cuda.nvtx.range_pop()
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    _native.set_probe(None)
    clocks = sampler.stop()
    total_ms = sum(a.elapsed_time(b) for a, b in evs)
    dom_ms = gprobe.times_ms(dominant) if graphed else probe.times_ms(dominant)
    gpu_launches = graph_launches * K if graphed else probe.launches

    # ---- timed region 2: end to end from pinned host buffers through the public API
    host_pos = [p.cpu().pin_memory() for p in md_positions(data_cpu.pos, K, seed=100 + (0 if world > 1 else rank))]
    f_host = torch.empty(N, 3).pin_memory()
    e_host = torch.empty(1).pin_memory()
    s_host = torch.empty(1, 3, 3).pin_memory()
    st_host = torch.zeros(K, dtype=torch.int32).pin_memory()   # each step's GEMM error status
    pos_dev = torch.empty(N, 3, device=device)
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    evs2 = []
    for k in range(K):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        pos_dev.copy_(host_pos[k], non_blocking=True)
        res = step(pos_dev)
        f_host.copy_(res["forces"], non_blocking=True)
        e_host.copy_(res["energy"], non_blocking=True)
        if with_stress:
            s_host.copy_(res["stress"], non_blocking=True)
        if "status" in res:
            st_host[k:k + 1].copy_(res["status"], non_blocking=True)
        e1.record()
        evs2.append((e0, e1))
    torch.cuda.synchronize()
    e2e_ms = sum(a.elapsed_time(b) for a, b in evs2)
    from flash_uma_b200.linear import raise_status
    for k in range(K):   # a failed GEMM in any timed step invalidates the run
        raise_status(st_host[k:k + 1], device)

    if gstep is not None and world > 1:
        gstep.release()   # the graph holds NCCL work: free it before the process group goes
    t = torch.tensor([total_ms, e2e_ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    total_ms, e2e_ms = t.tolist()

    hbm, bf16, peak_kind = load_peaks()
    avg_ms = sum(dom_ms) / max(1, len(dom_ms))
    # per-launch sizes: this rank's local graph
    Ek, Nk = (len(plan.edges), len(plan.local_ids)) if world > 1 else (E, N)
    gm = gemm_mode(args.gemm, bf16)
    if dominant in GEMM_OPS:
        # tensor-bound. achieved / frac: ALGORITHMIC fp32 FLOPs per launch (the model's dense
        # FLOPs, 2 x M x N x K per product) over the measured dense bf16 peak; the split modes run
        # ``passes`` tensor-pipe products per fp32 product, reported apart as the pipe utilisation
        launches = gprobe.counts.get(dominant, 1) if graphed else probe.counts.get(dominant, 1) // K
        f16 = args.gemm in ("f16x3", "f16")
        n_aw = (len(plan.owned) if world > 1 else N) if f16 else 0   # atom-wise blocks run on owned atoms
        flops = gemm_flops_per_step(Ek, C, B, L, gauss_only=f16, N_atomwise=n_aw)
        flops_launch = flops / max(1, launches)
        achieved = flops_launch / (avg_ms * 1e-3) / 1e12
        roof = {"kernel": gm["kernel"], "bound": "tensor", "achieved": achieved,
                "peak": bf16, "unit": "TFLOP/s", "frac": achieved / bf16,
                "peak_kind": f"{peak_kind} dense bf16 (burst)",
                "traffic": None,
                "alg_flops_per_launch": flops_launch,
                "tensor_pipe_util": {"pipe": gm["pipe"], "products_per_fp32_product": gm["passes"],
                                     "pipe_tflops": gm["passes"] * achieved,
                                     "frac_of_pipe_peak": gm["passes"] * achieved / gm["peak"],
                                     "pipe_peak": gm["peak"], "pipe_peak_note": gm["peak_note"]}}
    else:
        nbytes = alg_bytes(dominant, Nk, Ek, C, B, M_rows=Ek, D=128)
        achieved = nbytes / (avg_ms * 1e-3) / 1e9 if nbytes and avg_ms > 0 else None
        roof = {"kernel": dominant, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                "frac": (achieved / hbm) if achieved else None, "peak_kind": peak_kind, "traffic": None,
                "alg_bytes_per_launch": nbytes}
    roof.update(avg_launch_ms=avg_ms, launches_timed=len(dom_ms),
                share_of_step=(sum(dom_ms) / (total_ms / K)) if world == 1 else None)   # dom_ms: one step
    # the top HBM-bound kernel as well (device time from the probe pass)
    mem_ops = {k: v for k, v in per_op.items() if k not in GEMM_OPS and alg_bytes(k, Nk, Ek, C, B, Ek, 128)}
    top_mem = max(mem_ops, key=mem_ops.get) if mem_ops else None
    roof_mem = None
    if top_mem:
        launches = max(1, probe_counts.get(top_mem, 1))
        ms_launch = per_op[top_mem] / launches
        nb = alg_bytes(top_mem, Nk, Ek, C, B, M_rows=Ek, D=128)
        gbs = nb / (ms_launch * 1e-3) / 1e9
        roof_mem = {"kernel": top_mem, "bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                    "frac": gbs / hbm, "alg_bytes_per_launch": nb, "avg_launch_ms": ms_launch, "traffic": None}
    atoms_total = N if world > 1 else world * N
    out = {
        "metric": METRIC, "value": atoms_total * K / (total_ms * 1e-3), "unit": UNIT, "n_gpus": world, "steps": K,
        "warmup": W, "ms_per_step": total_ms / K, "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded positions, random-init weights)",
        "config": {"workload": f"{label}: {N} atoms, {E} edges"
                               + (", slab decomposition with per-layer halo exchange (NCCL)" if world > 1 else ""),
                   "atoms": N, "edges": E, "sphere_channels": C, "layers": L, "num_distance_basis": B,
                   "cutoff": 6.0, "max_neighbors": 30, "gemm": gm["label"],
                   "l2": "flushed (256 MB write) before every step, outside the timed events",
                   "launch": ("one CUDA graph replay per step (graph build, forward, backward"
                              + (", NCCL halo exchanges and all-reduces" if world > 1 else "") + " captured once)")
                   if graphed else "eager (every kernel launched from the host)",
                   "parallelism": f"spatial slabs x{world} (halo atoms per rank: {len(plan.halo)} on rank 0)"
                   if world > 1 else "single GPU"},
        "e2e": {"value": atoms_total * K / (e2e_ms * 1e-3), "unit": UNIT, "h2d_bytes_per_step": N * 3 * 4,
                "d2h_bytes_per_step": N * 3 * 4 + 4 + (36 if with_stress else 0) + 4},
        "max_device_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9,
        "roofline": roof,
        "roofline_top_hbm_kernel": roof_mem,
        "gemm": gemm_summary(per_op, Ek, C, B, L, args.gemm, len(plan.owned) if world > 1 else N),
        "gpu_launches": gpu_launches,
        "per_kernel_ms_one_step": {k: round(v, 4) for k, v in sorted(per_op.items(), key=lambda kv: -kv[1])},
        "clocks": clocks,
    }
    out["_check"] = check0
    out["_pos0"] = pos_seq[0].detach().cpu()
    return out


def partition_parity(args, device, check0, pos0):
    """N > 1: the same system and positions on this one GPU (single-GPU path, no partition)
    against the partitioned result of every rank (energy, forces; stress with it)."""
    import dataclasses
    system, with_stress, _, _ = workload_system(args.workload, int(os.environ.get("WORLD_SIZE", "1")))
    torch.cuda.empty_cache()
    _, data_cpu, pred = build_problem(device, args.gemm, system)
    data = data_cpu.to(device)
    res = pred(dataclasses.replace(data, pos=pos0.to(device)), stress=with_stress, check=True)
    e, f = check0[0].double(), check0[1].double()
    er, fr = res["energy"].double(), res["forces"].double()
    out = {"energy_rel": float(((e - er).abs() / er.abs().clamp_min(1.0)).max()),
           "forces_max_abs": float((f - fr).abs().max()),
           "against": "single-GPU path on the same system and positions (rank 0, after the timed run)",
           "bar": {"energy_rel": 1e-5, "forces_max_abs": 1e-4}}
    del pred, res, data
    torch.cuda.empty_cache()
    return out


def run_mode(device, gemm: str, steps: int, warmup: int, system, check=None):
    """This build's step in another GEMM mode on the same workload (CUDA-graph replay, CUDA events
    per step, L2 flushed in between): atom-steps/s and, with ``check`` (energy, forces of the
    default f16x3 mode at the first position), the deviation from that fp32-level result."""
    import dataclasses

    from flash_uma_b200.predict import GraphedStep
    system, data_cpu, pred = build_problem(device, gemm, system)
    data = data_cpu.to(device)
    N = data_cpu.pos.shape[0]
    pos_seq = [p.to(device) for p in md_positions(data_cpu.pos, steps + warmup, seed=0)]
    out = {}
    if check is not None:
        res = pred(dataclasses.replace(data, pos=pos_seq[0]), check=True)
        e, f = res["energy"].double(), res["forces"].double()
        out["deviation_from_f16x3"] = {
            "energy_rel": float(((e - check[0].double()).abs() / check[0].double().abs().clamp_min(1.0)).max()),
            "forces_max_abs": float((f - check[1].double()).abs().max())}
        del res
    step = GraphedStep(pred, dataclasses.replace(data, pos=pos_seq[0]))
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    for w in range(warmup):
        step(pos_seq[w])
    torch.cuda.synchronize()
    evs = []
    for k in range(steps):
        flush.zero_()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step(pos_seq[warmup + k])
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    from flash_uma_b200.linear import raise_status
    raise_status(step.out["status"])
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    out.update(value=N / (ms * 1e-3), unit=UNIT, ms_per_step=ms, gemm=gemm_mode(gemm, 0.0)["label"],
               launch="one CUDA graph replay per step", steps=steps, warmup=warmup)
    del step, pred, flush
    torch.cuda.empty_cache()
    return out


def run_strong5(args, rank, world, device, steps: int = 3, warmup: int = 2):
    """BASELINE config 5 (bulk fcc Cu 30x30x28, 100,800 atoms, 3,024,000 edges, energy + forces) at
    this run's N (strong scaling: the same system at every N): atom-steps/s, ms per step (CUDA
    events, max over ranks), halo atoms per rank, device memory, and the device time of every
    collective kind per step (halo all-to-all forward / backward, the energy / force all-reduce).
    Eager launches; one GPU runs the memory-lean mode when the activations would not fit."""
    import dataclasses

    from flash_uma_b200 import partition as part
    from flash_uma_b200.systems import config5_system
    torch.cuda.empty_cache()
    torch.cuda.reset_peak_memory_stats(device)
    system = config5_system()
    halo = 0
    if world > 1:
        system, data_cpu, step, plan, _ = build_partitioned(device, args.gemm, world, rank, system, False)
        halo = len(plan.halo)
    else:
        _, data_cpu, pred = build_problem(device, args.gemm, system)
        data = data_cpu.to(device)

        def step(pos):
            return pred(dataclasses.replace(data, pos=pos))
    N, E = data_cpu.pos.shape[0], data_cpu.edge_index.shape[1]
    pos_seq = [p.to(device) for p in md_positions(data_cpu.pos, steps + warmup, seed=0)]
    for w in range(warmup):
        step(pos_seq[w])
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    part.collective_events = [] if world > 1 else None
    evs = []
    for k in range(steps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        step(pos_seq[warmup + k])
        e1.record()
        evs.append((e0, e1))
    torch.cuda.synchronize()
    coll = {k: v / steps for k, v in part.collective_times_ms().items()}
    part.collective_events = None
    ms = sum(a.elapsed_time(b) for a, b in evs) / steps
    halos = torch.zeros(world, dtype=torch.float64, device=device)
    halos[rank] = halo
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        torch.distributed.all_reduce(halos)
    ms = float(t.item())
    from flash_uma_b200 import fused
    lean = fused.lean_needed(E // world if world > 1 else E, 128, 128, 4, device)
    return {"workload": "bulk_cu_100800 (BASELINE config 5), E+F per step, strong scaling", "atoms": N, "edges": E,
            "n_gpus": world, "value": N / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms, "steps": steps,
            "warmup": warmup, "launch": "eager", "memory_lean_mode": lean,
            "halo_atoms_per_rank": [int(h) for h in halos.tolist()] if world > 1 else [0],
            "max_device_memory_gb_rank0": torch.cuda.max_memory_allocated(device) / 1e9,
            "collectives_ms_per_step_rank0": {k: round(v, 4) for k, v in coll.items()},
            "timing": "CUDA events per step, max over ranks; collectives: events around each NCCL call on rank 0"}


def run_micro(args, device):
    """one message-passing layer (radial MLP with LN-SiLU -> gather-rotate ->
    SO(2) conv1 -> gating -> conv2 -> FP64 rotate-scatter), forward + backward, inputs resident.
    Geometry is computed once from the synthetic edge vectors (uniform directions, lengths
    U(0.8, 6) A) outside the timed region. Every C-ABI call is bracketed with CUDA events;
    prints per-kernel time, algorithmic bytes and fraction of the measured HBM / tensor peaks."""
    import functools

    from flash_uma_b200 import _native, fused, ops
    from flash_uma_b200.linear import FrozenLinear
    from flash_uma_b200.model import PackedLayer
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone
    from flash_uma_b200.systems import microbench_layer_inputs
    _native.load()
    N, E, C, B = args.nodes, args.edges, 128, 64
    inp = microbench_layer_inputs(N=N, E=E, C=C, seed=0)
    off = SyntheticESCNMDBackbone(num_layers=1, seed=0).to(device)
    layer = PackedLayer(off.blocks[0], C, args.gemm).to(device)
    ii, jj = inp["idx_i"].to(device), inp["idx_j"].to(device)
    graph = ops.build_graph_csr(ii, jj, N)
    Z = torch.full((N,), 29, dtype=torch.long, device=device)
    batch = torch.zeros(N, dtype=torch.long, device=device)
    offset = torch.linspace(0, 6.0, B, device=device)
    coeff = float(-0.5 / (2.0 * (6.0 / (B - 1))) ** 2)
    # f16x3: the production path, one fused message block (split operands, pre-split GEMMs)
    use_fused = args.gemm in ("f16x3", "f16")
    geom = fused.geometry if use_fused else functools.partial(ops.precompute_geometry, graph=graph)
    geom_args = (inp["pos"].to(device), Z, ii, jj, inp["shifts"].to(device), off.source_embedding.weight.detach(),
                 off.target_embedding.weight.detach(), offset, coeff, 6.0) + ((graph,) if use_fused else ())
    if use_fused:
        layer.rad.n_gauss = B
        for lin in layer.modules():
            if isinstance(lin, FrozenLinear):
                lin.prepare()
    xe, wig, env = geom(*geom_args)
    csd = torch.randn(1, C, device=device)
    x0 = inp["x"].to(device)
    gout = torch.randn(N, 9, C, device=device)

    def step():
        x = x0.detach().requires_grad_(True)
        if use_fused:
            out = fused.message_block(layer, x, x, xe, wig, env, csd, ii, jj, batch, graph)
            (gx,) = torch.autograd.grad(out, [x], gout)
            return gx
        rad = layer.rad(xe)
        X0, X1, X2 = ops.gather_wigner_split(x, ii, jj, wig, rad, csd, batch, graph=graph)
        Z0, Z1, Z2 = ops.fused_gating_split(layer.conv1_m0(X0), layer.conv1_m1(X1), layer.conv1_m2(X2), C)
        out = ops.rotate_scatter_split(layer.conv2_m0(Z0), layer.conv2_m1(Z1), layer.conv2_m2(Z2), wig, env, x, jj,
                                       graph.dst_row_ptr, graph.dst_col, N)
        (gx,) = torch.autograd.grad(out, [x], gout)
        return gx

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    probe = _native.LaunchProbe(timed=list(_native.KERNELS_PER_CALL))
    _native.set_probe(probe)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        torch.cuda.nvtx.range_push("fuma_step")
        step()
        torch.cuda.nvtx.range_pop()
    e1.record()
    torch.cuda.synchronize()
    _native.set_probe(None)
    total = e0.elapsed_time(e1) / args.steps
    hbm, bf16, kind = load_peaks()
    kernels = {}
    for name in probe.events:
        t = probe.times_ms(name)
        per_step = sum(t) / args.steps
        launches = len(t) // args.steps
        entry = {"ms_per_step": per_step, "launches_per_step": launches}
        nb = alg_bytes(name, N, E, C, B, M_rows=E, D=128)
        if nb:
            gbs = nb * launches / (per_step * 1e-3) / 1e9
            entry.update(alg_bytes_per_launch=nb, achieved_gbs=gbs, frac_hbm=gbs / hbm)
        kernels[name] = entry
    gm = gemm_mode(args.gemm, bf16)
    if gm["op"] in kernels:
        H = C
        so2 = 2 * 70 * C * C + 2 * 29 * C * C
        rad = 2 * ((B + 2 * C) * H + H * H + H * 12 * C)
        flops = 2 * E * (so2 + rad) - (E * 2 * 2 * C * H if use_fused else 0)
        ms = kernels[gm["op"]]["ms_per_step"]
        tf = flops / (ms * 1e-3) / 1e12
        kernels[gm["op"]].update(alg_flops_per_step=flops, alg_tflops=tf, frac_tensor_peak=tf / bf16,
                                 passes=gm["passes"], pipe=gm["pipe"], tflops_pipe=gm["passes"] * tf,
                                 frac_pipe_peak=gm["passes"] * tf / gm["peak"])
    del step, layer, inp, gout, x0, xe, wig, env, graph
    torch.cuda.empty_cache()
    return {"metric": "one message-passing layer fwd+bwd (BASELINE config 2)", "nodes": N, "edges": E,
            "ms_per_layer": total, "gemm": gm["label"],
            "peaks": {"hbm_gbs": hbm, "tensor_tflops": bf16, "pipe_tflops": gm["peak"], "kind": kind,
                      "note": gm["peak_note"]},
            "kernels": dict(sorted(kernels.items(), key=lambda kv: -kv[1]["ms_per_step"]))}


# (K, N, launches per config-3 step) of the step's dense contractions (M = edges): forward radial
# MLPs (4 layers + the initial one), SO(2) convolutions, and the input-gradient GEMMs
STEP_GEMMS = [(320, 128, 5), (128, 128, 5), (128, 1536, 4), (128, 384, 1), (768, 640, 4), (1024, 512, 4),
              (512, 256, 4), (384, 384, 4), (512, 512, 4), (256, 256, 4),
              (384, 384, 4), (512, 512, 4), (256, 256, 4), (640, 768, 4), (512, 1024, 4), (256, 512, 4),
              (1536, 128, 4), (384, 128, 1), (128, 128, 5), (128, 64, 5)]


def run_gemm_shapes(args, device, M=120000, reps=10):
    """Device time of every dense-contraction shape of the config-3 step on pre-split operands,
    row-major tiles against the transposed 128 x 256 tiles (FUMA_GEMM_T), CUDA events over
    ``reps`` launches with the L2 flushed first; fp16-pipe TF/s (3 products per fp32 product)."""
    from flash_uma_b200 import _native
    from flash_uma_b200.linear import _gemm16, _split16, check_errors, split_rows
    _native.load()
    _, bf16, _ = load_peaks()
    flush = torch.empty(256 * 1024 * 1024 // 4, device=device)
    rows, tot = [], {"0": 0.0, "1": 0.0}
    g = torch.Generator(device=device).manual_seed(0)
    for K, N, count in STEP_GEMMS:
        W = torch.randn(N, K, device=device, generator=g) / K ** 0.5
        w16 = _split16(W)
        xp = split_rows(torch.randn(M, K, device=device, generator=g))
        row = {"K": K, "N": N, "launches_per_step": count}
        for t in ("0", "1"):
            os.environ["FUMA_GEMM_T"] = t
            for _ in range(3):
                _gemm16(xp, w16, None, K)
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(reps):
                _gemm16(xp, w16, None, K)
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / reps
            row[f"ms_T{t}"] = round(ms, 4)
            row[f"pipe_frac_T{t}"] = round(3 * 2 * M * N * K / (ms * 1e-3) / 1e12 / bf16, 4)
            tot[t] += ms * count
        rows.append(row)
    os.environ.pop("FUMA_GEMM_T", None)
    check_errors()
    print(json.dumps({"metric": "dense-contraction shapes of the config-3 step (M = 120,000, pre-split f16x3)",
                      "ms_per_step_T0": round(tot["0"], 3), "ms_per_step_T1": round(tot["1"], 3),
                      "shapes": rows}), flush=True)


def kernel_fractions(micro):
    """Compact per-kernel HBM fractions of the config-2 microbench for the bench line."""
    out = {}
    for name, k in micro["kernels"].items():
        if "frac_hbm" in k:
            out[name] = {"frac_hbm": round(k["frac_hbm"], 4), "achieved_gbs": round(k["achieved_gbs"], 1),
                         "ms_per_call": round(k["ms_per_step"] / max(1, k["launches_per_step"]), 4)}
        elif "frac_tensor_peak" in k:
            out[name] = {"frac_tensor_peak": round(k["frac_tensor_peak"], 4),
                         "frac_pipe_peak": round(k["frac_pipe_peak"], 4), "ms_per_step": round(k["ms_per_step"], 4)}
    return {"workload": f"BASELINE config 2: one layer fwd+bwd, N={micro['nodes']}, E={micro['edges']}",
            "ms_per_layer": round(micro["ms_per_layer"], 4), "hbm_peak_gbs": micro["peaks"]["hbm_gbs"],
            "timing": "CUDA events around every C-ABI call (fwd+bwd of the layer, inputs resident)",
            "kernels": out}


# the reference's published FlashUMA step times for its atom-count sweep (random graphs, ~50
# edges per atom, pretrained uma-s-1p2, E+F+S, torch.compile, GPU model not stated):
# examples/make_plots.py:14
REFERENCE_SWEEP_MS = {100: 15.27, 200: 16.88, 500: 16.92, 1000: 23.00, 2000: 43.51}


def run_sweep(args, device):
    """Step time (energy + forces + stress) over the reference's atom-count sweep: random
    clusters of 100-2,000 atoms with 50 edges per atom, C = 128, 4 layers, random-init weights.
    Each size: CUDA-graph replays (the whole step captured once) and eager launches, CUDA-event
    medians over ``--steps`` steps after ``--warmup``."""
    import dataclasses
    import statistics as st

    from flash_uma_b200 import _native
    from flash_uma_b200.predict import GraphedStep, Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import random_cluster_graph
    from flash_uma_b200.wrapper import ZeroAllocBackbone
    _native.load()
    off = SyntheticESCNMDBackbone(seed=0).to(device)
    pred = Predictor(ZeroAllocBackbone(off, gemm=args.gemm), make_energy_head(128, 128, seed=1).to(device))
    rows = []
    for n in sorted(REFERENCE_SWEEP_MS):
        data = random_cluster_graph(n, 50, seed=n).to(device)
        g = torch.Generator().manual_seed(n)
        pos = [data.pos + 0.01 * torch.randn(data.pos.shape, generator=g).to(device) for _ in range(args.steps)]

        def timed(fn):
            for k in range(args.warmup):
                fn(pos[k % len(pos)])
            torch.cuda.synchronize()
            ts = []
            for k in range(args.steps):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record()
                fn(pos[k])
                b.record()
                ts.append((a, b))
            torch.cuda.synchronize()
            return st.median(x.elapsed_time(y) for x, y in ts)

        eager = timed(lambda p: pred(dataclasses.replace(data, pos=p), stress=True))
        step = GraphedStep(pred, data, stress=True)
        graph = timed(step)
        rows.append({"atoms": n, "edges": int(data.edge_index.shape[1]), "ms_per_step_graph": graph,
                     "ms_per_step_eager": eager, "reference_published_ms": REFERENCE_SWEEP_MS[n]})
        del step
    print(json.dumps({"metric": "ms per energy+forces+stress step, reference atom-count sweep (50 edges/atom)",
                      "unit": "ms", "higher_is_better": False, "gemm": args.gemm, "steps": args.steps,
                      "warmup": args.warmup, "data": "synthetic random clusters, random-init weights",
                      "reference_note": "published FlashUMA times (examples/make_plots.py:14) are for the "
                                        "pretrained uma-s-1p2 on an unstated GPU with torch.compile",
                      "sizes": rows}), flush=True)


REF_DIR = os.path.join(ROOT, "baseline", "_ref")


def load_reference_gpu():
    """The unmodified reference implementation from ``baseline/_ref`` (installed by
    ``baseline/install_reference.py``): its wrapper module, whose ``ZeroAllocBackbone`` runs the
    reference's Triton kernels natively on the GPU. ``model.py`` imports
    ``balance_channels_batched`` from fairchem at load time (``model.py:11``), which is not
    installed; the same stand-in this build uses is registered under that module name (it is
    only called for models with charge / spin channel ranges). None if not installed."""
    import types
    if not os.path.isfile(os.path.join(REF_DIR, "wrapper.py")):
        return None
    # The reference autotunes its Triton kernels on first use (minutes of compiling and timing
    # candidate configurations on a fresh machine). Triton's own on-disk cache, with autotuning
    # results included, is kept next to the installed reference so that a fresh box starts from
    # the results of an earlier run on the same GPU model. TRITON_CACHE_DIR is set, not
    # defaulted: torch.compile points it at inductor's own cache once it has compiled anything in
    # the process, and the reference would then autotune from scratch (~11 minutes measured in a
    # test session that compiled a model first). FLASHUMA_REF_TRITON_CACHE_DIR picks another.
    os.environ["TRITON_CACHE_DIR"] = os.environ.get("FLASHUMA_REF_TRITON_CACHE_DIR",
                                                    os.path.join(REF_DIR, "triton_cache"))
    os.environ.setdefault("TRITON_CACHE_AUTOTUNING", "1")
    from flash_uma_b200.nodewise import balance_channels_batched
    for name in ["fairchem", "fairchem.core", "fairchem.core.models", "fairchem.core.models.uma",
                 "fairchem.core.models.uma.escn_md"]:
        sys.modules.setdefault(name, types.ModuleType(name))
    sys.modules["fairchem.core.models.uma.escn_md"].balance_channels_batched = balance_channels_batched
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    import wrapper as ref_wrapper   # noqa: E402  (baseline/_ref/wrapper.py)
    return ref_wrapper


def run_reference_gpu(device, steps: int, warmup: int, system, tf32: bool, check=None):
    """The reference's own Triton path on this GPU (``ZeroAllocBackbone`` of ``baseline/_ref``,
    ``wrapper.py:171-211`` -> ``model.py:187-221`` -> ``ops/*.py``) on the bench workload: the
    same seed-0 weights, node-wise stand-ins, energy head and MD-like positions as the flash arm,
    energy + forces per step, eager launches (its stock path), CUDA events per step with the L2
    flushed in between, as ``examples/benchmark.py:33-56`` times it. ``tf32``: cuBLAS TF32 for
    its F.linear calls (the reference's published setting) or full fp32. ``check``: (energy,
    forces) of the flash arm at the first position, compared with the reference's result."""
    import dataclasses

    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from flash_uma_b200.systems import to_graph
    ref_wrapper = load_reference_gpu()
    if ref_wrapper is None:
        return {"unavailable": "baseline/_ref not installed (python baseline/install_reference.py <reference>)"}
    prev = (torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32)
    torch.backends.cuda.matmul.allow_tf32 = tf32
    torch.backends.cudnn.allow_tf32 = tf32
    try:
        off = SyntheticESCNMDBackbone(seed=0).to(device)
        head = make_energy_head(128, 128, seed=1).to(device)
        pred = Predictor(ref_wrapper.ZeroAllocBackbone(off, dtype=torch.float32), head)
        data_cpu = to_graph([system])
        data = data_cpu.to(device)
        N = data_cpu.pos.shape[0]
        pos_seq = [p.to(device) for p in md_positions(data_cpu.pos, steps + warmup, seed=0)]
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        t0 = time.perf_counter()
        for w in range(warmup):   # the first call autotunes and compiles the Triton kernels
            res = pred(dataclasses.replace(data, pos=pos_seq[w]))
        torch.cuda.synchronize()
        warm_s = time.perf_counter() - t0
        parity = None
        if check is not None:
            res = pred(dataclasses.replace(data, pos=pos_seq[0]))
            e_ref, f_ref = res["energy"].double(), res["forces"].double()
            e, f = check[0].double(), check[1].double()
            parity = {"energy_rel": float(((e - e_ref).abs() / e_ref.abs().clamp_min(1.0)).max()),
                      "forces_max_abs": float((f - f_ref).abs().max()),
                      "note": "flash arm vs this reference run at the same positions"}
        sampler = ClockSampler(device.index if device.index is not None else 0)
        torch.cuda.synchronize()
        sampler.start()
        evs = []
        for k in range(steps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            pred(dataclasses.replace(data, pos=pos_seq[warmup + k]))
            e1.record()
            evs.append((e0, e1))
        torch.cuda.synchronize()
        clocks = sampler.stop()
        ms = sum(a.elapsed_time(b) for a, b in evs) / steps
        out = {"value": N / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms, "steps": steps, "warmup": warmup,
               "tf32": tf32, "launch": "eager (the reference's stock path)", "warmup_s": round(warm_s, 1),
               "max_device_memory_gb": torch.cuda.max_memory_allocated(device) / 1e9, "clocks": clocks}
        if parity is not None:
            out["parity"] = parity
        return out
    except Exception as exc:   # noqa: BLE001 - reported in the line, the flash arm's number stands
        return {"unavailable": f"reference Triton path failed: {type(exc).__name__}: {exc}"[:400]}
    finally:
        torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = prev
        torch.cuda.empty_cache()


def _oracle_predictor():
    from flash_uma_b200.predict import Predictor
    from flash_uma_b200.synthetic import SyntheticESCNMDBackbone, make_energy_head
    from oracle.model import OracleBackbone
    return Predictor(OracleBackbone(SyntheticESCNMDBackbone(seed=0)), make_energy_head(128, 128, seed=1))


def cpu_oracle_rate(max_seconds: float = 30.0):
    """``cpu_baseline`` of the N = 1 line: the CPU oracle (PyTorch restatement of the reference,
    fp32, all host threads) on the full config-3 system, one E+F step timed after a warm-up step
    on a 256-atom bulk-Cu cell (thread pool and allocator); more steps while under max_seconds."""
    from flash_uma_b200.systems import bulk_fcc, config3_system, to_graph
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    pred = _oracle_predictor()
    pred(to_graph([bulk_fcc(4, 4, 4, jitter=0.05, seed=0)]))
    data = to_graph([config3_system()])
    atoms = data.pos.shape[0]
    t0 = time.perf_counter()
    steps = 0
    while steps == 0 or time.perf_counter() - t0 < max_seconds / 2:
        pred(data)
        steps += 1
    dt = time.perf_counter() - t0
    return {"value": atoms * steps / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"the full config-3 system (bulk Cu 10x10x10, {atoms} atoms, {data.edge_index.shape[1]} edges), "
                      f"{steps} E+F step(s) in {dt:.1f} s after a 256-atom warm-up step"}


def run_reference(args, budget_s: float = 180.0):
    """``--impl reference``: the reference's CPU implementation of the path (its PyTorch
    restatement, ``oracle/``; the reference itself is Triton-only) on all host threads, on the
    same workload as the flash arm (config 3, 4,000 atoms, E+F per step). A CPU step takes tens
    of seconds, so the run is bounded: one warm-up step, then timed steps until ``--steps`` are
    done or ``budget_s`` has passed (at least two); ``steps`` reports the steps actually timed."""
    from flash_uma_b200.systems import config3_system, to_graph
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    data = to_graph([config3_system()])
    atoms, edges = data.pos.shape[0], data.edge_index.shape[1]
    pred = _oracle_predictor()
    warm = min(args.warmup, 1)
    for _ in range(warm):
        pred(data)
    t0 = time.perf_counter()
    steps = 0
    while steps < args.steps and (steps < 2 or time.perf_counter() - t0 < budget_s):
        pred(data)
        steps += 1
    dt = time.perf_counter() - t0
    v = atoms * steps / dt
    return {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
            "steps": steps, "steps_requested": args.steps, "warmup": warm, "ms_per_step": dt * 1e3 / steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded bulk Cu positions, random-init weights)",
            "config": {"workload": f"bulk_cu_4000 (BASELINE config 3), E+F per step: {atoms} atoms, {edges} edges, "
                                   "CPU (PyTorch restatement of the reference)",
                       "atoms": atoms, "edges": edges, "sphere_channels": 128, "layers": 4,
                       "num_distance_basis": 64, "same_config": True},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"the full config-3 system per step ({atoms} atoms), {steps} timed steps "
                                       f"(bounded to ~{budget_s:.0f} s), {warm} warm-up"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def summarize_launches(path):
    """Kernels between the first two L2-flush fills of an ncu launch list of ``bench.py --steps 1``
    (the one timed step of the device-resident region), grouped by kernel: launches, total
    device time, share. ncu serialises launches and runs them with cold caches, so the shares
    are what compares with the bench, not the absolute times."""
    import collections
    import csv
    rows = list(csv.reader(open(path)))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    h = rows[hi]
    ki, vi, ui = h.index("Kernel Name"), h.index("Metric Value"), h.index("Metric Unit")
    seq = []
    for r in rows[hi + 1:]:
        if len(r) <= vi:
            continue
        v = float(r[vi].replace(",", ""))
        unit = r[ui]
        v = v / 1e3 if unit.startswith("n") else v * 1e3 if unit.startswith("m") else v   # -> microseconds
        seq.append((r[ki], v))
    flush = [i for i, (n, v) in enumerate(seq) if "FillFunctor" in n and v > 20.0]
    a, b = flush[0] + 1, flush[1]
    tot, cnt = collections.defaultdict(float), collections.Counter()
    for n, v in seq[a:b]:
        k = n.split("(")[0].replace("void ", "")
        k = k if len(k) < 80 else k[:77] + "..."
        tot[k] += v
        cnt[k] += 1
    T = sum(tot.values())
    own = sum(v for k, v in tot.items() if k.startswith("fuma::"))
    print(f"one timed step: {b - a} launches, {T / 1e3:.2f} ms of kernel time (serialised, cold caches); "
          f"this library's kernels {100 * own / T:.1f}%, others {100 * (T - own) / T:.1f}%")
    print(f"{'ms':>9} {'share':>6} {'n':>4}  kernel")
    for k, v in sorted(tot.items(), key=lambda kv: -kv[1]):
        print(f"{v / 1e3:9.3f} {100 * v / T:5.1f}% {cnt[k]:4d}  {k}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="flash", choices=["flash", "reference"])
    ap.add_argument("--workload", default="default", choices=["default", "config4", "config5"],
                    help="default: config 3 (weak scaling of it for N > 1); config4: water box E+F+S; "
                         "config5: 100,800-atom bulk Cu (strong scaling)")
    ap.add_argument("--gemm", default="f16x3", choices=["f16x3", "tf32x3", "tf32", "f16"],
                    help="dense-contraction mode: f16x3 / tf32x3 (fp32-level) or tf32 (single pass, the "
                         "reference's published setup)")
    ap.add_argument("--summarize-launches", metavar="CSV",
                    help="print the per-kernel table of one timed step from an ncu launch list "
                         "(--metrics gpu__time_duration.sum --csv of 'bench.py --steps 1') and exit")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", dest="graph", action="store_false",
                    help="launch every kernel from the host each step instead of replaying a CUDA graph")
    ap.add_argument("--micro", action="store_true", help="one-layer kernel microbench (BASELINE config 2)")
    ap.add_argument("--sweep", action="store_true",
                    help="step time over the reference's atom-count sweep (100-2,000 atoms, 50 edges/atom, E+F+S)")
    ap.add_argument("--no-reference-gpu", dest="reference_gpu", action="store_false",
                    help="skip timing the reference's Triton path on this GPU (N = 1 default workload)")
    ap.add_argument("--no-strong5", dest="strong5", action="store_false",
                    help="skip the config-5 strong-scaling object (100,800 atoms at this run's N)")
    ap.add_argument("--no-kernels", dest="kernels", action="store_false",
                    help="skip the per-kernel config-2 fractions of the N = 1 line")
    ap.add_argument("--gemm-shapes", action="store_true",
                    help="time the step's dense-contraction shapes, row-major vs transposed tiles")
    ap.add_argument("--nodes", type=int, default=20000)
    ap.add_argument("--edges", type=int, default=600000)
    args = ap.parse_args()
    if args.workload == "config5":
        # ~150 GB of activations on one GPU: growable segments keep the caching allocator from
        # stranding tens of GB in fragments (set before the first CUDA allocation)
        os.environ.setdefault("PYTORCH_CUDA_ALLOC_CONF", "expandable_segments:True")
    if args.summarize_launches:
        summarize_launches(args.summarize_launches)
        return
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    if args.micro:
        if rank == 0:
            print(json.dumps(run_micro(args, device)), flush=True)
        return
    if args.sweep:
        if rank == 0:
            run_sweep(args, device)
        return
    if args.gemm_shapes:
        if rank == 0:
            run_gemm_shapes(args, device)
        return
    if world > 1:
        import datetime
        torch.distributed.init_process_group("nccl", device_id=device, timeout=datetime.timedelta(seconds=120))
    try:
        out = run_flash(args, rank, world, device)
        check0 = out.pop("_check")
        pos0 = out.pop("_pos0")
        if args.strong5 and args.workload == "default":
            # every rank takes part (the partitioned step has collectives)
            out["strong_config5"] = run_strong5(args, rank, world, device)
        if rank == 0 and world == 1 and args.workload == "default":
            if args.reference_gpu:
                # the reference's own Triton path on the same GPU and workload: full fp32 (the
                # accuracy class of this build's f16x3 path and of the parity bar) and TF32 (its
                # published setting); ratio = this build's value / the reference's
                system, _, _, _ = workload_system(args.workload, world)
                rg = {}
                for key, tf32 in (("fp32", False), ("tf32", True)):
                    r = run_reference_gpu(device, min(args.steps, 10), 3, system, tf32, check=check0)
                    if "value" in r:
                        r["ratio"] = out["value"] / r["value"]
                        r["e2e_ratio"] = out["e2e"]["value"] / r["value"]
                    rg[key] = r
                out["reference_triton_gpu"] = rg
            if args.gemm == "f16x3":
                # the TF32 accuracy class on both sides: this build's single-product fp16 mode
                # against the reference with TF32 on
                fast = run_mode(device, "f16", min(args.steps, 10), 3, workload_system(args.workload, world)[0],
                                check=check0)
                ref_tf32 = out.get("reference_triton_gpu", {}).get("tf32", {})
                if "value" in ref_tf32:
                    fast["ratio_vs_reference_tf32"] = fast["value"] / ref_tf32["value"]
                out["tf32_class_mode"] = fast
            if args.kernels:
                margs = argparse.Namespace(**vars(args))
                margs.nodes, margs.edges, margs.steps, margs.warmup = 20000, 600000, 5, 3
                out["kernels"] = kernel_fractions(run_micro(margs, device))
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()
    if rank == 0:
        if world > 1:
            # after the process group is gone, so no rank waits on a collective meanwhile
            out["parity"] = partition_parity(args, device, check0, pos0)
        if world == 1 and not args.no_cpu_baseline:
            out["cpu_baseline"] = cpu_oracle_rate()
        print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
