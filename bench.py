#!/usr/bin/env python
"""Benchmark of the hot path: forward + exact adjoint, compartment-timesteps/s.

Default line (config 4, the network configuration the metric is quoted on at
1/2/4/8 GPUs): one event network of 10,000 seeded random-tree cells (hh +
pas, somatic IClamp), 100 Exp2Syn per cell from random presynaptic cells plus
one NetStim-driven Exp2Syn (5 Hz, noise 1), 8000 steps of dt 0.025 ms.  One
step = forward with checkpointed tape, soma-voltage MSE against a teacher
network (weights perturbed lognormally, sigma 0.2), and the reverse sweep
producing the gradients of every synaptic weight and every hh gnabar (the
kinds the bench asks for; the sweep accumulates only those).  On N GPUs the
SAME network is
sharded by cell (strong scaling); after every minimum-delay window the ranks
all-gather their window spikes over NCCL.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config 2|3|4|5|6]

Other configurations of the same metric (not the default line):
  --config 2   1024 independent random-tree cells per GPU, 4000 steps (no
               collective; weak scaling);
  --config 3   one 50,000-compartment cell (<= 40 branch levels), 2000 steps,
               split across CTAs (cooperative launch), gradients of every
               segment's conductances;
  --config 5   302 cells coupled by 900 HalfGap pairs and 2000 graded
               synapses, 8000 steps (replicas on N GPUs);
  --config 6   library cells: --ncell random trees (default 1024, config-2
               morphology) carrying the user-mech channel set of a layer-5
               pyramidal cell with calcium dynamics (NaTg, Nap_Et2, K_Pst,
               K_Tst, SKv3_1, SK_E2, Im, Ca_HVA, Ca_LVAst, CaDynamics_E2,
               ions) and pas, 4000 steps, gradients of every channel density
               and CaDynamics_E2 gamma.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "fwd+bwd compartment-timesteps/sec"
UNIT = "comp-steps/s"
T_STEPS = 4000
NCELL = 1024
NCELL_NET = 10000
SEED0 = 20240
# DRAM bytes per compartment-step of the network reverse kernel, measured by
# ncu (dram__bytes_read.sum + dram__bytes_write.sum of one bwd_kernel launch
# over 1250 config-4 cells x 200 steps with this bench's gradient kinds, / its
# compartment-steps); scaled to a launch of the timed configuration as
# roofline.traffic (config 4 only)
REV_DRAM_BYTES_PER_UNIT_NET = 209.9


def _alg_bytes(g):
    """Algorithmic HBM bytes per timestep for the whole group.

    Per compartment B_c = 8*(3 p_c + 8 s_c) + 12 (p_c parameters, s_c states):
    one forward, one checkpoint-recompute forward and one adjoint step.  The
    forward's share is 8*(p_c + 2 s_c) + 4 (read parameters and states, write
    the tape), the backward pass's the rest, of which the reverse kernel alone
    (parameters, tape row, state adjoints read and written) moves
    8*(p_c + 4 s_c) + 4.  Returns (forward, backward pass, reverse kernel,
    total).
    """
    import numpy as np

    hh = np.zeros(g.nnode, bool)
    hh[g.hh.nodes] = True
    pas = np.zeros(g.nnode, bool)
    pas[g.pas.nodes] = True
    p = 3 + 4 * hh + 2 * pas
    s = 1 + 3 * hh
    # library mechanisms: their states and parameters per instance (ions: erev / cai, cao)
    from heliox_b200.model import LIB_FIELDS, LIB_STATES

    for nm, tab in g.lib.items():
        np.add.at(s, tab.nodes, len(LIB_STATES.get(nm, ())))
        np.add.at(p, tab.nodes, len(LIB_FIELDS[nm]))
    # event synapses: 2 states, 2 parameters each (188 B per instance-step)
    nsyn = g.expsyn.n + g.exp2syn.n
    p_all, s_all, n_all = float(p.sum()) + 2 * nsyn, float(s.sum()) + 2 * nsyn, g.nnode + nsyn
    fwd = 8 * (p_all + 2 * s_all) + 4 * n_all
    tot = 8 * (3 * p_all + 8 * s_all) + 12 * n_all
    rev = 8 * (p_all + 4 * s_all) + 4 * n_all
    return fwd, tot - fwd, rev, tot


def _peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, phys_index: int):
        self.idx = phys_index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "--query-gpu=" + self.FIELDS, "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except Exception:
            self.proc.kill()
            out, _ = self.proc.communicate()
        sm, smax, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in out.strip().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# ----------------------------------------------------------------------------- CPU baseline
def _cpu_sample(config: int):
    """The bounded CPU sample of a configuration: (description, jobs, steps per
    job).  A job is one independent unit the reference integrates in one
    process (it is single-threaded and has no multi-process mode): a
    config-2 cell, or a small network of the config-4 recipe (its own cells'
    synapses and NetStims, sources among its 8 cells)."""
    if config == 4:
        return "8-cell networks of the config-4 recipe, 2000 steps each", "net8", 2000
    return "cells of the config-2 batch, 4000 steps each", "cell", T_STEPS


def _cpu_job(args):
    """One job on one host core: forward + adjoint; returns (units, seconds).

    With the reference harness built (oracle/_ref), the forward is the
    reference's own CPU integrator (its CoreNEURON loader, Simulate::
    finitialize + fadvance), timed inside the harness around the integration
    alone; the reverse sweep -- which the reference does not have -- is the
    oracle's, timed inside the oracle around its reverse loop.  Otherwise the
    forward is the oracle's taped forward, timed the same way.
    """
    kind, seed, nstep, use_ref = args
    sys.path.insert(0, ROOT)
    import numpy as np

    from heliox_b200 import synth
    from oracle import oracle as O

    if kind == "net8":
        g = synth.network_config4_shard(8, 0, 1, seed=1000 + seed)
    else:
        g = synth.random_tree_cell(seed)
    t0 = time.perf_counter()
    tr, _ = O.forward(g, nstep)
    t_fwd_port = time.perf_counter() - t0
    dLdv = np.zeros_like(tr)
    dLdv[1:] = 2.0 * tr[1:] / nstep
    _, gr = O.adjoint(g, nstep, dLdv)
    t_rev = gr["reverse_s"]
    t_fwd = O.ref_forward(g, nstep, timing=True)[2] if use_ref else t_fwd_port
    return g.nnode * nstep, t_fwd + t_rev


def cpu_baseline(config: int, njobs: int, procs: int):
    """Forward + adjoint of a bounded sample on host cores (spawn pool, no CUDA
    in the workers).  Returns (units per second over all cores, units, busy
    seconds per core, kind, sample description)."""
    import multiprocessing as mp

    from oracle import oracle as O

    use_ref = O.ref_available()
    desc, kind, nstep = _cpu_sample(config)
    ctx = mp.get_context("spawn")
    jobs = [(kind, SEED0 + c, nstep, use_ref) for c in range(njobs)]
    with ctx.Pool(procs) as pool:
        res = pool.map(_cpu_job, jobs)
    units = sum(r[0] for r in res)
    busy = sum(r[1] for r in res) / procs  # all cores busy in parallel
    return units / busy, units, busy, ("reference" if use_ref else "port"), f"{njobs} {desc}"


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    ws, rank, local = _dist()
    if rank != 0:
        return 0
    procs = os.cpu_count() or 1
    vals = []
    njobs = max(procs, 8)
    kind, desc = "port", ""
    for it in range(args.warmup + args.steps):
        v, units, wall, kind, desc = cpu_baseline(args.config, njobs, procs)
        if it >= args.warmup:
            vals.append(v)
    value = statistics.median(vals)
    fwd_by = "the reference's CPU integrator (timed inside its harness)" if kind == "reference" else "oracle port"
    line = {
        "impl": "reference",
        "metric": METRIC,
        "value": value,
        "unit": UNIT,
        "n_gpus": args.gpus,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "strong" if args.config == 4 else "weak",
        "vs_baseline": None,
        "dtype": "f64",
        "data": "synthetic",
        "config": {"workload": _workload_name(args), "sample": f"{desc} per step, on {procs} host cores"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": procs, "kind": kind,
                         "sample": f"{desc}; forward: {fwd_by}, adjoint: oracle port (the reference has none)"},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def _workload_name(args) -> str:
    return {2: f"config2: random-tree cells x {T_STEPS} steps per GPU, fwd+bwd",
            3: "config3: one 50,000-compartment cell x 2000 steps, fwd+bwd",
            4: f"config4: event network of {args.ncell or NCELL_NET} cells x 8000 steps, fwd+bwd",
            5: "config5: 302 coupled cells x 8000 steps, fwd+bwd",
            6: f"config6: library cells x {T_STEPS} steps per GPU, fwd+bwd"}[args.config]


# ----------------------------------------------------------------------------- our arm
def run_ours(args):
    import numpy as np
    import torch

    from heliox_b200 import synth
    from heliox_b200.runtime import Sim

    ws, rank, local = _dist()
    dist = None
    if ws > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    # an explicit stream: the legacy default stream (handle 0) would not order
    # the library's launches against the timing events
    stream = torch.cuda.Stream(dev)
    torch.cuda.set_stream(stream)

    # ---- synthetic workload (per rank: its own cells)
    W = build_workload(args, ws, rank)
    g, teacher, T, keys = W["group"], W["teacher"], W["nstep"], W["keys"]
    probes = W["probes"]
    ncomp = g.nnode

    if W.get("exchange"):
        # one window for all ranks: the smallest over the ranks' own bounds
        wt = torch.tensor([W["window"]], dtype=torch.int64, device=dev)
        dist.all_reduce(wt, op=dist.ReduceOp.MIN)
        W["window"] = int(wt.item())
        W["exchange_cap"] = 0  # the library's default window buffer, grown together on overflow

    def new_sim(grp):
        sim = Sim(local)
        sim.set_stream(stream.cuda_stream)
        sim.load_group(grp, gid_base=W.get("gid_base", 0), nsrc_cells=W.get("nsrc_cells", 0))
        if W.get("exchange"):
            from heliox_b200 import shard

            sim.set_window(W["window"])
            sim.set_exchange(shard.allgather_exchange(), ws, W["exchange_cap"])
        return sim

    tsim = new_sim(teacher)
    target_h = tsim.simulate(T, probes=probes)
    torch.cuda.synchronize()
    if W.get("exchange"):
        tsim.set_exchange(None, 1)
    tsim.close()
    del tsim

    s = new_sim(g)
    s.set_grad_kinds(keys)  # the workload's gradients only (the reverse sweep skips the other accumulators)
    target = torch.from_numpy(target_h).to(dev)
    trace = torch.empty_like(target)
    dLdv = torch.empty_like(target)
    loss = torch.zeros(1, dtype=torch.float64, device=dev)
    counts = {k: s._count(k) for k in keys}
    grads = {k: torch.empty(max(n, 1), dtype=torch.float64, device=dev) for k, n in counts.items()}
    nprobe = int(probes.shape[0])
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)  # > L2 (126 MB)

    def step(ev=None):
        if ev is not None:
            ev[0].record(stream)
        s.forward_capture_dev(T, trace.data_ptr(), probes=probes)
        if ev is not None:
            ev[1].record(stream)
        s.mse_loss_grad_dev(trace.data_ptr(), target.data_ptr(), T + 1, nprobe, dLdv.data_ptr(), loss.data_ptr())
        if ev is not None:
            ev[2].record(stream)
        s.backward_dev(dLdv.data_ptr(), {k: v.data_ptr() for k, v in grads.items()})
        if ev is not None:
            ev[3].record(stream)

    for _ in range(args.warmup):
        step()
        flush.fill_(1.0)
    torch.cuda.synchronize()

    phys = local
    cvd = os.environ.get("CUDA_VISIBLE_DEVICES")
    if cvd:
        try:
            phys = int(cvd.split(",")[local])
        except ValueError:
            phys = local
    sampler = ClockSampler(phys)
    sampler.start()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    t_start = torch.cuda.Event(enable_timing=True)
    t_end = torch.cuda.Event(enable_timing=True)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    t_start.record(stream)
    for k in range(args.steps):
        step(evs[k])
        flush.fill_(1.0)  # L2 flush between timed steps
    t_end.record(stream)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    clocks = sampler.stop()
    ms = t_start.elapsed_time(t_end)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    loss_val = float(loss.item())
    # launches of our kernels per step, as the runtime counts them (forward
    # and backward kernels, incl. windows / checkpoint replays / per-step
    # launches of coupled groups) plus init, MSE (2) and the gradient gathers
    _, nf = s.last_kernel_ms(0)
    _, nb = s.last_kernel_ms(1)
    gpu_launches = args.steps * (1 + nf + 2 + nb + len(keys))
    # the reverse kernel alone (last timed step; a checkpointed backward
    # alternates segment recompute and reverse launches)
    rev_ms, nrev = s.last_kernel_ms(2)

    # ---- end to end through the public host-buffer API (params in, loss/grads out),
    # host buffers page-locked (inputs from pinned host memory, results read
    # into pinned memory), allocated once outside the timed region
    from heliox_b200.runtime import pinned_empty

    host_params = {}
    for k in keys:
        host_params[k] = pinned_empty(counts[k])
        host_params[k][:] = s.get_param_array(k)
    tr_h = pinned_empty((T + 1, nprobe))
    dl_h = pinned_empty((T + 1, nprobe))
    grads_h = {k: pinned_empty(counts[k]) for k in keys}
    if not W.get("exchange"):  # host API on the context's own stream
        s.set_stream(0)
    torch.cuda.synchronize()
    h2d = sum(v.nbytes for v in host_params.values()) + (T + 1) * nprobe * 8
    d2h = (T + 1) * nprobe * 8 + sum(8 * counts[k] for k in keys)
    if dist:
        dist.barrier()
    e2e_steps = args.steps if args.config == 2 else min(args.steps, 2)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        for k in keys:
            s.set_param_array(k, host_params[k])
        s.forward_capture(T, probes=probes, out=tr_h)
        np.subtract(tr_h, target_h, out=dl_h)
        dl_h *= 2.0 / (T * nprobe)
        dl_h[0] = 0.0
        s.backward(dl_h, keys=keys, out=grads_h)
    e2e_s = (time.perf_counter() - t0) * args.steps / e2e_steps
    if dist:
        dist.barrier()

    # ---- max over ranks
    fb, bb, rb, tb = _alg_bytes(g)
    vals = torch.tensor([ms, e2e_s, fwd_ms, bwd_ms, rev_ms, float(ncomp), fb, bb, rb, tb], dtype=torch.float64,
                        device=dev)
    if dist:
        mx = vals.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        tot = vals.clone()
        dist.all_reduce(tot, op=dist.ReduceOp.SUM)
        ms, e2e_s, fwd_ms, bwd_ms, rev_ms = (float(x) for x in mx[:5])
        total_comp = float(tot[5])
        fb, bb, rb, tb = (float(x) for x in mx[6:10])  # the slowest rank's share bounds the kernel times
    else:
        total_comp = float(ncomp)
    units_per_step = total_comp * T
    value = units_per_step * args.steps / (ms / 1e3)
    e2e_value = units_per_step * args.steps / e2e_s

    if rank == 0:
        peak, peak_src = _peaks()
        # roofline of the reverse kernel (the dominant one): its algorithmic bytes
        # per launch / its mean launch time (CUDA events on the launch stream)
        achieved = rb * T / (rev_ms / 1e3) / 1e9
        line = {
            "metric": METRIC,
            "value": value,
            "unit": UNIT,
            "n_gpus": ws,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": ms / args.steps,
            "higher_is_better": True,
            "scaling": W["scaling"],
            "vs_baseline": None,
            "dtype": "f64",
            "data": "synthetic",
            "config": {
                "workload": W["workload"],
                "compartments_total": int(total_comp),
                "compartments_per_gpu": ncomp,
                "parallelism": W["parallelism"].format(ws=ws),
                "l2": "tape exceeds L2; 256 MiB flush write between steps",
                "loss": loss_val,
            },
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
            "gpu_launches": gpu_launches,
            "fwd_ms": fwd_ms,
            "bwd_ms": bwd_ms,
            "roofline": {
                "bound": "hbm",
                "kernel": "bwd_kernel" + ("<net>" if g.has_network else ""),
                "achieved": achieved,
                "peak": peak,
                "peak_source": peak_src,
                "unit": "GB/s",
                "frac": achieved / peak,
                "traffic": (REV_DRAM_BYTES_PER_UNIT_NET * ncomp * T / max(nrev, 1) if args.config == 4 else None),
                "traffic_source": "ncu, 1250 config-4 cells x 200 steps, per compartment-step x this launch's",
                "alg_bytes_per_launch": rb * T / max(nrev, 1),
                "launches_per_step": nrev,
                "kernel_ms_per_step": rev_ms,
                "fwd_frac": (fb * T / (fwd_ms / 1e3) / 1e9) / peak,
                "bwd_pass_frac": (bb * T / (bwd_ms / 1e3) / 1e9) / peak,
                "path_frac": (tb * T / ((fwd_ms + bwd_ms) / 1e3) / 1e9) / peak,
            },
            "clocks": clocks,
        }
        if ws == 1 and not args.no_cpu and args.config in (2, 4):
            procs = os.cpu_count() or 1
            v, units, wall, kind, desc = cpu_baseline(args.config, 2 * max(procs, 8), procs)
            fwd_by = "the reference's CPU integrator" if kind == "reference" else "oracle port"
            line["cpu_baseline"] = {"value": v, "unit": UNIT, "cores": procs, "kind": kind,
                                    "sample": f"{desc}; forward: {fwd_by}, adjoint: oracle port; "
                                              f"{wall:.1f} s per core"}
        print(json.dumps(line), flush=True)
    if W.get("exchange"):
        s.set_exchange(None, 1)
    s.close()
    if dist:
        dist.destroy_process_group()
    return 0


def build_workload(args, ws, rank):
    """The synthetic group of one rank, its teacher, probes and trained parameters."""
    import numpy as np

    from heliox_b200 import shard, synth

    if args.config == 2:
        ncell = args.ncell or NCELL
        seed0 = SEED0 + 100000 * rank
        g = synth.random_tree_batch(ncell, seed0=seed0)
        return {"group": g, "teacher": synth.perturb_conductances(g, 0.2, seed=seed0 + 7), "nstep": args.nstep,
                "keys": ("hh.gnabar", "hh.gkbar", "hh.gl", "pas.g"), "probes": g.soma_nodes(), "scaling": "weak",
                "workload": f"config2: {ncell} seeded random-tree cells per GPU (hh+pas, IClamp), "
                            f"{args.nstep} steps dt 0.025 ms, soma-MSE vs lognormal teacher, forward + exact adjoint",
                "parallelism": "cells sharded, {ws} GPU(s), no collective on the data path"}
    if args.config == 3:
        g = synth.giant_cell()
        probes = np.unique(np.linspace(0, g.nnode - 1, 64).astype(np.int32))
        T = 2000 if args.nstep == T_STEPS else args.nstep
        return {"group": g, "teacher": synth.perturb_conductances(g, 0.2, seed=SEED0 + 3), "nstep": T,
                "keys": ("hh.gnabar", "hh.gkbar", "hh.gl", "pas.g"), "probes": probes, "scaling": "weak",
                "workload": f"config3: one {g.nnode}-compartment random tree ({g.meta.get('levels')} branch levels), "
                            f"{T} steps, MSE at 64 probes vs lognormal teacher, gradients of every segment's "
                            "conductances; split across CTAs (cooperative launch)",
                "parallelism": "replicas: one cell per GPU ({ws} GPU(s))"}
    if args.config == 4:
        total = args.ncell or NCELL_NET
        T = 8000 if args.nstep == T_STEPS else args.nstep
        g = synth.network_config4_shard(total, rank, ws)
        teacher = g.copy()
        teacher.exp2syn.fields["weight"] = g.meta["teacher_weight"].copy()
        c0, c1 = synth.config4_cell_range(total, rank, ws)
        return {"group": g, "teacher": teacher, "nstep": T, "keys": ("Exp2Syn.weight", "hh.gnabar"),
                "probes": g.soma_nodes(), "gid_base": c0, "nsrc_cells": total, "exchange": ws > 1,
                "window": shard.window_of(g), "cells_max": -(-total // ws), "scaling": "strong",
                "workload": f"config4: event network of {total} cells (hh+pas random trees, IClamp) x 100 Exp2Syn "
                            f"from random cells + 1 NetStim (5 Hz, noise 1) each, {T} steps dt 0.025 ms, soma MSE vs "
                            "teacher (weights perturbed lognormally), weight and gnabar gradients",
                "parallelism": "one network sharded by cell over {ws} GPU(s); window spike all-gather over NCCL"}
    if args.config == 5:
        g = synth.worm_config5()
        teacher = g.copy()
        rng = np.random.default_rng(SEED0 + 5)
        teacher.halfgap.fields["g"] = teacher.halfgap.fields["g"] * np.exp(0.2 * rng.standard_normal(g.halfgap.n))
        teacher.graded.fields["w"] = teacher.graded.fields["w"] * np.exp(0.2 * rng.standard_normal(g.graded.n))
        T = 8000 if args.nstep == T_STEPS else args.nstep
        return {"group": g, "teacher": teacher, "nstep": T, "scaling": "weak",
                "keys": ("HalfGap.g", "neuron_to_neuron_syn_lr.w", "hh.gnabar"), "probes": g.soma_nodes(),
                "workload": f"config5: {g.ncell} cells, {g.halfgap.n // 2} HalfGap pairs, {g.graded.n} graded "
                            f"synapses, {T} steps, soma MSE vs teacher, gap and synapse gradients",
                "parallelism": "replicas only ({ws} GPU(s)): coupled every step"}
    if args.config == 6:
        ncell = args.ncell or NCELL
        seed0 = 51000 + 100000 * rank
        g = synth.lib_tree_batch(ncell, seed0=seed0, nmin=200, nmax=1000, channels=synth.LIB_BBP_CHANNELS)
        keys = ("NaTg.gNaTgbar", "Nap_Et2.gNap_Et2bar", "K_Pst.gK_Pstbar", "K_Tst.gK_Tstbar", "SKv3_1.gSKv3_1bar",
                "SK_E2.gSK_E2bar", "Im.gImbar", "Ca_HVA.gbar", "Ca_LVAst.gCa_LVAstbar", "CaDynamics_E2.gamma")
        return {"group": g, "teacher": synth.perturb_lib(g, 0.2, seed=seed0 + 7), "nstep": args.nstep, "keys": keys,
                "probes": g.soma_nodes(), "scaling": "weak",
                "workload": f"config6: {ncell} seeded random-tree library cells per GPU (user-mech channel set "
                            f"+ CaDynamics_E2 + pas, IClamp), {args.nstep} steps dt 0.025 ms, soma-MSE vs lognormal "
                            "teacher, forward + exact adjoint",
                "parallelism": "cells sharded, {ws} GPU(s), no collective on the data path"}
    raise ValueError(f"unknown config {args.config}")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--ncell", type=int, default=0, help="cells (config 4: of the whole network; 2/6: per GPU)")
    ap.add_argument("--nstep", type=int, default=T_STEPS)
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU-baseline leg")
    ap.add_argument("--config", type=int, default=4, choices=(2, 3, 4, 5, 6))
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
