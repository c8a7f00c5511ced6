"""Benchmark of the per-step MD hot path (BASELINE configs 1 and 4) -- prints ONE JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: the 135-atom ABX3 perovskite (3x3x3, a = 6.2 A, jitter N(0, 0.05 A),
seed = replica index), Maxwell-Boltzmann momenta at 500 K, NVT Nose-Hoover
chain (tchain 3, tloop 1, tdamp 25 fs, dt 0.25 fs), the MACE-architecture
potential (128 channels, l <= 1, correlation 3, 2 interactions, 8 Bessel,
r_max 6 A, 89 elements; random weights, seed 1; IEEE FP32), whole-step
CUDA-graph mode. One MD step = NHC half -> exact neighbour re-filter ->
model energy and forces -> NHC half. ``--replicas R`` runs R independent
135-atom replicas per GPU as one disjoint-union graph; the default 64 is
config 4's shard (64/128/256/512 replicas on 1/2/4/8 GPUs), so ``value`` is
config 4's whole-job atom-steps/s at every N. At N = 1 the line also carries
``config1`` (one 135-atom replica alone: its ms/step, roofline and the three
execution modes), ``config0_matris`` (the same system under MatRIS-10M,
whole_step, beside the CPU port of the reference's config-0 path) and
``sevennet_s01`` (the same system under the SevenNet-0-architecture NequIP
potential, beside the reference's published 7net-0 step on H100).

Under torchrun (N > 1) every rank integrates its own replicas (seeds
rank*R .. rank*R+R-1), no collective on the step path; the per-replica
(E_pot, T) are all-gathered over NCCL once per window (the thermo log),
inside each timed window.

``--impl reference``: the CPU restatement of the same path (oracle/md.py:
dense neighbour search, FP64 model with autograd forces, NHC) timed on the
host cores -- the reference's own CPU path cannot run here (mace-torch is
not installed), so its restatement stands in.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "ms/MD-step at 135 atoms (1 B200); atom-steps/s per box at 1/2/4/8 B200"
UNIT = "atom-steps/s"
TEMPERATURE = 500.0


def _args():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=2000)
    p.add_argument("--warmup", type=int, default=100)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--replicas", type=int, default=64,
                   help="135-atom replicas per GPU (config 4 shards 64 per GPU; 1 = config 1 alone)")
    p.add_argument("--no-matris", action="store_true", help="skip the config-0 MatRIS-10M leg")
    p.add_argument("--steps-per-launch", type=int, default=10)
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--no-ops", action="store_true", help="skip the config-2 op microbenchmark")
    p.add_argument("--op", choices=["wide_gemm", "hbm_ops", "bond_graph", "nequip", "matris"], default=None,
                   help="time one op alone (the profiling entry of profiles/): prints its own JSON line")
    p.add_argument("--rows", type=int, default=300_000, help="rows of --op wide_gemm")
    p.add_argument("--atoms", type=int, default=25_000, help="atoms of --op hbm_ops (config 2's box density)")
    p.add_argument("--reps", type=int, default=10, help="ABX3 supercell repeats of --op nequip (config 3: 10)")
    p.add_argument("--kernels", action="store_true",
                   help="--op matris: also list the step's kernels (CUPTI device times over one window)")
    return p.parse_args()


def _config(args, world):
    workload = ("config4: 64 x 135-atom CsSnI3 replicas per B200 as one disjoint-union graph, MACE-arch"
                if args.replicas == 64 else
                f"{args.replicas} x 135-atom CsSnI3 replica(s) per B200" + (" (config 1)" if args.replicas == 1 else ""))
    return {"workload": workload + " 128ch L1 corr3 2 layers, NVT-NHC whole_step; (E_pot, T) all-gathered over "
                                   "NCCL once per window inside the timed region",
            "atoms_per_replica": 135, "replicas_per_gpu": args.replicas, "replicas_total": args.replicas * world,
            "dt_fs": 0.25, "temperature_K": TEMPERATURE, "tchain": 3, "tdamp_fs": 25.0,
            "steps_per_launch": args.steps_per_launch, "parallelism": f"replicas x{world} (no step-path collective)",
            "l2": "flushed (256 MB write) before every timed window; windows timed by CUDA events"}


def _system(seed):
    from fastmd_b200.structures import perovskite

    return perovskite(seed=seed)


def _reference(args):
    """The CPU oracle path, rank 0 only, all host threads."""
    import torch

    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.mace import MACEConfig, init_weights
    from fastmd_b200 import units
    from oracle.md import OracleMD

    if int(os.environ.get("RANK", "0")) != 0:
        return None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = MACEConfig()
    weights = init_weights(cfg, 1)
    pos, cell, numbers, masses = _system(0)
    md = OracleMD(weights, cfg, pos, cell, numbers, masses, maxwell_boltzmann_momenta(masses, TEMPERATURE, 0),
                  temperature_K=TEMPERATURE, timestep=0.25 * units.fs, tdamp=25 * units.fs)
    for _ in range(max(args.warmup // 50, 1)):
        md.step()
    steps = max(min(args.steps // 20, 60), 3)  # a bounded sample of the workload (~0.2 s per CPU step)
    t0 = time.perf_counter()
    for _ in range(steps):
        md.step()
    elapsed = time.perf_counter() - t0
    ms = 1e3 * elapsed / steps
    value = 135 * steps / elapsed
    return {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": steps, "warmup": max(args.warmup // 50, 1), "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": _config(argparse.Namespace(**{**vars(args), "replicas": 1}), 1),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{steps} MD steps of one 135-atom replica (oracle/md.py, FP64 torch on "
                                       f"{threads} threads)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


class _Clocks:
    """nvidia-smi samples of this GPU during the timed region."""

    def __init__(self, index: int):
        self.proc = None
        self.path = ROOT / "gpurun_out" / f"clocks_{index}.csv"
        try:
            self.path.parent.mkdir(exist_ok=True)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={index}", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                 "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                 "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                 "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "50"],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        self.proc.wait(timeout=10)
        self.out.close()
        sm, smax, reasons = [], [], set()
        names = ["active", "hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names[1:], parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def _peaks():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return float(data["hbm_gbs"]), float(data["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


def _ours(args):
    import torch
    import torch.distributed as dist

    from fastmd_b200 import _lib, units
    from fastmd_b200.mace import MACEModel
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.replicas import ThermoLog, replica_seeds

    R = args.replicas
    seeds = replica_seeds(rank, world, R)  # replica i: jitter and momentum seed i (config 4)
    systems = [_system(seed) for seed in seeds]
    cell, numbers, masses = systems[0][1], systems[0][2], systems[0][3]
    positions = np.concatenate([s[0] for s in systems])
    momenta = np.concatenate([maxwell_boltzmann_momenta(masses, TEMPERATURE, seed=seed) for seed in seeds])
    model = MACEModel(device=device, seed=1)
    S = math.gcd(args.steps, args.steps_per_launch) or 1
    md = GPUResidentMolecularDynamics(model, positions=positions, momenta=momenta, cell=cell, atomic_numbers=numbers,
                                      masses=masses, temperature_K=TEMPERATURE, timestep=0.25 * units.fs, tdamp=25 * units.fs,
                                      replicas=R, steps_per_launch=S, device=device)
    runner = md.runner
    # kernels of one window (counted on an eager window; the graph replays the same launches)
    snapshot = md.integrator.snapshot()
    _lib.count_launches(True)
    runner._window_body()
    counted = _lib.count_launches(False)
    md.integrator.load_snapshot(snapshot)
    launches_per_window = sum(n * (_lib.fused_step_kernels(model.config.num_interactions)
                                   if name == "fmd_mace_fused_step" else _lib.KERNELS_PER_CALL.get(name, 1))
                              for name, n in counted.items())
    log = ThermoLog(R, device)

    def thermo_log():  # the per-replica (E_pot, T) of every rank, once per window (NCCL over NVLink)
        if world > 1:
            log.gather(md.integrator.state.energy, md.integrator.temperature())

    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
    # the clock sampler runs from the first warm-up window to the end of the timed region; the warm-up
    # lasts at least the W steps asked for and at least ~1 s of work, so the record holds samples under load
    clocks = _Clocks(local)
    t_warm = time.perf_counter()
    warm_windows = 0
    while True:
        runner.launch()
        thermo_log()
        runner.settle()
        warm_windows += 1
        done = torch.tensor([float(warm_windows * S >= args.warmup and time.perf_counter() - t_warm >= 1.0)],
                            device=device)
        if world > 1:  # every rank leaves the warm-up together (the same collective steps on all ranks)
            dist.all_reduce(done, op=dist.ReduceOp.MIN)
        if float(done[0]) > 0:
            break
    windows = args.steps // S
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(windows)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(windows)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for w in range(windows):
        flush.zero_()
        starts[w].record()
        runner.launch()
        thermo_log()  # the window's only collective, timed with it
        ends[w].record()
        runner.settle()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    device_ms = sum(s.elapsed_time(e) for s, e in zip(starts, ends))
    total = torch.tensor([device_ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(total, op=dist.ReduceOp.MAX)
    device_ms = float(total[0])
    ms_per_step = device_ms / (windows * S)
    atoms = 135 * R * world
    value = atoms * 1e3 / ms_per_step

    # e2e: host state in, host state out, every window through the public API
    pin = lambda t: torch.empty(t.shape, dtype=t.dtype).pin_memory()  # noqa: E731
    integ = md.integrator
    host_q, host_p = pin(integ.state.q), pin(integ.state.p)
    host_q.copy_(integ.state.q)
    host_p.copy_(integ.state.p)
    out = {"positions": pin(integ.state.q), "momenta": pin(integ.state.p), "forces": pin(integ.state.f),
           "energy": pin(integ.state.energy)}
    e2e_windows = max(1, min(windows, 200))
    md.step_host(host_q, host_p, out)
    torch.cuda.synchronize()
    t1 = time.perf_counter()
    for _ in range(e2e_windows):
        md.step_host(out["positions"], out["momenta"], out)
        thermo_log()
    e2e_s = time.perf_counter() - t1
    e2e_ms_step = 1e3 * e2e_s / (e2e_windows * S)
    e2e_t = torch.tensor([e2e_ms_step], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_value = atoms * 1e3 / float(e2e_t[0])
    h2d = (host_q.numel() + host_p.numel()) * 8 / S
    d2h = sum(t.numel() * t.element_size() for t in out.values()) / S

    roofline = None
    if rank == 0:
        try:
            roofline = _roofline(md, device)
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            roofline = {"error": f"{type(error).__name__}: {error}"}
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = _cpu_baseline()
    modes = None
    if rank == 0 and world == 1 and R == 1 and not args.no_ops:
        try:
            modes = _execution_modes(md, model, systems[0], momenta, device)
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            modes = {"error": f"{type(error).__name__}: {error}"}
    config1 = None
    if rank == 0 and world == 1 and R != 1:
        try:
            config1 = _config1(args, model, device, flush, S)
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            config1 = {"error": f"{type(error).__name__}: {error}"}
    matris = None
    if rank == 0 and world == 1 and not args.no_matris:
        try:
            matris = _config0_matris(args, device, flush)
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            matris = {"error": f"{type(error).__name__}: {error}"}
    sevennet = None
    if rank == 0 and world == 1 and not args.no_matris:
        try:  # the reference's S01 system under the SevenNet-0-architecture potential (README.md:82)
            sevennet = _op_nequip(argparse.Namespace(reps=3, steps=1000, warmup=100))
            sevennet.update({"workload": "S01: the 135-atom CsSnI3 cell (config 1's system) under the "
                                         "SevenNet-0-architecture NequIP potential (seeded weights), NVT-NHC "
                                         "whole_step", "reference_published_h100_ms_per_step": 2.5952,
                             "reference_source": "README.md:82 (7net-0 on S01, H100, incl. trajectory output)"})
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            sevennet = {"error": f"{type(error).__name__}: {error}"}
    ops = None
    if rank == 0 and world == 1 and not args.no_ops:
        try:
            ops = _ops_c2(device)
        except Exception as error:  # noqa: BLE001 - the line still reports the measured step
            ops = {"error": f"{type(error).__name__}: {error}"}
    thermo_now = md.thermodynamics() if rank == 0 else None
    if world > 1:
        dist.barrier()
        del runner
        md.runner.graph = None
        dist.destroy_process_group()
    if rank != 0:
        return None
    return {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": windows * S,
            "warmup": warm_windows * S, "ms_per_step": ms_per_step, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32 (NHC state f64)", "data": "synthetic",
            "config": _config(args, world), "wall_s_timed": wall,
            "wall_ms_per_step": 1e3 * wall / (windows * S),
            "timing": "value: CUDA-event time of each window (launch + the NCCL thermo-log all-gather), max over "
                      "ranks; wall_ms_per_step: host clock over the same windows incl. the per-window settle",
            "e2e": {"value": e2e_value, "unit": UNIT, "ms_per_step": float(e2e_t[0]), "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "path": "GPUResidentMolecularDynamics.step_host: pinned host "
                    "positions+momenta in, positions/momenta/forces/energy out, per window of "
                    f"{S} steps"},
            "gpu_launches": launches_per_window * windows, "launches_per_step": launches_per_window / S,
            "roofline": roofline, "cpu_baseline": cpu, "clocks": clk, "ops_config2": ops,
            "execution_modes": modes, "config1": config1, "config0_matris": matris, "sevennet_s01": sevennet,
            "fallbacks": md.runner.fallbacks, "candidate_refreshes": md.runner.refreshes,
            "final_temperature_K": float(thermo_now["temperature"][0]),
            "final_conserved_eV": float(thermo_now["conserved_energy"][0])}


def _timed_windows(runner, windows, flush, device):
    """CUDA-event ms per window, each window after an L2 flush (the same protocol as the headline)."""
    import torch

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(windows)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(windows)]
    torch.cuda.synchronize(device)
    for w in range(windows):
        flush.zero_()
        starts[w].record()
        runner.launch()
        ends[w].record()
        runner.settle()
    torch.cuda.synchronize(device)
    return sum(a.elapsed_time(b) for a, b in zip(starts, ends))


def _config1(args, model, device, flush, S):
    """Config 1 alone: ms per MD step of ONE 135-atom replica (whole_step, same model), timed like the
    headline over the same number of steps, with the roofline of its dominant fused stage and the three
    execution modes."""
    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    pos, cell, numbers, masses = _system(0)
    momenta = maxwell_boltzmann_momenta(masses, TEMPERATURE, seed=0)
    md = GPUResidentMolecularDynamics(model, positions=pos, momenta=momenta, cell=cell, atomic_numbers=numbers,
                                      masses=masses, temperature_K=TEMPERATURE, timestep=0.25 * units.fs,
                                      tdamp=25 * units.fs, replicas=1, steps_per_launch=S, device=device)
    for _ in range(max(3, -(-args.warmup // S))):
        md.runner.launch()
        md.runner.settle()
    windows = max(args.steps // S, 1)
    ms = _timed_windows(md.runner, windows, flush, device) / (windows * S)
    out = {"workload": "config1: one 135-atom replica, MACE-arch, NVT-NHC whole_step", "ms_per_step": ms,
           "atom_steps_per_s": 135e3 / ms, "steps": windows * S}
    try:
        out["roofline"] = _roofline(md, device)
    except Exception as error:  # noqa: BLE001
        out["roofline"] = {"error": f"{type(error).__name__}: {error}"}
    if not args.no_ops:
        try:
            out["execution_modes"] = _execution_modes(md, model, (pos, cell, numbers, masses), momenta, device)
        except Exception as error:  # noqa: BLE001
            out["execution_modes"] = {"error": f"{type(error).__name__}: {error}"}
    return out


def _config0_matris(args, device, flush):
    """Config 0 on the GPU: the 135-atom system under MatRIS-10M (seeded weights), NVT-NHC whole_step,
    ms per MD step over up to 100 timed steps; beside it the CPU port of the reference's config-0 path
    (oracle/md.py MatRISOracleMD: dense neighbour search, FP64 MatRIS with autograd forces, the NHC) on all
    host threads, a bounded sample of 3 steps."""
    import torch

    from fastmd_b200 import units
    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.matris import MatRISModel
    from fastmd_b200.matris_params import MATRIS_10M, seeded_parameters
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    pos, cell, numbers, masses = _system(0)
    momenta = maxwell_boltzmann_momenta(masses, TEMPERATURE, seed=0)
    model = MatRISModel(MATRIS_10M, seed=0, device=device)
    S = 10
    md = GPUResidentMolecularDynamics(model, positions=pos, momenta=momenta, cell=cell, atomic_numbers=numbers,
                                      masses=masses, temperature_K=TEMPERATURE, timestep=0.25 * units.fs,
                                      tdamp=25 * units.fs, replicas=1, steps_per_launch=S, device=device)
    for _ in range(3):
        md.runner.launch()
        md.runner.settle()
    windows = max(1, min(args.steps, 100) // S)
    ms = _timed_windows(md.runner, windows, flush, device) / (windows * S)
    kernels = None
    if getattr(args, "kernels", False):  # one window under CUPTI: per kernel name, launches and device time
        from torch.profiler import ProfilerActivity, profile

        torch.cuda.synchronize(device)
        with profile(activities=[ProfilerActivity.CUDA]) as prof:
            md.runner.launch()
            torch.cuda.synchronize(device)
        md.runner.settle()
        rows = sorted(((e.device_time_total, e.count, e.key) for e in prof.key_averages()
                       if e.device_time_total > 0), reverse=True)
        total = sum(r[0] for r in rows)
        kernels = {"window_steps": S, "kernel_us_per_step": total / S, "launches_per_step": sum(r[1] for r in rows) / S,
                   "top": [{"kernel": k[:90], "us_per_step": round(t / S, 1), "launches_per_step": c / S,
                            "share": round(t / total, 4)} for t, c, k in rows[:20]]}
    out = {"workload": "config0 on the GPU: 135-atom CsSnI3, MatRIS-10M (10 layers, 128 wide, energy head "
                       "256/256, seeded weights), NVT-NHC whole_step, 3xTF32 tcgen05 GEMMs",
           "ms_per_step": ms, "atom_steps_per_s": 135e3 / ms, "steps": windows * S,
           "reference_published_h100_ms_per_step": 28.018, "kernels": kernels}
    if not args.no_cpu_baseline:
        from oracle.md import MatRISOracleMD

        threads = os.cpu_count() or 1
        torch.set_num_threads(threads)
        ref = MatRISOracleMD(seeded_parameters(MATRIS_10M, 0), MATRIS_10M, pos, cell, numbers, masses, momenta,
                             temperature_K=TEMPERATURE, timestep=0.25 * units.fs, tdamp=25 * units.fs)
        t0 = time.perf_counter()
        steps = 3
        for _ in range(steps):
            ref.step()
        cpu_ms = 1e3 * (time.perf_counter() - t0) / steps
        out["cpu_baseline"] = {"ms_per_step": cpu_ms, "cores": threads, "kind": "port",
                               "sample": f"{steps} MD steps of the 135-atom system (MatRISOracleMD: FP64 MatRIS-10M "
                                         f"forces by autograd, the reference's equations) on {threads} threads"}
        out["speedup_vs_cpu_port"] = cpu_ms / ms
    return out


def _execution_modes(md_ws, model, system, momenta, device, steps=200, warmup=20):
    """ms per MD step of config 1 in the reference's three execution modes (gpu_md.py:104) through the
    same driver: whole_step (the headline, from the timed windows above: here again over ``steps``),
    model_graph (a ragged build per step, the model replayed from its bucket's graph) and eager.
    Host wall clock over ``steps`` steps after ``warmup`` (the two per-step modes synchronise on the
    host every step, for the ragged build's edge count)."""
    import torch

    from fastmd_b200 import units
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    pos, cell, numbers, masses = system
    out = {}
    for execution in ("whole_step", "model_graph", "eager"):
        md = md_ws if execution == "whole_step" else GPUResidentMolecularDynamics(
            model, positions=pos, momenta=momenta, cell=cell, atomic_numbers=numbers, masses=masses,
            temperature_K=TEMPERATURE, timestep=0.25 * units.fs, tdamp=25 * units.fs, execution=execution,
            device=device)
        n = steps - steps % md_ws.runner.steps_per_launch if execution == "whole_step" else steps
        w = warmup - warmup % md_ws.runner.steps_per_launch if execution == "whole_step" else warmup
        md.run(max(w, md_ws.runner.steps_per_launch if execution == "whole_step" else 1))
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        md.run(n)
        torch.cuda.synchronize()
        out[execution] = round(1e3 * (time.perf_counter() - t0) / n, 4)
    out["unit"] = "ms/MD-step (host wall clock, 135 atoms)"
    return out


STAGES = {0: ("edge_fwd_kernel", 1), 1: ("message_fused_kernel (per layer)", 2), 2: ("node_fwd_kernel", 1),
          3: ("node_last_kernel", 1), 4: ("msg_bwd_edge_kernel (per layer)", 2), 5: ("sender_node_kernel", 1),
          6: ("edge_bwd_kernel", 1), 7: ("forces_kernel", 1)}


def _time_stage(md, device, bit, per_graph=20, replays=10):
    """GPU time of one launch group of fused stage ``bit``: ``per_graph`` launches captured in a CUDA
    graph (no host launch cost between them), replayed ``replays`` times between CUDA events."""
    import torch

    model, batch = md.model, md.builder.batch
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for _ in range(3):
            model.energy_forces_fused(batch, n_systems=md.replicas, stages=1 << bit)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for _ in range(per_graph):
            model.energy_forces_fused(batch, n_systems=md.replicas, stages=1 << bit)
    with torch.cuda.stream(s):
        graph.replay()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(s)
        for _ in range(replays):
            graph.replay()
        end.record(s)
    torch.cuda.synchronize(device)
    del graph
    return start.elapsed_time(end) / (replays * per_graph) * 1e3  # us per launch group


def _roofline(md, device):
    """Every fused stage timed alone (CUDA events around replays of a CUDA graph of 20 launches of the
    stage, after the timed run); the roofline of the dominant single-kernel stage against the measured
    HBM copy bandwidth (algorithmic bytes: the stage's compulsory reads and writes)."""
    hbm, _, kind = _peaks()
    names = dict(STAGES)
    E_rows = int(md.builder.batch.edge_index.shape[0])
    c = md.model.config
    layers = c.num_interactions
    if 0 < md.model.radial_tc_min_edges <= E_rows:
        # a large union: the radial MLPs run as chained tcgen05 GEMMs (several kernels per stage)
        names[0] = ("radial MLP forward (edge_geom_tc + 6 tcgen05 3xTF32 GEMMs)", 7)
        names[6] = ("radial MLP backward (6 tcgen05 3xTF32 GEMMs + edge_geom_bwd_tc)", 7)
        if layers == 2:  # and the node kernels' channel mixings as grouped tcgen05 GEMMs
            names[2] = ("node_fwd on the tensor cores (3 grouped tcgen05 GEMMs + the contraction kernel)", 4)
            names[3] = ("node_last on the tensor cores (6 grouped tcgen05 GEMMs + 4 CUDA-core kernels)", 10)
            names[5] = ("sender side on the tensor cores (3 grouped tcgen05 GEMMs + 3 CUDA-core kernels)", 6)
    stages = {names[bit][0]: round(_time_stage(md, device, bit), 3) for bit in names}
    # the single-kernel launches: a stage of one kernel, or of one kernel per layer (per-launch average)
    per_launch = {bit: stages[names[bit][0]] / (layers if names[bit][1] == 2 else 1)
                  for bit in names if names[bit][1] in (1, 2)}
    bit = max(per_launch, key=per_launch.get)
    us = per_launch[bit]
    N = md.builder.n_real
    E = int(md.builder.batch.n_edges.item())
    pc = sum(c.paths(L) * c.channels for L in range(c.num_interactions))
    weights = 4 * sum(c.num_bessel * 64 + 2 * 64 * 64 + 64 * c.paths(L) * c.channels
                      for L in range(c.num_interactions))
    # per-stage algorithmic bytes / flops (one launch over the step's real edges)
    algo = {0: (E * (8 + 12 + 16 + 4 * pc) + N * 12 + weights,
                2.0 * E * sum(c.num_bessel * 64 + 2 * 64 * 64 + 64 * c.paths(L) * c.channels
                              for L in range(c.num_interactions))),
            6: (E * (16 + 12 + 12 + 4 * pc) + weights,
                2.0 * E * sum(2 * (c.num_bessel * 64 + 2 * 64 * 64) + 64 * c.paths(L) * c.channels
                              for L in range(c.num_interactions)))}
    # the per-layer edge kernels (average per launch over the layers): message_fused reads the R row (P_L C
    # floats), 16 B of harmonics and the sender index per edge and the sender rows and writes the A rows once
    # per atom; msg_bwd_edge reads half the R row and writes the dR row per edge, plus dY, and reads the dA
    # and sender rows once per atom
    C = c.channels
    P = [c.paths(L) for L in range(layers)]
    sender = [4 * (C + (3 * C if P[L] == 4 else 0)) for L in range(layers)]
    algo[1] = (sum(E * (4 * P[L] * C + 20) + N * (sender[L] + 16 * C + 8) for L in range(layers)) / layers,
               sum(2.0 * E * C * (2 + 6 * (P[L] == 4)) for L in range(layers)) / layers)
    algo[4] = (sum(E * (2 * P[L] * C + 4 * P[L] * C + 20 + 12 * (1 + (L != layers - 1))) + N * (16 * C + sender[L])
                   for L in range(layers)) / layers,
               sum(2.0 * E * C * (4 + 8 * (P[L] == 4)) for L in range(layers)) / layers)
    # the node-side stages (2-layer model: node_fwd at layer 0, node_last and sender_node at layer 1); rows of
    # C floats per atom read or written once, R rows of P_L C floats and 16 B of harmonics per edge, the
    # C x C mixings once from HBM (per-element skip and product weights included)
    Lz = c.num_interactions - 1
    mix = 4 * C * C
    per_elem = 4 * c.num_elements * (2 * C * C + 9 * C)
    if c.num_interactions == 2:
        algo[2] = (N * 4 * 16 * C + 6 * mix + 4 * c.num_elements * 9 * C,
                   2.0 * N * 4 * C * C * 4)
        algo[3] = (N * (4 * 10 * C + 8) + 7 * mix + 4 * c.readout_hidden * C + per_elem,
                   2.0 * N * C * C * (4 + 1 + 1 + 1 + 1 + 4) + 4.0 * N * c.readout_hidden * C)
        algo[5] = (E * (4 * c.paths(Lz) * C + 16 + 4 + 4) + N * 4 * (4 * C + 4 * C + 4 * C + C) + 6 * mix
                   + 4 * c.num_elements * 9 * C,
                   2.0 * N * C * C * 4 * 3 + 2.0 * E * C * 12)
    bytes_, flops = algo.get(bit, (None, None))
    traffic = None
    tpath = ROOT / "profiles" / "traffic.json"
    if tpath.exists():
        # DRAM bytes per launch from one ncu capture of the same stage; entries keyed by kernel and edge
        # count scale with the edges processed (the per-edge rows dominate)
        entry = json.loads(tpath.read_text()).get(names[bit][0])
        if isinstance(entry, dict) and entry.get("edges"):
            traffic = entry["dram_bytes"] * E / entry["edges"]
        elif isinstance(entry, (int, float)):
            traffic = entry
    out = {"kernel": names[bit][0], "bound": "hbm", "unit": "GB/s", "peak": hbm,
           "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else "fallback 6650 GB/s",
           "avg_launch_us": us, "stages_us": stages, "traffic": traffic, "edges": E, "atoms": N,
           "note": ("135 atoms / 2,054 edges: every stage is latency-bound" if N <= 135 else
                    "the dominant launch of a single kernel (per-layer stages: the average launch); the multi-kernel "
                    "stages (radial chains, the node sequences of grouped tcgen05 GEMMs) are timed in stages_us")}
    if bytes_ is not None:
        achieved = bytes_ / (us * 1e-6) / 1e9
        out.update({"achieved": achieved, "frac": achieved / hbm, "algorithmic_bytes_per_launch": bytes_,
                    "flops_per_launch": flops, "achieved_tflops_fp32": flops / (us * 1e-6) / 1e12})
    return out


def _ops_c2(device):
    """BASELINE config 2, the op microbenchmark: 100,000 atoms uniform at 0.06 / A^3 (seed 2), rc 6 A,
    node features N(0,1) of width 128; each stage timed alone with CUDA events (inputs larger than
    L2; median of 5 after 2 warm-ups) against the measured HBM bandwidth (or the FP32 rate of the
    IEEE GEMM)."""
    import ctypes

    import torch

    from fastmd_b200 import _lib
    from fastmd_b200._lib import call, ptr
    from fastmd_b200.graph import _host_cell, estimate_max_neighbors
    from fastmd_b200.mace import _gemm
    from fastmd_b200.structures import random_box

    hbm, bf16, kind = _peaks()
    # the tensor pipe's own kind::tf32 rate, measured here (fmd_tf32_mma_rate: back-to-back MMAs, no data
    # movement); 3xTF32 makes three TF32 products per FP32 product
    tf32_peak, tf32_kind = _tf32_rate(device), "measured this run (fmd_tf32_mma_rate, tcgen05 issue rate)"
    s = torch.cuda.current_stream(device)
    sp = s.cuda_stream

    def timed(fn, reps=5):
        for _ in range(2):
            fn()
        times = []
        for _ in range(reps):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(s)
            fn()
            b.record(s)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        return statistics.median(times)

    n = 100_000
    pos_np, cell_np, _ = random_box(n, density=0.06, seed=2)
    pos = torch.from_numpy(pos_np).float().to(device)
    cell_host, cell_ptr = _host_cell(torch.from_numpy(cell_np).float())
    bmax = estimate_max_neighbors(6.0, atomic_density=0.06, safety_factor=2.0)
    e_cap = n * 64
    nbytes = ctypes.c_size_t(0)
    call("fmd_neighbor_list_workspace_bytes", cell_ptr, 6.0, n, bmax, ctypes.byref(nbytes))
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=device)
    center = torch.empty(e_cap, dtype=torch.int64, device=device)
    neighbor = torch.empty(e_cap, dtype=torch.int64, device=device)
    images = torch.empty(e_cap, 3, dtype=torch.int32, device=device)
    dist = torch.empty(e_cap, dtype=torch.float32, device=device)
    offsets = torch.empty(n + 1, dtype=torch.int64, device=device)
    wrapped = torch.empty(n, 3, dtype=torch.float32, device=device)
    flags = torch.zeros(1, dtype=torch.int32, device=device)

    def nlist():
        call("fmd_neighbor_list", ptr(pos), cell_ptr, n, 6.0, bmax, e_cap, ptr(wrapped), ptr(center), ptr(neighbor),
             ptr(images), ptr(dist), ptr(offsets), ptr(ws), ws.numel(), ptr(flags), sp)

    t_nl = timed(nlist)
    E = int(offsets[n].item())
    if int(flags.item()) or E > e_cap:
        return {"error": f"neighbour list flags {int(flags.item())}, {E} edges"}
    D = 128
    g = torch.Generator(device=device).manual_seed(2)
    X = torch.randn(n, D, device=device, generator=g)
    rbf = torch.randn(E, 8, device=device, generator=g)
    cat = torch.empty(E, 2 * D + 8, device=device)
    parts = (_lib.FmdCatPart * 3)()
    for k, (src, idx, width, rows) in enumerate(((X, neighbor, D, n), (X, center, D, n), (rbf, None, 8, E))):
        parts[k].src, parts[k].index, parts[k].ld, parts[k].n_src, parts[k].width = ptr(src), ptr(idx), width, rows, width

    def gather():
        call("fmd_gather_cat", parts, 3, E, ptr(cat), 2 * D + 8, ptr(flags), sp)

    t_gc = timed(gather)
    W0 = torch.randn(256, 2 * D + 8, device=device, generator=g) / 16.0
    W1 = torch.randn(256, 256, device=device, generator=g) / 16.0
    h = torch.empty(E, 256, device=device)
    y = torch.empty(E, 256, device=device)

    def mlp():
        _gemm(cat, W0, h, act=1, s=sp)
        _gemm(h, W1, y, s=sp)

    t_mlp = timed(mlp, reps=3)
    from fastmd_b200 import wide_gemm

    def mlp_tc():
        wide_gemm.linear_into(h, cat, W0, b0, act=1)
        wide_gemm.linear_into(y, h, W1, b1)

    b0 = torch.zeros(256, device=device)
    b1 = torch.zeros(256, device=device)
    wide_gemm._split(W0, False), wide_gemm._split(W1, False)  # once per weight version, outside the timing
    t_tc = timed(mlp_tc, reps=5)
    t_l1 = timed(lambda: wide_gemm.linear_into(h, cat, W0, b0, act=1), reps=5)
    seg = torch.empty(n, 256, device=device)

    def segsum():
        call("fmd_csr_segment_sum", ptr(y), 256, None, 0, None, ptr(offsets), n, 256, -1, ptr(seg), 256, sp)

    t_ss = timed(segsum)
    # segment attention (MatRIS receiver softmax-weighted sum) on the same receiver CSR, width 128
    from fastmd_b200.segment_attention import segment_attention

    logits = torch.randn(E, D, device=device, generator=g)
    vals = torch.randn(E, D, device=device, generator=g)
    t_sa = timed(lambda: segment_attention(logits, vals, center, n, off=offsets, identity_perm=True))
    b_sa = 2 * E * D * 4 + (n + 1) * 8 + n * D * 4
    b_nl = E * (8 + 8 + 12 + 4) + n * (12 + 16)
    b_gc = E * (2 * D + 8) * 4 + 2 * E * 8 + E * 8 * 4 + n * D * 4
    b_ss = E * 256 * 4 + (n + 1) * 8 + n * 256 * 4
    f_mlp = 2.0 * E * ((2 * D + 8) * 256 + 256 * 256)

    def hb(bytes_, ms):
        gbs = bytes_ / (ms * 1e-3) / 1e9
        return {"ms": round(ms, 4), "algorithmic_bytes": bytes_, "achieved_GBs": round(gbs, 1),
                "frac_of_hbm": round(gbs / hbm, 3)}

    return {"workload": "config2: 100,000 atoms, 0.06/A^3, rc 6 A, seed 2", "edges": E,
            "edges_per_atom": round(E / n, 2), "hbm_peak_GBs": hbm, "peak_source": kind,
            "neighbor_list": hb(b_nl, t_nl), "gather_cat_264": hb(b_gc, t_gc),
            "edge_mlp_264_256_256_ieee_fp32": {"ms": round(t_mlp, 3), "flops": f_mlp,
                                               "achieved_TFLOPs": round(f_mlp / (t_mlp * 1e-3) / 1e12, 2)},
            "edge_mlp_264_256_256_tf32x3_tcgen05": _tc_line(f_mlp, t_tc, E, tf32_peak, tf32_kind),
            "edge_linear_264_256_silu_tf32x3_tcgen05": _tc_line(2.0 * E * 264 * 256, t_l1, E, tf32_peak, tf32_kind),
            "segment_sum_256": hb(b_ss, t_ss), "segment_attention_128": hb(b_sa, t_sa)}


def _tf32_rate(device, iters=20000):
    """TF/s of back-to-back tcgen05 kind::tf32 MMAs (M = N = 128, K = 8) on every SM."""
    import torch

    from fastmd_b200._lib import call, ptr

    flags = torch.zeros(1, dtype=torch.int32, device=device)
    s = torch.cuda.current_stream(device)
    call("fmd_tf32_mma_rate", 1000, ptr(flags), s.cuda_stream)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(s)
    call("fmd_tf32_mma_rate", iters, ptr(flags), s.cuda_stream)
    end.record(s)
    torch.cuda.synchronize(device)
    sms = torch.cuda.get_device_properties(device).multi_processor_count
    return sms * iters * 2.0 * 128 * 128 * 8 / (start.elapsed_time(end) * 1e-3) / 1e12


def _tc_line(flops, ms, rows, tf32_peak, kind):
    """A 3xTF32 GEMM line: FP32-equivalent TFLOP/s, the TF32 tensor rate it implies (3 products per FP32
    product) and its fraction of the TF32 dense peak."""
    fp32_tflops = flops / (ms * 1e-3) / 1e12
    return {"ms": round(ms, 3), "rows": rows, "flops": flops, "achieved_TFLOPs_fp32_equivalent": round(fp32_tflops, 2),
            "tf32_tensor_TFLOPs": round(3 * fp32_tflops, 1), "tf32_peak_TFLOPs": round(tf32_peak, 1),
            "frac_of_tf32_peak": round(3 * fp32_tflops / tf32_peak, 3), "peak_source": kind}


def _cpu_baseline():
    """The oracle MD on the host cores, a bounded sample (~10-20 s)."""
    import torch

    from fastmd_b200.gpu_nhc import maxwell_boltzmann_momenta
    from fastmd_b200.mace import MACEConfig, init_weights
    from fastmd_b200 import units
    from oracle.md import OracleMD

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    cfg = MACEConfig()
    pos, cell, numbers, masses = _system(0)
    md = OracleMD(init_weights(cfg, 1), cfg, pos, cell, numbers, masses,
                  maxwell_boltzmann_momenta(masses, TEMPERATURE, 0), temperature_K=TEMPERATURE,
                  timestep=0.25 * units.fs, tdamp=25 * units.fs)
    md.step()
    steps, t0 = 0, time.perf_counter()
    while steps < 3 or (time.perf_counter() - t0 < 10.0 and steps < 200):
        md.step()
        steps += 1
    elapsed = time.perf_counter() - t0
    return {"value": 135 * steps / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
            "ms_per_step": 1e3 * elapsed / steps,
            "sample": f"{steps} MD steps of one 135-atom replica (oracle/md.py: dense neighbour search, FP64 "
                      f"MACE-arch forces with autograd, NHC) on {threads} threads"}


def _op_hbm(args):
    """``--op hbm_ops``: config 2's HBM-bound ops on a box of ``--atoms`` atoms at its density (rc 6 A):
    gather-cat (neighbour 128 | centre 128 | basis 8), the CSR segment sum of [E x 256], the segment
    attention of [E x 128] and the residual add of [E x 128] (12 bytes per element: its GB/s is
    reported), 3 warm-up calls then 5 timed (CUDA events each)."""
    import torch

    from fastmd_b200.graph import neighbor_list
    from fastmd_b200.ops import csr_segment_sum, gather_cat, segment_csr
    from fastmd_b200.residual_add import residual_add
    from fastmd_b200.segment_attention import segment_attention
    from fastmd_b200.structures import random_box

    dev = torch.device("cuda", 0)
    n = args.atoms
    pos_np, cell_np, _ = random_box(n, density=0.06, seed=2)
    center, neighbor, _, _ = neighbor_list(torch.from_numpy(pos_np).float().to(dev), torch.from_numpy(cell_np).float(),
                                           6.0)
    E = int(center.shape[0])
    g = torch.Generator(device=dev).manual_seed(0)
    h = torch.randn(n, 128, device=dev, generator=g)
    rbf = torch.randn(E, 8, device=dev, generator=g)
    v = torch.randn(E, 256, device=dev, generator=g)
    logits = torch.randn(E, 128, device=dev, generator=g)
    val = torch.randn(E, 128, device=dev, generator=g)
    res_w = torch.randn(128, device=dev, generator=g)
    perm, off = segment_csr(center, n)
    ops = {"gather_cat_264": lambda: gather_cat([(h, neighbor), (h, center), (rbf, None)]),
           "segment_sum_256": lambda: csr_segment_sum(v, center, n, perm, off),
           "segment_attention_128": lambda: segment_attention(logits, val, center, n, perm, off),
           "residual_add_128": lambda: residual_add(logits, val, res_w)}
    out = {"op": "hbm_ops", "atoms": n, "edges": E}
    for name, fn in ops.items():
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(5):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
        out[name + "_ms"] = round(statistics.median(times), 4)
    out["residual_add_128_gbs"] = round(12 * E * 128 / out["residual_add_128_ms"] / 1e6, 1)
    return out


def _op_bond_graph(args):
    """``--op bond_graph``: the per-step fixed-capacity MatRIS build (re-filter of reused candidates, then
    the bond graph: pairs and triplets at rc 6 / 4.5 A, sink padding) of ``--replicas`` 135-atom systems
    (config 0's perovskite), against the edges-only re-filter of the same positions. Each build is
    captured in a CUDA graph (as a whole step runs it); 3 warm-up replays, then 20 timed (CUDA events
    around each replay)."""
    import numpy as np
    import torch

    from fastmd_b200.graph import FixedCapacityGraphBuilder, PaddingRule
    from fastmd_b200.structures import perovskite

    dev = torch.device("cuda", 0)
    R = max(args.replicas, 1)
    pos = np.concatenate([perovskite(seed=s)[0] for s in range(R)]).astype(np.float32)
    cell = torch.tensor(perovskite(seed=0)[1], dtype=torch.float32)
    numbers = torch.tensor(perovskite(seed=0)[2])
    common = dict(cell=cell, atomic_numbers=numbers, u_capacity=1100 * R, atom_graph_cutoff=6.0, candidate_cutoff=8.0,
                  device=dev, replicas=R)
    builders = {"refilter": FixedCapacityGraphBuilder(**common),
                "refilter_bond_graph": FixedCapacityGraphBuilder(**common, line_graph_cutoff=4.5, t_capacity=19_000 * R,
                                                                 padding=PaddingRule("sink_atoms"), n_dummy=64)}
    x = torch.from_numpy(pos).to(dev)
    out = {"op": "bond_graph", "replicas": R, "atoms": int(pos.shape[0])}
    for name, b in builders.items():
        b.refresh_candidates(x)
        b.build(x, rebuild_candidates=False)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            b.build(x, rebuild_candidates=False)
        for _ in range(3):
            graph.replay()
        torch.cuda.synchronize()
        times = []
        for _ in range(20):
            a, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            graph.replay()
            e.record()
            torch.cuda.synchronize()
            times.append(a.elapsed_time(e))
        graph.reset()
        out[name + "_us"] = round(1e3 * statistics.median(times), 1)
        if name == "refilter_bond_graph":
            out["edges"] = int(b.batch.n_edges.item())
            out["triplets"] = int(b.n_triplets.item())
            out["flags"] = int(b.flags.item())
    out["bond_graph_us"] = round(out["refilter_bond_graph_us"] - out["refilter_us"], 1)
    return out


def _op_nequip(args):
    """``--op nequip``: BASELINE config 3, a 10x10x10 ABX3 supercell (5,000 atoms, jitter seed 3; ``--reps``
    sets the repeats) under the
    NequIP-architecture (SevenNet-0-style) potential (5 interaction blocks, 128x0e + 64x1e + 32x2e, rc
    5 A, random weights, the linears on the 3xTF32 tensor-core GEMM), NVT-NHC at 500 K with dt 0.25 fs,
    in the whole_step mode (windows of 10 steps as one CUDA graph; eager if the capture is refused);
    ``--steps`` timed steps after ``--warmup`` (CUDA events around the timed windows)."""
    import torch

    from fastmd_b200 import units
    from fastmd_b200.nequip import NequIPConfig, NequIPModel
    from fastmd_b200.structures import perovskite
    from fastmd_b200.whole_step import GPUResidentMolecularDynamics

    dev = torch.device("cuda", 0)
    pos, cell, numbers, masses = perovskite(reps=args.reps, seed=3)
    model = NequIPModel(NequIPConfig(), device=dev)
    steps = max(10, args.steps // 10 * 10)
    out = {"op": "nequip", "atoms": int(pos.shape[0]), "layers": 5}
    for execution in ("whole_step", "eager"):
        try:
            md = GPUResidentMolecularDynamics(model, positions=pos, cell=cell, atomic_numbers=numbers, masses=masses,
                                              temperature_K=TEMPERATURE, timestep=0.25 * units.fs,
                                              tdamp=25 * units.fs, steps_per_launch=10, execution=execution,
                                              device=dev)
        except Exception as error:  # a capture the driver refuses: report it and time the eager mode
            out[f"{execution}_error"] = f"{type(error).__name__}: {str(error)[:200]}"
            continue
        md.run(max(10, args.warmup // 10 * 10))
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        md.run(steps)
        b.record()
        torch.cuda.synchronize()
        ms = a.elapsed_time(b) / steps
        out.update({"execution": execution, "steps": steps, "ms_per_step": round(ms, 4),
                    "atom_steps_per_s": round(pos.shape[0] / ms * 1e3, 1),
                    "edges": int(md.builder.batch.n_edges.item()) if execution == "whole_step" else None,
                    "temperature_K": round(float(md.integrator.temperature()), 1)})
        break
    return out


def _op(args):
    """One op alone on cuda:0, the profiling entry: ``--op wide_gemm`` runs the config-2 first edge
    layer (264 -> 256, bias, SiLU, 3xTF32 on tcgen05) over ``--rows`` rows, 3 warm-up launches then
    10 timed ones (CUDA events; the input is larger than L2 from 120,000 rows on); ``--op hbm_ops``
    the HBM-bound ops (``_op_hbm``)."""
    if args.op == "hbm_ops":
        return _op_hbm(args)
    if args.op == "bond_graph":
        return _op_bond_graph(args)
    if args.op == "nequip":
        return _op_nequip(args)
    if args.op == "matris":  # config 0 on the GPU: MatRIS-10M whole_step (``--steps`` up to 100 timed)
        import torch

        device = torch.device("cuda", 0)
        flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=device)
        return {"op": "matris_whole_step", **_config0_matris(args, device, flush)}
    import torch

    from fastmd_b200 import wide_gemm

    dev = torch.device("cuda", 0)
    m, n, k = args.rows, 256, 264
    g = torch.Generator(device=dev).manual_seed(5)
    x = torch.randn(m, k, device=dev, generator=g)
    w = torch.randn(n, k, device=dev, generator=g) / 16
    b = torch.randn(n, device=dev, generator=g)
    y = torch.empty(m, n, device=dev)
    wide_gemm._split(w, False)
    for _ in range(3):
        wide_gemm.linear_into(y, x, w, b, act=1)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(10):
        wide_gemm.linear_into(y, x, w, b, act=1)
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / 10
    flops = 2.0 * m * n * k
    return {"op": "wide_gemm_tf32x3", "rows": m, "k": k, "n": n, "ms": round(ms, 4),
            "tflops_fp32_equivalent": round(flops / ms / 1e9, 1), "tf32_tensor_tflops": round(3 * flops / ms / 1e9, 1)}


def main():
    args = _args()
    if args.op is not None:
        print(json.dumps(_op(args)), flush=True)
        return
    result = _reference(args) if args.impl == "reference" else _ours(args)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
