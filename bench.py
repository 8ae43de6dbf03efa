"""Benchmark of the B200 neighbor-list provider (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload cfg5]
    python bench.py --impl reference ...     # reference CPU arm

Workload (default cfg5, tonari_b200/workloads.py): 8192 triclinic structures,
50-5000 atoms, mixed pbc, float32, cutoff 5, half list, 'PS'.

Scaling is strong by default: with N ranks the one cfg5 batch is split into N
contiguous shards balanced by estimated pair count (tonari_b200.sharding);
each rank searches its shard with globally numbered indices and keeps its
pairs; there is no collective on the data path.  value = the batch's pairs /
max-over-ranks time.  At N>1 the weak-scaling figure (N seeded copies of the
batch, one per rank) is measured as well and reported under "weak".

A step is one neighbor_list call over the rank's shard.
* value: inputs already in HBM, device time per step from CUDA events on the
  launching stream; L2 is flushed (256 MiB write) between steps, outside the
  events.
* e2e: the same call from pinned host inputs: H2D of positions/cell/pbc/
  batch_ptr, the call, and D2H of every output into pinned host memory.
* roofline: algorithmic bytes (inputs read once + requested outputs written
  once) over the device time of the dominant phase (the library's phase
  events, which bracket exactly that phase's kernel launches), against
  MEASURED_PEAKS.json hbm_gbs; the write pass and the whole call are reported
  beside it.
* cpu_baseline: the reference CPU core (oracle/_ref, else the C port) on the
  whole workload, one thread per physical core, rank 0 at N=1 only.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

FALLBACK_HBM_GBS = 6650.0


def parse_args():
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", default="cfg5")
    parser.add_argument("--size", type=int, default=None,
                        help="reduced size for profiling: atoms (cfg4) or structures (cfg2/3/5)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-e2e", action="store_true")
    parser.add_argument("--scaling", choices=["strong", "weak"], default="strong")
    parser.add_argument("--reference-cuda", default="cfg5,cfg4",
                        help="configs on which the reference's own CUDA provider (baseline/_ref) "
                             "is timed as a GPU comparator at N=1; empty to skip")
    parser.add_argument("--extra", default="cfg4,cfg2,cfg3",
                        help="comma list of extra configs measured at N=1 on rank 0")
    return parser.parse_args()


def peak_hbm():
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


SEEDS = {"cfg1": 0, "cfg2": 2, "cfg3": 3, "cfg4": 4, "cfg5": 5}


SIZE_KEYWORD = {"cfg2": "n_structures", "cfg3": "n_structures", "cfg4": "n_atoms",
                "cfg5": "n_structures"}


def make_workload(name: str, rank: int, world: int = 1, size: int | None = None,
                  scaling: str = "strong"):
    """The rank's share of the job.  N=1: the configuration itself.  N>1,
    strong: the configuration's batch split into N contiguous shards balanced
    by estimated pair count (tonari_b200.sharding); weak: the global batch is
    N seeded copies of the configuration (seeds s, s+1, ...), split the same
    way.  A single structure is never split: it is replicated."""
    from tonari_b200 import sharding, workloads

    extra = {SIZE_KEYWORD[name]: size} if size else {}
    if world == 1:
        return workloads.CONFIGS[name](seed=SEEDS[name], **extra)
    copies = world if scaling == "weak" else 1
    parts = [workloads.CONFIGS[name](seed=SEEDS[name] + k, **extra) for k in range(copies)]
    whole = parts[0] if copies == 1 else workloads.concatenate(parts, f"{name}x{world}")
    if whole.n_structures == 1:
        return whole
    weights = sharding.estimate_pairs(whole.batch_ptr, whole.cell, whole.pbc, whole.cutoff,
                                      half_list=whole.options.get("half_list", False))
    shard = sharding.partition(whole.batch_ptr, weights, world)[rank]
    part = whole.shard(shard.structure_begin, shard.structure_end)
    part.name = f"{whole.name}[rank {rank} of {world}]"
    return part


def physical_cores() -> int:
    """Physical cores of this host (unique core/socket pairs from lscpu)."""
    try:
        text = subprocess.run(["lscpu", "-p=CORE,SOCKET"], capture_output=True, text=True,
                              check=True).stdout
        cores = {line for line in text.splitlines() if line and not line.startswith("#")}
        if cores:
            return len(cores)
    except (OSError, subprocess.CalledProcessError):
        pass
    return os.cpu_count() or 1


def call_kwargs(w):
    return {
        "algorithm": w.options.get("algorithm", "auto"),
        "sorted": w.options.get("sorted", False),
        "half_list": w.options.get("half_list", False),
    }


class Clocks:
    """nvidia-smi sampler running during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.process = None

    def __enter__(self):
        try:
            self.process = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=self.file, stderr=subprocess.DEVNULL)
        except OSError:
            self.process = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.process is not None:
            self.process.terminate()
            self.process.wait()

    def summary(self):
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[5 + k] == "Active"})
        loaded = [v for v in sm if v > 0.5 * max(sm)] if sm else []
        return {"sm_mhz": statistics.median(loaded) if loaded else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": reasons, "samples": len(rows)}


def core_library():
    from tonari_b200._extensions import CORE_LIBRARY

    lib = ctypes.CDLL(str(CORE_LIBRARY))
    lib.tnr_last_launch_count.restype = ctypes.c_int64
    lib.tnr_last_phase_times.restype = ctypes.c_int
    lib.tnr_last_phase_times.argtypes = [ctypes.POINTER(ctypes.c_float), ctypes.c_int]
    lib.tnr_last_host_times.restype = ctypes.c_int
    lib.tnr_last_host_times.argtypes = [ctypes.POINTER(ctypes.c_double), ctypes.c_int]
    return lib


PHASES = ("prepare", "bin", "count", "scan", "readback", "write")


def phase_times(lib):
    buffer = (ctypes.c_float * 6)()
    lib.tnr_last_phase_times(buffer, 6)
    return list(buffer)


def host_times(lib):
    buffer = (ctypes.c_double * 12)()
    lib.tnr_last_host_times(buffer, 12)
    return list(buffer)


def measure_device(w, steps, warmup, device):
    """Device-resident inputs; per-step CUDA events; L2 flushed between steps."""
    import torch

    from tonari_b200 import neighbor_list

    lib = core_library()
    positions, cell, pbc, batch_ptr = w.torch_inputs(device)
    kwargs = call_kwargs(w)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        out = neighbor_list(w.quantities, positions, cell, pbc, w.cutoff, batch_ptr, **kwargs)
        del out
    torch.cuda.synchronize(device)
    # Timed steps run without the library's phase timers (their events and
    # final synchronisation would add host time to every call); the phase and
    # host breakdown comes from a second loop of the same steps.
    step_ms, phases, hosts, launches, n_pairs = [], [], [], [], 0
    for _ in range(steps):
        flush.zero_()
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        out = neighbor_list(w.quantities, positions, cell, pbc, w.cutoff, batch_ptr, **kwargs)
        end.record(stream)
        end.synchronize()
        step_ms.append(start.elapsed_time(end))
        launches.append(int(lib.tnr_last_launch_count()))
        n_pairs = int(out[0].shape[0])
        del out
    os.environ["TONARI_B200_PHASE_TIMERS"] = "1"
    try:
        for _ in range(steps):
            flush.zero_()
            out = neighbor_list(w.quantities, positions, cell, pbc, w.cutoff, batch_ptr, **kwargs)
            torch.cuda.synchronize(device)
            phases.append(phase_times(lib))
            hosts.append(host_times(lib))
            del out
    finally:
        os.environ.pop("TONARI_B200_PHASE_TIMERS", None)
    median_phase = [statistics.median(p[k] for p in phases) for k in range(6)]
    median_host = [statistics.median(h[k] for h in hosts) for k in range(12)]
    return {"step_ms": step_ms, "phase_ms": median_phase, "host_ms": median_host,
            "launches": launches, "n_pairs": n_pairs}


def measure_e2e(w, steps, warmup, device):
    """Pinned host inputs -> H2D -> call -> D2H of every output, per step."""
    import torch

    from tonari_b200 import neighbor_list

    kwargs = call_kwargs(w)
    host = [torch.from_numpy(a).pin_memory() for a in (w.positions, w.cell, w.pbc, w.batch_ptr)]
    stream = torch.cuda.current_stream(device)
    sinks = None
    times, h2d, d2h = [], sum(t.numel() * t.element_size() for t in host), 0
    for step in range(warmup + steps):
        start = torch.cuda.Event(enable_timing=True)
        end = torch.cuda.Event(enable_timing=True)
        start.record(stream)
        positions, cell, pbc, batch_ptr = (t.to(device, non_blocking=True) for t in host)
        out = neighbor_list(w.quantities, positions, cell, pbc, w.cutoff, batch_ptr, **kwargs)
        if sinks is None or any(s.shape != o.shape for s, o in zip(sinks, out)):
            sinks = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in out]
        for s, o in zip(sinks, out):
            s.copy_(o, non_blocking=True)
        end.record(stream)
        end.synchronize()
        if step >= warmup:
            times.append(start.elapsed_time(end))
        d2h = sum(o.numel() * o.element_size() for o in out)
        del out
    return {"step_ms": times, "h2d": h2d, "d2h": d2h}


def cpu_reference_rate(w, threads=None):
    """Reference CPU core (oracle/_ref; the C port when it was not built) on
    the whole workload, one thread per physical core.  Returns a dict."""
    from oracle import oracle

    threads = threads or physical_cores()
    kind = "reference" if oracle.ref_available() else "port"
    start = time.perf_counter()
    if kind == "reference":
        pairs, _ = oracle.ref_neighbor_list(
            w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr,
            half_list=w.options.get("half_list", False),
            algorithm=w.options.get("algorithm", "auto"), threads=threads)
    else:
        pairs, _ = oracle.port_neighbor_list(
            w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr,
            half_list=w.options.get("half_list", False))
        threads = 1
    seconds = time.perf_counter() - start
    return {"value": len(pairs) / seconds, "unit": "pairs/s", "cores": threads, "kind": kind,
            "sample": f"{w.name}: all {w.n_structures} structures, {w.n_atoms} atoms, "
                      f"{len(pairs)} pairs in {seconds:.2f} s ({threads} threads = physical "
                      f"cores from lscpu)",
            "structures_per_s": w.n_structures / seconds}


# DRAM bytes (read + write) of the dominant kernel per emitted pair, keyed by
# (workload, phase), from one ncu capture of that kernel on a reduced case of
# the same workload; `traffic` scales it by the call's pairs.  Sources:
#   cfg4 write pass: profiles/cell_emit_cfg4_200k.md (40.7 MB + 738.5 MB for
#     18,104,094 pairs at 200,000 atoms);
#   cfg5 write pass: profiles/cell_emit_cfg5_1024.md (99.8 MB + 567.4 MB for
#     22,354,478 half pairs at 1,024 structures);
#   cfg5 count pass: profiles/cell_count_cfg5_1024.md (80.7 MB + 10.0 MB for
#     the same 22,354,478 half pairs).
TRAFFIC_PER_PAIR = {("cfg4", "write"): (40.664832e6 + 738.508032e6) / 18_104_094,
                    ("cfg5", "write"): (99.836160e6 + 567.427328e6) / 22_354_478,
                    ("cfg5", "count"): (80.659712e6 + 10.031104e6) / 22_354_478}


def roofline(w, n_pairs, phase_ms, step_ms):
    from tonari_b200.workloads import algorithmic_bytes

    peak, source = peak_hbm()
    algorithmic = algorithmic_bytes(w, n_pairs)
    kernel_phases = [k for k in range(6) if PHASES[k] != "readback"]
    dominant = max(kernel_phases, key=lambda k: phase_ms[k])
    achieved = algorithmic / (phase_ms[dominant] * 1e-3) / 1e9
    write = algorithmic / (phase_ms[5] * 1e-3) / 1e9 if phase_ms[5] > 0 else None
    call = algorithmic / (step_ms * 1e-3) / 1e9
    per_pair = TRAFFIC_PER_PAIR.get((w.name.split("[")[0], PHASES[dominant]))
    return {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
            "frac": round(achieved / peak, 4), "peak_source": f"{source} hbm_gbs",
            "kernel": f"{PHASES[dominant]} phase", "kernel_ms": round(phase_ms[dominant], 4),
            "algorithmic_bytes": algorithmic,
            "traffic": int(per_pair * n_pairs) if per_pair else None,
            "phase_ms": {PHASES[k]: round(phase_ms[k], 4) for k in range(6)},
            "write_frac": round(write / peak, 4) if write else None,
            "call_achieved": round(call, 1), "call_frac": round(call / peak, 4)}


def reference_cuda_rate(name, steps, warmup, device):
    """The reference's stock CUDA path on this GPU, as a comparator: the
    unmodified reference package from baseline/_ref, its public
    tonari.neighbor_list on CUDA tensors (its own provider and frontend), with
    the same inputs, options and timing rules as `value`."""
    import torch

    site = ROOT / "baseline" / "_ref"
    if not (site / "tonari" / "api.py").exists():
        return {"unavailable": "the reference package is not installed in baseline/_ref"}
    sys.path.insert(0, str(site))
    try:
        import tonari
    finally:
        sys.path.remove(str(site))
    w = make_workload(name, 0)
    positions, cell, pbc, batch_ptr = w.torch_inputs(device)
    kwargs = call_kwargs(w)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    times, n_pairs = [], 0
    try:
        for step in range(warmup + steps):
            flush.zero_()
            start = torch.cuda.Event(enable_timing=True)
            end = torch.cuda.Event(enable_timing=True)
            start.record(stream)
            out = tonari.neighbor_list(w.quantities, positions, cell, pbc, w.cutoff, batch_ptr,
                                       **kwargs)
            end.record(stream)
            end.synchronize()
            if step >= warmup:
                times.append(start.elapsed_time(end))
            n_pairs = int(out[0].shape[0])
            del out
    except (RuntimeError, ValueError) as error:
        return {"unavailable": f"the reference CUDA provider failed: {str(error)[:200]}"}
    ms = statistics.mean(times)
    return {"pairs_per_s": n_pairs / (ms * 1e-3), "structures_per_s": w.n_structures / (ms * 1e-3),
            "ms_per_step": ms, "pairs": n_pairs, "steps": steps, "warmup": warmup,
            "path": "baseline/_ref tonari.neighbor_list on CUDA tensors (reference CUDA provider)"}


def run_reference(args):
    """Reference arm: the reference's CPU implementation on the whole
    workload, one thread per physical core; rank 0 only."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle

    w = make_workload(args.workload, 0, 1, args.size)
    rates, samples = [], None
    for step in range(args.warmup + args.steps):
        result = cpu_reference_rate(w)
        if step >= args.warmup:
            rates.append(result["value"])
            samples = result
    value = statistics.median(rates)
    line = {
        "impl": "reference", "metric": "pairs/s", "value": value, "unit": "pairs/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32" if w.positions.dtype == np.float32 else "f64", "data": "synthetic",
        "config": {"workload": w.name, "structures": w.n_structures, "atoms": w.n_atoms,
                   "cutoff": w.cutoff, "quantities": w.quantities, **call_kwargs(w)},
        "cpu_baseline": {"value": value, "unit": "pairs/s", "cores": samples["cores"],
                         "kind": samples["kind"], "sample": samples["sample"]},
        "e2e": {"value": value, "unit": "pairs/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "structures_per_s": samples["structures_per_s"],
        "reference_available": oracle.ref_available(),
        "same_config": True,
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse_args()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    from tonari_b200._extensions import load_torch_cuda

    load_torch_cuda()

    w = make_workload(args.workload, rank, world, args.size, args.scaling)
    replicas = world > 1 and w.n_structures == 1
    scaling = "weak" if (args.scaling == "weak" or replicas) else "strong"

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(device)

    def max_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(value: float) -> float:
        if world == 1:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    def gather(obj):
        if world == 1:
            return [obj]
        out = [None] * world
        dist.all_gather_object(out, obj)
        return out

    barrier()
    with Clocks(local_rank) as clocks:
        device_run = measure_device(w, args.steps, args.warmup, device)
        barrier()
    total_ms = max_over_ranks(sum(device_run["step_ms"]))
    ms_per_step = total_ms / args.steps
    pairs_all = sum_over_ranks(device_run["n_pairs"])
    structures_all = sum_over_ranks(w.n_structures)
    value = pairs_all / (ms_per_step * 1e-3)
    per_rank = gather({
        "rank": rank, "structures": w.n_structures, "atoms": w.n_atoms,
        "pairs": device_run["n_pairs"],
        "ms_per_step": round(statistics.mean(device_run["step_ms"]), 4),
        "phase_ms": {PHASES[k]: round(v, 4) for k, v in enumerate(device_run["phase_ms"])},
        "host_marks_ms": [round(v, 3) for v in device_run["host_ms"]],
    })

    weak = None
    if world > 1 and scaling == "strong":
        ww = make_workload(args.workload, rank, world, args.size, "weak")
        barrier()
        weak_run = measure_device(ww, args.steps, args.warmup, device)
        barrier()
        weak_ms = max_over_ranks(sum(weak_run["step_ms"])) / args.steps
        weak_pairs = sum_over_ranks(weak_run["n_pairs"])
        weak = {"value": weak_pairs / (weak_ms * 1e-3), "unit": "pairs/s",
                "ms_per_step": weak_ms, "pairs_per_step": int(weak_pairs),
                "workload": f"{args.workload} x{world} (seeded copies, one batch per rank)"}

    e2e = None
    if not args.no_e2e:
        barrier()
        e2e_run = measure_e2e(w, max(3, args.steps // 2), 2, device)
        barrier()
        e2e_ms = max_over_ranks(statistics.mean(e2e_run["step_ms"]))
        e2e = {"value": pairs_all / (e2e_ms * 1e-3), "unit": "pairs/s", "ms_per_step": e2e_ms,
               "h2d_bytes_per_step": int(sum_over_ranks(e2e_run["h2d"])),
               "d2h_bytes_per_step": int(sum_over_ranks(e2e_run["d2h"]))}

    if world == 1:
        workload_name = args.workload
        parallelism = "1 GPU"
    elif replicas:
        workload_name = f"{args.workload} (one structure, replicated on {world} GPUs)"
        parallelism = f"{world} replicas, no data-path collective"
    else:
        workload_name = (f"{args.workload} split into {world} shards" if scaling == "strong"
                         else f"{args.workload} x{world}")
        parallelism = f"{world} ranks, contiguous shards, no data-path collective"
    line = {
        "metric": "pairs/s", "value": value, "unit": "pairs/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
        "higher_is_better": True, "scaling": scaling, "vs_baseline": None,
        "dtype": "f32" if w.positions.dtype == np.float32 else "f64", "data": "synthetic",
        "config": {"workload": workload_name,
                   "structures_per_step": int(structures_all),
                   "atoms_per_step": int(sum_over_ranks(w.n_atoms)), "cutoff": w.cutoff,
                   "quantities": w.quantities, **call_kwargs(w),
                   "pairs_per_step": int(pairs_all),
                   "l2": "flushed between steps (256 MiB write)",
                   "parallelism": parallelism},
        "structures_per_s": structures_all / (ms_per_step * 1e-3),
        "gpu_launches": int(sum_over_ranks(sum(device_run["launches"]))),
        "roofline": roofline(w, device_run["n_pairs"], device_run["phase_ms"],
                             statistics.mean(device_run["step_ms"])),
        "clocks": clocks.summary(),
        "e2e": e2e,
        "ranks": per_rank,
    }
    if weak is not None:
        line["weak"] = weak
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_reference_rate(w)
    if rank == 0 and world == 1 and args.extra:
        extras = {}
        for name in filter(None, args.extra.split(",")):
            xw = make_workload(name, 0)
            run = measure_device(xw, max(3, args.steps // 2), 3, device)
            ms = statistics.mean(run["step_ms"])
            extras[name] = {"pairs_per_s": run["n_pairs"] / (ms * 1e-3),
                            "structures_per_s": xw.n_structures / (ms * 1e-3),
                            "ms_per_step": ms, "pairs": run["n_pairs"],
                            "host_marks_ms": [round(v, 3) for v in run["host_ms"]],
                            "roofline": roofline(xw, run["n_pairs"], run["phase_ms"], ms)}
        line["extra_configs"] = extras
    if rank == 0 and world == 1 and args.reference_cuda:
        # The reference's CUDA path takes about 15 s per cfg5 call on a B200:
        # one warm-up and one timed call there, three of each elsewhere.
        line["reference_cuda"] = {
            name: reference_cuda_rate(name, 1 if name == "cfg5" else 3, 1 if name == "cfg5" else 2,
                                      device)
            for name in filter(None, args.reference_cuda.split(","))}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
