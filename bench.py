#!/usr/bin/env python
"""Benchmark of the dependence-DAG hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl reference]

One step is one pass of the hot path over one batch of synthetic input.  The
default workload is the sync-free / wavefront SpTRSV configuration: a random
lower-triangular CSR matrix with n = 4,194,304 rows (about 15.6 entries per
row, half of them inside a band of 64), fp64, one right-hand side; the metric is
SpTRSV GFLOP/s with the reference's formula (n + 2 nnz) / t
(benchmark/sptrsv_benchmark.py:626 of the reference).  With N > 1 every rank holds
the matrix and solves its own right-hand side (multi-RHS sharding by column,
no data-path collective, weak scaling).

The same JSON line carries, under "configs", one record per other configuration of the
path: on one GPU the CSC demo on the 256 x 256 grid, ILU0 on the 128^3 grid with the two
solves on its factors, the supernodal solve with 1,048,576 rows and 64 right-hand sides on
the 192^3 grid; on N > 1 GPUs the 64 right-hand sides split by column over the ranks and
one solve on the 256^3 grid partitioned by block rows (both strong scaling).  Each record
holds its time, its fraction of the measured copy bandwidth, a parity figure against the
CPU restatement and (one GPU) that restatement's time on one host core.

Prints ONE JSON line (rank 0).  ``--impl reference`` times the CPU restatement of
the reference's sequential loop on the host cores instead.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "sptrsv_gflops_fp64"
UNIT = "GFLOP/s"
WORKLOADS = {
    # name: (kind, size)
    "sptrsv_random_n4194304": ("band", 4_194_304),
    "sptrsv_random_n1048576": ("band", 1_048_576),
    "sptrsv_lap2d_g256": ("lap2d", 256),
    "sptrsv_lap3d_g128": ("lap3d", 128),
    "sptrsv_lap3d_g256": ("lap3d", 256),
}
# side workloads (other configurations of the path); they print their own JSON line
SIDE_WORKLOADS = {
    "csc_lap2d_g256": ("csc", 256),
    "ilu0_lap3d_g128": ("ilu0", 128),
    "ilu0_lap3d_g64": ("ilu0", 64),
    "supernodal_n1048576": ("supernodal", 1_048_576),
    "supernodal_n131072": ("supernodal", 131_072),
    "multirhs_lap3d_g192": ("multirhs", 192),
    "multirhs_lap3d_g96": ("multirhs", 96),
    "partition_lap3d_g256": ("partition", 256),
    "partition_lap3d_g128": ("partition", 128),
    "literal_kernels_lap3d_g96": ("literal", 96),
    "literal_kernels_lap3d_g48": ("literal", 48),
}
DEFAULT_WORKLOAD = "sptrsv_random_n4194304"


def log(*args):
    print(*args, file=sys.stderr, flush=True)


# ------------------------------------------------------------------ inputs ----
def load_workload(name, rank=0, world=1, barrier=None):
    """Seeded synthetic matrix of the workload; generated once per box (rank 0) and
    shared through a cache file so that several ranks / both arms reuse it."""
    from lcd_b200 import generators as gen
    kind, size = WORKLOADS[name]
    cache = os.path.join(os.environ.get("LCD_B200_CACHE", "/tmp"), f"lcd_b200_{name}_seed0.npz")
    if rank == 0 and not os.path.exists(cache):
        t0 = time.time()
        if kind == "band":
            tri = gen.random_band_lower(size, seed=0)
        elif kind == "lap2d":
            tri = gen.laplacian2d_tril(size, seed=0)
        else:
            tri = gen.laplacian3d_tril(size, seed=0)
        Ap, Ai, Ax = tri.csr_arrays()
        tmp = cache + f".tmp{os.getpid()}.npz"
        np.savez(tmp, Ap=Ap, Ai=Ai, Ax=Ax, b=tri.b)
        os.replace(tmp, cache)
        log(f"[bench] generated {name} in {time.time() - t0:.1f}s")
    if barrier is not None:
        barrier()
    data = np.load(cache)
    Ap, Ai, Ax, b = data["Ap"], data["Ai"], data["Ax"], data["b"]
    if rank:
        b = np.random.default_rng([0, rank]).uniform(-1.0, 1.0, len(b))  # own RHS column
    return Ap, Ai, Ax, b


def algorithmic_bytes(n, nnz):
    """nnz (8 + 4) + (n + 1) 4 + n 8 (b) + n 8 (x): every matrix entry, pointer and
    vector element moved once; gathers of x, flags and DAG arrays are not counted."""
    return nnz * 12 + (n + 1) * 4 + n * 16


# DRAM traffic per row of the dominant kernel (dram__bytes_read.sum + dram__bytes_write.sum of one
# ncu capture at 1,048,576 rows divided by the rows; both kernels' traffic grows in proportion to
# the rows, so a launch on n rows is charged n times this; see profiles/)
TRAFFIC_BYTES_PER_ROW = {"csr_chain_kernel": 1.2314e9 / 1048576, "csr_syncfree_row_kernel": 227.3e6 / 1048576}


def flops(n, nnz):
    return n + 2 * nnz


# ------------------------------------------------------------------ clocks ----
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.rows = []
        self.proc = None
        self.gpu_index = gpu_index

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu_index)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append((time.perf_counter(), [c.strip() for c in line.split(",")]))

    def mark(self):
        """The timed region starts now: samples from here on are the ones reported."""
        self.marked = time.perf_counter()

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.15)
        self.proc.terminate()
        marked = getattr(self, "marked", 0.0)
        rows = [row for t, row in self.rows if t >= marked]
        note = None
        if not rows and self.rows:
            # the timed region was shorter than the sampling period: the last samples of the
            # warm-up steps (the same work, directly before) stand in
            rows = [row for _, row in self.rows[-3:]]
            note = "sampled during the warm-up steps directly before the timed region"
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for row in rows:
            try:
                sm.append(float(row[1]))
                smax.append(float(row[2]))
            except (ValueError, IndexError):
                continue
            for name, cell in zip(names, row[5:9]):
                if cell.lower().startswith("active"):
                    reasons.add(name)
        out = {"sm_mhz": float(np.median(sm)) if sm else None,
               "sm_max_mhz": max(smax) if smax else None, "samples": len(sm),
               "reasons": sorted(reasons)}
        if note:
            out["note"] = note
        return out


# ----------------------------------------------------------- reference arm ----
def run_reference(args):
    """The reference's CPU path for this operator is a sequential loop nest
    (compiler/demo/sptrsv.py:26-34); its compiled restatement (oracle/lcd_oracle.c)
    is timed on one host core.  A step is one full solve of the workload."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle as cpu
    cpu.build()
    Ap, Ai, Ax, b = load_workload(args.workload)
    n, nnz = len(Ap) - 1, len(Ai)
    for _ in range(max(1, min(args.warmup, 2))):
        cpu.sptrsv_csr_lower(Ap, Ai, Ax, b)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        x = cpu.sptrsv_csr_lower(Ap, Ai, Ax, b)
    elapsed = time.perf_counter() - t0
    per_step = elapsed / args.steps
    value = flops(n, nnz) / per_step / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": per_step * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": args.workload, "n": n, "nnz": nnz, "format": "csr_lower"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": 1, "kind": "port",
                         "sample": f"{args.steps} full solves of the workload",
                         "host_cores_available": os.cpu_count()},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "effective_gbs": algorithmic_bytes(n, nnz) / per_step / 1e9,
        "residual": cpu.relative_residual_csr(Ap, Ai, Ax, x, b),
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ our arm ----
def measured_peak_gbs():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as handle:
            return float(json.load(handle)["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return 6650.0, "fallback"


def bind_to_gpu_cpus(gpu_index):
    """Run this process on the CPUs next to its GPU (NVML's affinity mask), so that pinned host
    buffers are first touched on the memory node the PCIe link hangs off: host<->device copies
    of the end-to-end measurement otherwise lose up to half their bandwidth on two-socket
    hosts.  A process setting only; nothing of the GPU is changed."""
    try:
        import pynvml
        pynvml.nvmlInit()
        handle = pynvml.nvmlDeviceGetHandleByIndex(gpu_index)
        words = pynvml.nvmlDeviceGetCpuAffinity(handle, (os.cpu_count() + 63) // 64)
        cpus = {64 * w + b for w, word in enumerate(words) for b in range(64) if (word >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return len(cpus)
    except Exception as error:   # no NVML, no permission: measure where we are
        log("cpu affinity not set:", error)
        return None


def run_native(args):
    import torch
    import torch.distributed as dist
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    cpu_affinity = bind_to_gpu_cpus(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from lcd_b200 import _native as nat, ops
    nat.load()
    Ap, Ai, Ax, b = load_workload(args.workload, rank, world, barrier)
    n, nnz = len(Ap) - 1, len(Ai)
    up = lambda a: torch.from_numpy(a).to(dev)
    dAp, dAi, dAx, db = up(Ap), up(Ai), up(Ax), up(b)
    x = torch.empty(n, dtype=torch.float64, device=dev)
    status = ops.new_status(dev)
    lanes, threads = args.lanes, args.threads

    # the inspector's part (structure only, cached per matrix by the decorator): the level
    # count decides between the polling kernel and the block-recurrence chain solver
    from lcd_b200.scheduler import chain_solver_preferred
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dag = ops.dag_build("csr_lower", dAp, dAi)
    torch.cuda.synchronize()
    dag_build_ms = (time.perf_counter() - t0) * 1e3
    levels, dag_edges = dag.n_levels, dag.n_edges
    del dag
    # what the decorated call runs first: the build stops the level propagation as soon as a row
    # passes rows / 64 levels (enough to pick the chain solver); the level sets are completed
    # only if something asks for them
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    capped = ops.dag_build("csr_lower", dAp, dAi, level_cap=max(n // 64, 1))
    torch.cuda.synchronize()
    dag_build_capped_ms = (time.perf_counter() - t0) * 1e3
    level_cap_hit = bool(capped.capped)
    del capped
    solver = args.solver
    if solver == "auto":
        solver = "chain" if chain_solver_preferred(n, levels) else "row"
    if solver == "chain":
        workspace = ops.chain_workspace(n, dev)

        def step():
            # numeric preparation (block tiles from the values) and solve, both timed: the
            # preparation runs range by range on a second stream, the solve of a range follows
            # its own tiles (what the decorated call does when the values have changed)
            ops.chain_prepare_and_solve(dAp, dAi, dAx, db, workspace, x, status=status, sync=False)
        kernel_name = "csr_chain_kernel"
        launches_per_step = 2 * (len(ops.chain_pipeline_bounds(n)) - 1)
    else:
        def step():
            ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db, x, lanes=lanes, threads=threads,
                                    status=status, sync=False)
        kernel_name, launches_per_step = "csr_syncfree_row_kernel", 1

    # correctness before timing: status word and relative residual (fp64 tolerance 1e-12)
    step()
    code, node = ops.read_status(status)
    if code != 0:
        raise RuntimeError(f"solver reported {nat.error_string(code)} at row {node}")
    from oracle import oracle as cpu   # checker only (residual), never the measured path
    residual = cpu.relative_residual_csr(Ap, Ai, Ax, x.cpu().numpy(), b)
    if not residual <= 1e-12:
        raise RuntimeError(f"relative residual {residual:.3e} exceeds 1e-12")

    # (the sampler is started before the warm-up steps: nvidia-smi needs a few hundred
    # milliseconds before its first line, more than a short timed region lasts)
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    torch.cuda.synchronize()
    sampler.mark()
    events[0].record()
    for k in range(args.steps):
        step()
        events[k + 1].record()
    torch.cuda.synchronize()
    barrier()
    clocks = sampler.stop() if rank == 0 else None
    total_ms = events[0].elapsed_time(events[-1])
    per_launch_ms = [events[k].elapsed_time(events[k + 1]) for k in range(args.steps)]
    if ops.read_status(status)[0] != 0:
        raise RuntimeError("solver reported an error inside the timed region")
    if world > 1:
        t = torch.tensor([total_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t.item())
    ms_per_step = total_ms / args.steps
    value = world * flops(n, nnz) / (ms_per_step * 1e-3) / 1e9
    spread = {"p20": float(np.percentile(per_launch_ms, 20)), "p50": float(np.percentile(per_launch_ms, 50)),
              "p80": float(np.percentile(per_launch_ms, 80))}   # this rank's steps, CUDA events

    # end to end through the public API: the decorated operator called with host
    # (pinned) arrays; upload, solve and download are all inside the timed region
    e2e = None
    if not args.kernel_only:
        e2e = measure_e2e(args, Ap, Ai, Ax, b, n, nnz, world, dev, barrier)

    extras = {"dag_build_ms": dag_build_ms, "dag_build_capped_ms": dag_build_capped_ms,
              "level_cap_hit": level_cap_hit, "levels": levels, "dag_edges": dag_edges}
    if rank == 0 and solver == "chain":
        # the two kernels of a step apart (events around each)
        extras["prepare_ms"] = float(np.mean(_time_steps(
            lambda: ops.chain_prepare(dAp, dAi, dAx, workspace), 3, 1)))
        extras["solve_ms"] = float(np.mean(_time_steps(
            lambda: ops.sptrsv_csr_chain(dAp, dAi, dAx, db, workspace, x, status=status, sync=False), 3, 1)))
    if rank == 0 and not args.skip_extras and not args.kernel_only:
        extras.update(measure_extras(args, dAp, dAi, dAx, db, x, status, Ap, Ai, Ax, b, solver))
    cpu_baseline = None
    if rank == 0 and world == 1 and not args.kernel_only:
        cpu_baseline = measure_cpu_baseline(cpu, Ap, Ai, Ax, b, n, nnz)
    if rank == 0:
        peak, peak_kind = measured_peak_gbs()
        kernel_ms = float(np.mean(per_launch_ms))
        # the dominant kernel's own duration (a chain step also holds the preparation kernel)
        achieved = algorithmic_bytes(n, nnz) / (extras.get("solve_ms", kernel_ms) * 1e-3) / 1e9
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "ms_per_step_spread": spread,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
            "data": "synthetic",
            "config": {"workload": args.workload, "n": n, "nnz": nnz, "format": "csr_lower",
                       "mode": "sync_free", "solver": solver,
                       "step": ("lcd_chain_prepare_rows + lcd_sptrsv_csr_chain_rows, 16 row ranges, "
                                "preparation on a second stream" if solver == "chain"
                                else "lcd_sptrsv_csr_syncfree"),
                       "lanes_per_row": lanes or "auto",
                       "threads_per_block": threads or 1024, "rhs_per_gpu": 1,
                       "l2_policy": "inputs (%.2f GB) exceed the 126 MB L2" % (
                           algorithmic_bytes(n, nnz) / 1e9)},
            "e2e": e2e, "e2e_cold_ms": (e2e or {}).get("first_call_ms"),
            "gpu_launches": args.steps * launches_per_step,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "traffic": (TRAFFIC_BYTES_PER_ROW[kernel_name] * n
                                     if args.workload.startswith("sptrsv_random") else None),
                         "traffic_source": "ncu capture at n=1048576 scaled by rows",
                         "peak_kind": peak_kind,
                         "kernel": kernel_name,
                         "kernel_ms": extras.get("solve_ms", kernel_ms)},
            "cpu_baseline": cpu_baseline, "clocks": clocks, "cpus_near_gpu": cpu_affinity,
            "effective_gbs": world * achieved, "residual": residual,
        }
        line.update(extras)
    # the other configurations of the path (all ranks take part: the multi-GPU ones hold
    # collectives); their records travel in the same JSON line
    configs = None
    if not args.kernel_only and not args.skip_configs:
        del dAp, dAi, dAx, db, x
        torch.cuda.empty_cache()
        configs = other_configurations(args, rank, world)
    if rank == 0:
        line["configs"] = configs
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def measure_e2e(args, Ap, Ai, Ax, b, n, nnz, world, dev, barrier):
    import torch
    import torch.distributed as dist
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    from lcd_b200.decorator import parallel
    op = parallel(block_map="i", thread_map="j", execution_mode="sync_free", threads_per_block=128,
                  thread_unroll=1,
                  function_props={"Ap": ["monotonically_increasing"], "Ai": []})(_sptrsv_csr)
    pinned = [torch.from_numpy(a).pin_memory().numpy() for a in (Ap, Ai, Ax, b)]
    # The launcher keeps the chain solver's tiles while the value array is unchanged.  A caller
    # who solves with new values every time does not benefit, and that is the case timed here:
    # calls alternate between two value arrays that differ in one entry by one ulp.
    other = Ax.copy()
    other[-1] = np.nextafter(other[-1], np.inf)
    values = [pinned[2], torch.from_numpy(other).pin_memory().numpy()]
    torch.cuda.synchronize()
    t_cold = time.perf_counter()
    warm = [op(pinned[0], pinned[1], values[0], pinned[3], n)]    # first call: inspector + plan + solve
    cold_ms = (time.perf_counter() - t_cold) * 1e3
    warm.append(op(pinned[0], pinned[1], values[1], pinned[3], n))
    del warm                                    # (two page-locked result buffers exist afterwards)
    steps = max(2, min(args.steps, 5))
    torch.cuda.synchronize()
    barrier()
    t0 = time.perf_counter()
    marks = [t0]
    for k in range(steps):
        out = op(pinned[0], pinned[1], values[k % 2], pinned[3], n)
        marks.append(time.perf_counter())
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    if world > 1:
        t = torch.tensor([elapsed], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        elapsed = float(t.item())
    per_call = elapsed / steps
    h2d = sum(a.nbytes for a in pinned)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    copies = [torch.from_numpy(a).to(dev, non_blocking=True) for a in pinned]
    e1.record()
    torch.cuda.synchronize()
    h2d_ms = e0.elapsed_time(e1)
    del copies
    return {"value": world * flops(n, nnz) / per_call / 1e9, "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(out.nbytes),
            "ms_per_call": per_call * 1e3, "calls": steps, "first_call_ms": cold_ms,
            "h2d_copy_alone_ms": h2d_ms, "h2d_gb_per_s": h2d / h2d_ms / 1e6,
            "ms_each_call": [round((b - a) * 1e3, 2) for a, b in zip(marks, marks[1:])],
            "values_change_every_call": True,
            "api": "lcd_b200.decorator.parallel(...)(sptrsv_csr)(Ap, Ai, Ax, b, n)"}


def _sptrsv_csr(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


def measure_extras(args, dAp, dAi, dAx, db, x, status, Ap, Ai, Ax, b, solver):
    """The other execution modes on the same matrix (one run each): the level-synchronous
    kernel, and the polling sync-free kernel when the chain solver was the one timed."""
    import torch
    from lcd_b200 import ops
    out = {}
    dag = ops.dag_build("csr_lower", dAp, dAi)
    if solver == "chain":
        out["polling_kernel_ms"] = float(np.mean(_time_steps(
            lambda: ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db, x, lanes=args.lanes,
                                            threads=args.threads, status=status, sync=False), 2, 1)))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    ops.sptrsv_wavefront("csr_lower", dAp, dAi, dAx, db, dag.wavefronts, dag.wavefront_ptr, None,
                         x, mode="cooperative", lanes=16, status=status, sync=False)
    e1.record()
    torch.cuda.synchronize()
    out["wavefront_ms"] = e0.elapsed_time(e1)
    out["wavefront_status"] = ops.read_status(status)[0]
    return out


def measure_cpu_baseline(cpu, Ap, Ai, Ax, b, n, nnz):
    """The CPU restatement of the reference's loop on one host core: repeated full
    solves for about ten seconds (at least three)."""
    cpu.sptrsv_csr_lower(Ap, Ai, Ax, b)
    count, t0 = 0, time.perf_counter()
    while count < 3 or (time.perf_counter() - t0 < 10.0 and count < 200):
        cpu.sptrsv_csr_lower(Ap, Ai, Ax, b)
        count += 1
    per = (time.perf_counter() - t0) / count
    return {"value": flops(n, nnz) / per / 1e9, "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{count} full solves of the workload ({per * 1e3:.1f} ms each)",
            "host_cores_available": os.cpu_count()}


# ------------------------------------------------------------ side workloads ----
def _time_steps(step, steps, warmup):
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    events = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    events[0].record()
    for k in range(steps):
        step()
        events[k + 1].record()
    torch.cuda.synchronize()
    return [events[k].elapsed_time(events[k + 1]) for k in range(steps)]


def _host_time(fn, min_seconds=2.0, min_count=2):
    fn()
    count, t0 = 0, time.perf_counter()
    while count < min_count or time.perf_counter() - t0 < min_seconds:
        fn()
        count += 1
    return (time.perf_counter() - t0) / count, count


def _sptrsv_csc(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


def _roofline(nbytes, ms, peak, ranks=1):
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {"bound": "hbm", "achieved": achieved, "peak": peak * ranks, "unit": "GB/s",
            "frac": achieved / (peak * ranks)}


def _context():
    """(rank, local_rank, world, device) of this process; the process group is initialised by the
    caller."""
    import torch
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    return rank, local_rank, world, torch.device("cuda", local_rank)


def _max_over_ranks(value, world, dev):
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def numba_cuda_reference():
    """The reference's own Numba-CUDA path (wavefront variant of the sptrsv_csc demo) timed on
    this box by ``baseline/numba_wavefront.py`` in a child process: the unmodified reference from
    ``baseline/_ref`` (git-ignored; placed there by ``baseline/install_reference.py`` where the
    reference checkout exists).  Returns its JSON record, or the reason it could not run."""
    import tempfile
    script = os.path.join(ROOT, "baseline", "numba_wavefront.py")
    try:
        with tempfile.TemporaryDirectory() as scratch:      # the reference writes smt_file.smt2 into the cwd
            done = subprocess.run([sys.executable, script], cwd=scratch, capture_output=True, text=True,
                                  timeout=300)
        lines = [line for line in done.stdout.splitlines() if line.startswith("{")]
        if not lines:
            return {"unavailable": ("no result: " + (done.stderr.strip().splitlines() or ["?"])[-1])[:300]}
        return json.loads(lines[-1])
    except subprocess.TimeoutExpired:
        return {"unavailable": "the child process did not finish within 300 s"}
    except Exception as error:
        return {"unavailable": f"{type(error).__name__}: {error}"[:300]}


# ---- configuration 1: the sptrsv_csc demo on the 256 x 256 grid -------------------------
def config_csc_lap2d(args, size=256):
    """Lower triangle of the 2-D 5-point Laplacian, CSC, through the decorated operator
    (compiler/demo/sptrsv.py:35-43 of the reference) and through the C ABI."""
    import torch
    from scipy.sparse.linalg import spsolve_triangular
    import scipy.sparse as sp
    from lcd_b200 import generators as gen, ops
    from lcd_b200.decorator import parallel
    from oracle import oracle as cpu
    _, _, _, dev = _context()
    peak, _ = measured_peak_gbs()
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tri = gen.laplacian2d_tril(size, seed=0)
    Cp, Ci, Cx = tri.csc_arrays()
    n, nnz = tri.n, tri.nnz
    dCp, dCi, dCx, db = up(Cp), up(Ci), up(Cx), up(tri.b)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    dag = ops.dag_build("csc_lower", dCp, dCi)
    plan = ops.SmallPlan("csc_lower", dCp, dCi, dag)
    torch.cuda.synchronize()
    inspect_ms = (time.perf_counter() - t0) * 1e3
    x = torch.empty_like(db)
    ms = float(np.median(_time_steps(lambda: ops.sptrsv_small(plan, dCx, db, x), 50, 10)))
    got = x.cpu().numpy()
    want = cpu.sptrsv_csc_lower(Cp, Ci, Cx, tri.b)
    A = sp.csc_matrix((Cx, Ci, Cp), shape=(n, n))
    residual = float(np.linalg.norm(A @ got - tri.b) / np.linalg.norm(tri.b))
    t0 = time.perf_counter()
    xs = spsolve_triangular(sp.csr_matrix(A), tri.b, lower=True)
    scipy_ms = (time.perf_counter() - t0) * 1e3
    # end to end: the decorated operator with page-locked host arrays
    op = parallel(block_map="i", thread_map="j",
                  function_props={"Ap": ["monotonically_increasing"], "Ai": [],
                                  ("Ap", "Ai"): ["triangularity"]})(_sptrsv_csc)
    pinned = [torch.from_numpy(a).pin_memory().numpy() for a in (Cp, Ci, Cx, tri.b)]
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    out = op(pinned[0], pinned[1], pinned[2], pinned[3], n)
    cold_ms = (time.perf_counter() - t0) * 1e3
    for _ in range(3):
        out = op(pinned[0], pinned[1], pinned[2], pinned[3], n)
    calls = 30
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(calls):
        out = op(pinned[0], pinned[1], pinned[2], pinned[3], n)
    torch.cuda.synchronize()
    e2e_ms = (time.perf_counter() - t0) * 1e3 / calls
    e2e_residual = float(np.linalg.norm(A @ out - tri.b) / np.linalg.norm(tri.b))
    cpu_s, count = _host_time(lambda: cpu.sptrsv_csc_lower(Cp, Ci, Cx, tri.b), min_seconds=1.0)
    nbytes = algorithmic_bytes(n, nnz)
    if args.kernel_only:
        reference_gpu = {"unavailable": "skipped (--kernel-only)"}
    else:
        reference_gpu = numba_cuda_reference() if size == 256 else {
            "unavailable": "timed on the 256 x 256 grid only"}
    return {"workload": f"sptrsv_csc_lap2d_g{size}", "format": "csc_lower", "n": n, "nnz": nnz,
            "numba_cuda_wavefront_ms": reference_gpu.get("ms"), "numba_cuda_reference": reference_gpu,
            "levels": dag.n_levels, "kernel": "sptrsv_small_kernel (one thread block)",
            "ms": ms, "gflops": flops(n, nnz) / (ms * 1e-3) / 1e9,
            "inspector_ms": inspect_ms, "roofline": _roofline(nbytes, ms, peak),
            "latency_bound_note": f"{dag.n_levels} levels x one block barrier",
            "parity": {"relative_residual": residual,
                       "max_abs_diff_vs_oracle": float(np.max(np.abs(got - want))),
                       "max_abs_diff_vs_scipy": float(np.max(np.abs(got - xs))),
                       "tolerance": 1e-12, "ok": bool(residual <= 1e-12)},
            "e2e": {"ms_per_call": e2e_ms, "first_call_ms": cold_ms, "calls": calls,
                    "gflops": flops(n, nnz) / (e2e_ms * 1e-3) / 1e9,
                    "h2d_bytes_per_step": int(sum(a.nbytes for a in pinned)),
                    "d2h_bytes_per_step": int(out.nbytes), "relative_residual": e2e_residual,
                    "api": "lcd_b200.decorator.parallel(block_map='i', thread_map='j', "
                           "function_props=...)(sptrsv_csc)(Ap, Ai, Ax, b, n)",
                    "schedule": str(getattr(op.current_schedule, "execution_mode", None))},
            "cpu_baseline": {"value": flops(n, nnz) / cpu_s / 1e9, "unit": "GFLOP/s", "ms": cpu_s * 1e3,
                             "cores": 1, "kind": "port", "sample": f"{count} full solves",
                             "scipy_spsolve_triangular_ms": scipy_ms}}


# ---- configuration 3: ILU0 on the 3-D grid, then the two solves on the factors ----------
def config_ilu0(args, size=128):
    import torch
    from lcd_b200 import generators as gen, ops
    from oracle import oracle as cpu
    _, _, _, dev = _context()
    peak, _ = measured_peak_gbs()
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    mat, b = gen.laplacian3d_ilu0(size, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    n, nnz = len(Ap) - 1, len(Ai)
    dAp, dAi, dA0, db = up(Ap), up(Ai), up(Ax), up(b)
    work = dA0.clone()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    pos = ops.diag_positions(dAp, dAi)
    dag = ops.dag_build("ilu0_csr", dAp, dAi)
    back = ops.dag_build("csr_upper_rows", dAp, dAi)
    torch.cuda.synchronize()
    inspect_ms = (time.perf_counter() - t0) * 1e3
    done = torch.empty(n, dtype=torch.int32, device=dev)
    status = ops.new_status(dev)
    y, x = torch.empty_like(db), torch.empty_like(db)
    steps = max(3, min(args.steps, 10))
    copy_ms = float(np.median(_time_steps(lambda: work.copy_(dA0), steps, 2)))
    results = {}
    scratch = torch.empty_like(dA0)
    max_row = int((dAp[1:] - dAp[:-1]).max())
    for mode in ("sync_free", "ordered", "ordered_flags", "wavefront"):
        def step():
            work.copy_(dA0)
            ops.spilu0_csr(dAp, dAi, work, pos, mode=mode.split("_flags")[0], wavefronts=dag.wavefronts,
                           wavefront_ptr_host=dag.wavefront_ptr_host, done=done, status=status,
                           sync=False, max_row=max_row,
                           scratch=False if mode == "ordered_flags" else scratch)
        ms = _time_steps(step, steps, 2)
        results[mode] = float(np.median(ms)) - copy_ms   # the restore of A is not part of ILU0
        if ops.read_status(status)[0] != 0:
            raise RuntimeError(f"ILU0 ({mode}) reported an error")
    want = cpu.ilu0_csr(Ap, Ai, Ax, fast=True)
    identical = bool(np.array_equal(work.cpu().numpy(), want))
    forward = ops.OrderedPlan(dag.wavefronts, dag.n_levels)
    backward = ops.OrderedPlan(back.wavefronts, back.n_levels)
    fwd = _time_steps(lambda: ops.sptrsv_csr_ordered(dAp, dAi, work, db, forward, y, diag_pos=pos,
                                                     unit_diag=True, status=status, sync=False), steps, 2)
    bwd = _time_steps(lambda: ops.sptrsv_csr_ordered(dAp, dAi, work, y, backward, x, diag_pos=pos,
                                                     upper=True, status=status, sync=False), steps, 2)
    # the same two solves as level walks shared by many blocks (a preconditioner applied again
    # and again: the factors' coefficients are gathered into slot order once)
    walk_l = ops.SmallPlan("csr_lower", dAp, dAi, dag, diag_pos=pos, unit_diag=True, blocks=0)
    walk_u = ops.SmallPlan("csr_upper", dAp, dAi, back, diag_pos=pos, blocks=0)
    yw, xw = torch.empty_like(db), torch.empty_like(db)
    ops.sptrsv_small(walk_l, work, db, yw, sync=True)
    ops.sptrsv_small(walk_u, work, yw, xw, sync=True)
    fwd_walk = float(np.median(_time_steps(lambda: ops.sptrsv_small(walk_l, work, db, yw), steps, 2)))
    bwd_walk = float(np.median(_time_steps(lambda: ops.sptrsv_small(walk_u, work, yw, xw), steps, 2)))
    fwd_rep = float(np.median(_time_steps(
        lambda: ops.sptrsv_small(walk_l, work, db, yw, same_values=True), steps, 2)))
    bwd_rep = float(np.median(_time_steps(
        lambda: ops.sptrsv_small(walk_u, work, yw, xw, same_values=True), steps, 2)))
    hp = pos.cpu().numpy()
    x_ref = cpu.sptrsv_upper_of_full(Ap, Ai, want, hp, cpu.sptrsv_unit_lower_of_full(Ap, Ai, want, hp, b))
    walk_err = float(np.max(np.abs(xw.cpu().numpy() - x_ref)) / np.max(np.abs(x_ref)))
    err = float(np.max(np.abs(x.cpu().numpy() - x_ref)) / np.max(np.abs(x_ref)))
    cpu_s, count = _host_time(lambda: cpu.ilu0_csr(Ap, Ai, Ax, fast=True))
    solve_s, _ = _host_time(lambda: cpu.sptrsv_upper_of_full(
        Ap, Ai, want, hp, cpu.sptrsv_unit_lower_of_full(Ap, Ai, want, hp, b)), min_seconds=1.0)
    # the decorated call of the reference's demo loop (compiler/demo/spilu0.py:19-47) with host
    # arrays: upload, inspector plan from the cache, factorisation, download of the factor
    e2e = None
    if not args.kernel_only:
        from lcd_b200 import demos
        op = demos.compile_ilu0_csr("sync_free")
        pinned = [torch.from_numpy(a).pin_memory().numpy() for a in (Ax, Ai, Ap)]
        t0 = time.perf_counter()
        out = op(pinned[0].copy(), pinned[1], pinned[2])            # first call: inspector and plan
        cold_ms = (time.perf_counter() - t0) * 1e3
        calls = []
        for _ in range(3):
            data = torch.from_numpy(Ax.copy()).pin_memory().numpy()
            t0 = time.perf_counter()
            out = op(data, pinned[1], pinned[2])
            calls.append((time.perf_counter() - t0) * 1e3)
        e2e = {"ms_per_call": float(np.median(calls)), "first_call_ms": cold_ms, "calls": len(calls),
               "h2d_bytes_per_step": int(sum(a.nbytes for a in pinned)), "d2h_bytes_per_step": int(out.nbytes),
               "factor_bit_identical_to_sequential": bool(np.array_equal(out, want)),
               "api": "lcd_b200.decorator.parallel(...)(ilu0_csr)(A_data, A_indices, A_indptr)"}
    nbytes = 20 * nnz + 4 * (n + 1) + 4 * n
    best_mode = min(results, key=results.get)
    best = results[best_mode]
    tri_nnz = (nnz + n) // 2
    return {"workload": f"ilu0_lap3d_g{size}", "metric": "spilu0_ms_per_factorization", "n": n, "nnz": nnz,
            "numba_cuda_wavefront_ms": None,
            "numba_cuda_reference": {"unavailable": "not run: the reference's inspector is interpreted "
                                     "Python over sets of edges and needs minutes and gigabytes at "
                                     f"{n} rows before its first launch"},
            "levels": dag.n_levels, "ms": best, "mode": best_mode, "ms_by_mode": results,
            "gflops_2nnz": 2 * nnz / (best * 1e-3) / 1e9, "inspector_ms": inspect_ms,
            "roofline": _roofline(nbytes, best, peak), "e2e": e2e,
            "forward_solve_ms": float(np.median(fwd)), "backward_solve_ms": float(np.median(bwd)),
            "shared_walk": {"forward_ms": fwd_walk, "backward_ms": bwd_walk,
                            "forward_repeated_ms": fwd_rep, "backward_repeated_ms": bwd_rep,
                            "blocks": walk_l.blocks, "solve_max_rel_error": walk_err,
                            "note": "sptrsv_small_kernel, one block per node range; repeated = the "
                                    "factors' coefficients already in slot order"},
            "solve_kernel": "csr_ordered_kernel on the factors in place (unit lower / upper)",
            "solve_roofline": _roofline(2 * algorithmic_bytes(n, tri_nnz),
                                        float(np.median(fwd)) + float(np.median(bwd)), peak),
            "parity": {"factor_bit_identical_to_sequential": identical,
                       "solve_max_rel_error": err, "tolerance": 1e-10,
                       "ok": bool(identical and err <= 1e-10 and walk_err <= 1e-10)},
            "cpu_baseline": {"value": cpu_s * 1e3, "unit": "ms", "cores": 1, "kind": "port",
                             "sample": f"{count} full factorisations",
                             "forward_plus_backward_ms": solve_s * 1e3}}


# ---- configuration 4: supernodal solve ----------------------------------------------------
def config_supernodal(args, size=1_048_576):
    import torch
    from lcd_b200 import generators as gen, ops, supernodal
    from oracle import oracle as cpu
    _, _, _, dev = _context()
    peak, _ = measured_peak_gbs()
    t0 = time.time()
    s = gen.supernodal_random(size, seed=0)
    log(f"[bench] generated supernodal n={size} in {time.time() - t0:.1f}s "
        f"({s.Lx.nbytes / 1e9:.2f} GB of panels, {s.n_super} supernodes)")
    t0 = time.perf_counter()
    plan = supernodal.analyse(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.col_to_super, device=dev)
    torch.cuda.synchronize()
    analyse_ms = (time.perf_counter() - t0) * 1e3
    db = torch.from_numpy(np.ascontiguousarray(s.b)).to(dev)
    x = torch.empty_like(db)
    steps = max(3, min(args.steps, 10))
    ms = _time_steps(lambda: supernodal.solve(plan, db, x, sync=False), steps, 2)
    best = float(np.median(ms))
    code = ops.read_status(plan.status)[0]
    xs = x.cpu().numpy()
    cpu_s, count = _host_time(lambda: cpu.sptrsv_supernodal(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.b),
                              min_seconds=3.0, min_count=1)
    want = cpu.sptrsv_supernodal(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.b)
    err = float(np.max(np.abs(xs - want)) / np.max(np.abs(want)))
    conversion = None
    if size <= 131_072:
        # the layout built on the device from the same matrix stored by columns
        # (convert_csc_to_supernodal of the reference), then solved from the converted arrays
        L = s.to_csc()
        L.sort_indices()
        up = lambda a, t: torch.from_numpy(np.ascontiguousarray(a, dtype=t)).to(dev)
        dCp, dCi, dCx = up(L.indptr, np.int32), up(L.indices, np.int32), up(L.data, np.float64)
        supernodal.from_csc(dCp, dCi, dCx, device=dev)          # warm-up (allocations)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        layout = supernodal.from_csc(dCp, dCi, dCx, device=dev)
        torch.cuda.synchronize()
        convert_ms = (time.perf_counter() - t0) * 1e3
        plan2 = supernodal.analyse(layout.sn, layout.Lip, layout.Li, layout.Lp, layout.Lx,
                                   layout.col_to_super, device=dev)
        x2 = supernodal.solve(plan2, db).cpu().numpy()
        conversion = {"csc_nnz": int(L.nnz), "ms": convert_ms, "n_super": layout.n_super,
                      "max_width": layout.max_width, "panel_values": int(layout.Lx.numel()),
                      "solve_max_rel_error": float(np.max(np.abs(x2 - want)) / np.max(np.abs(want)))}
        del plan2, layout, dCp, dCi, dCx
    return {"workload": f"supernodal_n{size}", "n": size, "n_super": plan.n_super, "tasks": plan.n_tasks,
            "csc_to_supernodal": conversion,
            "panel_gb": plan.panel_values * 8 / 1e9, "ms": best,
            "gflops": plan.flops / (best * 1e-3) / 1e9, "analyse_and_upload_ms": analyse_ms,
            "status": code, "roofline": _roofline(plan.algorithmic_bytes, best, peak),
            "parity": {"max_rel_error_vs_sequential": err, "tolerance": 1e-10,
                       "ok": bool(code == 0 and err <= 1e-10)},
            "cpu_baseline": {"value": plan.flops / cpu_s / 1e9, "unit": "GFLOP/s", "ms": cpu_s * 1e3,
                             "cores": 1, "kind": "port", "sample": f"{count} full solves"}}


# ---- configuration 5a: 64 right-hand sides, sharded by column over the ranks ----------------
def config_multirhs(args, size=192, nrhs=64):
    """Strong scaling: the 64 columns are split over the ranks (matrix replicated, no data-path
    collective); the time is the slowest rank's, device-timed."""
    import torch
    from lcd_b200 import generators as gen
    from lcd_b200.multigpu import ShardedMultiRHS
    from oracle import oracle as cpu
    rank, _, world, dev = _context()
    peak, _ = measured_peak_gbs()
    tri = gen.laplacian3d_tril(size, seed=0)
    Ap, Ai, Ax = tri.csr_arrays()
    n, nnz = tri.n, tri.nnz
    solver = ShardedMultiRHS(Ap, Ai, Ax, device=dev)
    start, stop = solver.shard(nrhs)
    k = stop - start
    # every rank draws the same block and keeps its columns, row-major (what the kernels read)
    rng = np.random.default_rng([0, 7])
    full = rng.uniform(-1.0, 1.0, (n, nrhs)) if n * nrhs <= (1 << 27) else None
    if full is None:                      # large: draw this rank's columns only, column by column
        cols = [np.random.default_rng([0, 7, q]).uniform(-1.0, 1.0, n) for q in range(start, stop)]
        local = np.ascontiguousarray(np.stack(cols, axis=1))
    else:
        local = np.ascontiguousarray(full[:, start:stop])
    B = torch.from_numpy(local).to(dev)
    out = [None]
    steps = max(3, min(args.steps, 10))

    def step():
        out[0] = solver.solve(B, layout="rows")
    ms = _time_steps(step, steps, 3)
    per = _max_over_ranks(np.median(ms), world, dev)
    X = out[0].cpu().numpy()
    checks = sorted({0, k - 1})
    err = 0.0
    for q in checks:
        want = cpu.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(local[:, q]))
        err = max(err, float(np.max(np.abs(X[:, q] - want)) / np.max(np.abs(want))))
    err = _max_over_ranks(err, world, dev)
    # the column-major interface (two transpositions around the kernel), this rank's shard
    cm = torch.from_numpy(np.ascontiguousarray(local.T)).to(dev)
    cm_ms = _max_over_ranks(np.median(_time_steps(lambda: solver.solve(cm), 3, 1)), world, dev)
    nbytes = world * (12 * nnz + 4 * (n + 1)) + 16 * n * nrhs
    record = {"workload": f"multirhs_lap3d_g{size}", "n": n, "nnz": nnz, "nrhs": nrhs, "n_gpus": world,
              "rhs_per_gpu": k, "scaling": "strong", "ms": per,
              "gflops": nrhs * flops(n, nnz) / (per * 1e-3) / 1e9,
              "column_major_interface_ms": cm_ms,
              "roofline": _roofline(nbytes, per, peak, world),
              "parity": {"max_rel_error_checked_columns": err, "columns_checked_per_rank": len(checks),
                         "tolerance": 1e-10, "ok": bool(err <= 1e-10)}}
    if rank == 0 and world == 1:
        cpu_s, count = _host_time(lambda: cpu.sptrsv_csr_lower(Ap, Ai, Ax, local[:, 0].copy()), min_seconds=2.0)
        record["cpu_baseline"] = {"value": flops(n, nnz) / cpu_s / 1e9, "unit": "GFLOP/s", "cores": 1,
                                  "kind": "port", "ms_per_rhs": cpu_s * 1e3,
                                  "sample": f"{count} single right-hand-side solves"}
    return record


# ---- configuration 5b: one solve partitioned by block rows over the ranks --------------------
def config_partition(args, size=256):
    """The 3-D grid matrix cut into contiguous row blocks, one per GPU; cross-block operands are
    plain peer stores over NVLink, the final x is gathered with NCCL.  Times the whole call
    (fill of x, two barriers, kernel, gather), slowest rank, device-timed."""
    import torch
    from lcd_b200 import generators as gen
    from lcd_b200.multigpu import PartitionedSolve
    from oracle import oracle as cpu
    rank, _, world, dev = _context()
    peak, _ = measured_peak_gbs()
    tri = gen.laplacian3d_tril(size, seed=0)
    Ap, Ai, Ax = tri.csr_arrays()
    n, nnz = tri.n, tri.nnz
    if world == 1:
        # the one-GPU point of the curve: the same kernel on the whole matrix, no partition
        from lcd_b200 import ops
        up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        dAp, dAi, dAx, db = up(Ap), up(Ai), up(Ax), up(tri.b)
        t0 = time.perf_counter()
        dag = ops.dag_build("csr_lower", dAp, dAi)
        torch.cuda.synchronize()
        inspect_ms = (time.perf_counter() - t0) * 1e3
        plan = ops.OrderedPlan(dag.wavefronts, dag.n_levels)
        x = torch.empty_like(db)
        status = ops.new_status(dev)
        ms = float(np.median(_time_steps(lambda: ops.sptrsv_csr_ordered(
            dAp, dAi, dAx, db, plan, x, status=status, sync=False), max(3, min(args.steps, 10)), 3)))
        residual = cpu.relative_residual_csr(Ap, Ai, Ax, x.cpu().numpy(), tri.b)
        # the level walk shared by one block per SM (hand-off in shared memory inside a block's
        # node range): with the coefficients gathered into slot order in the call, and as a
        # repeated solve (same matrix, new right-hand side: only the walk)
        steps = max(3, min(args.steps, 10))
        walk = ops.SmallPlan("csr_lower", dAp, dAi, dag, blocks=0)
        xw = torch.empty_like(db)
        ops.sptrsv_small(walk, dAx, db, xw, sync=True)
        walk_ms = float(np.median(_time_steps(lambda: ops.sptrsv_small(walk, dAx, db, xw), steps, 3)))
        repeat_ms = float(np.median(_time_steps(
            lambda: ops.sptrsv_small(walk, dAx, db, xw, same_values=True), steps, 3)))
        walk_residual = cpu.relative_residual_csr(Ap, Ai, Ax, xw.cpu().numpy(), tri.b)
        by_kernel = {"csr_ordered_kernel": ms, "sptrsv_small_kernel shared walk, coefficients gathered": walk_ms}
        residual = max(residual, walk_residual)
        ordered_ms, ms = ms, min(ms, walk_ms)
        cpu_s, count = _host_time(lambda: cpu.sptrsv_csr_lower(Ap, Ai, Ax, tri.b), min_seconds=1.0)
        return {"workload": f"partition_lap3d_g{size}", "n": n, "nnz": nnz, "n_gpus": 1,
                "levels": dag.n_levels, "scaling": "strong", "ms": ms, "inspector_ms": inspect_ms,
                "ms_by_kernel": by_kernel, "walk_blocks": walk.blocks,
                "repeated_solve_ms": repeat_ms,
                "repeated_solve_note": "same matrix, new right-hand side: the shared level walk alone "
                                       "(coefficients already in slot order)",
                "repeated_solve_roofline": _roofline(algorithmic_bytes(n, nnz), repeat_ms, peak),
                "kernel": ("csr_ordered_kernel" if ordered_ms <= walk_ms else "sptrsv_small_kernel (shared walk)")
                          + " (whole matrix on one GPU)",
                "gflops": flops(n, nnz) / (ms * 1e-3) / 1e9,
                "roofline": _roofline(algorithmic_bytes(n, nnz), ms, peak), "cut_planes": 0,
                "parity": {"relative_residual": residual, "tolerance": 1e-12, "ok": bool(residual <= 1e-12)},
                "cpu_baseline": {"value": flops(n, nnz) / cpu_s / 1e9, "unit": "GFLOP/s", "ms": cpu_s * 1e3,
                                 "cores": 1, "kind": "port", "sample": f"{count} full solves"}}
    solver = PartitionedSolve(Ap, Ai, Ax)
    b = torch.from_numpy(tri.b).to(dev)
    out = [None]

    def step():
        out[0] = solver.solve(b, gather=True)
    ms = _time_steps(step, max(3, min(args.steps, 5)), 2)
    per = _max_over_ranks(np.median(ms), world, dev)

    def local_only():
        out[0] = solver.solve(b, gather=False)
    local_ms = _max_over_ranks(np.median(_time_steps(local_only, 3, 1)), world, dev)
    step()
    x = out[0].cpu().numpy()
    residual = cpu.relative_residual_csr(Ap, Ai, Ax, x, tri.b) if rank == 0 else 0.0
    residual = _max_over_ranks(residual, world, dev)
    levels = solver.levels
    solver.close()
    return {"workload": f"partition_lap3d_g{size}", "n": n, "nnz": nnz, "n_gpus": world, "levels": levels,
            "scaling": "strong", "ms": per, "ms_without_gather": local_ms,
            "gflops": flops(n, nnz) / (per * 1e-3) / 1e9,
            "roofline": _roofline(algorithmic_bytes(n, nnz), per, peak, world),
            "cut_planes": world - 1,
            "parity": {"relative_residual": residual, "tolerance": 1e-12, "ok": bool(residual <= 1e-12)}}


# ---- the literal counterparts of the reference's generated kernels, one small grid ------------
def config_literal_kernels(args, size=96):
    """Every kernel that mirrors one of the reference's generated variants directly (index-ordered
    polling with one and with several lanes per row, the push kernel on CSC storage, per-level
    and cooperative wavefront kernels, the multi-right-hand-side polling and wavefront kernels,
    ILU0 by index / per level), once each on the 3-D grid, checked against the CPU port.  The
    launcher prefers the level-ordered kernels over all of these on such a matrix; the record
    says by how much."""
    import torch
    import scipy.sparse as sp
    from lcd_b200 import generators as gen, ops
    from oracle import oracle as cpu
    _, _, _, dev = _context()
    up = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    tri = gen.laplacian3d_tril(size, seed=0)
    Ap, Ai, Ax = tri.csr_arrays()
    Cp, Ci, Cx = tri.csc_arrays()
    n, nnz = tri.n, tri.nnz
    dAp, dAi, dAx, db = up(Ap), up(Ai), up(Ax), up(tri.b)
    dCp, dCi, dCx = up(Cp), up(Ci), up(Cx)
    status = ops.new_status(dev)
    want = cpu.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
    dag = ops.dag_build("csr_lower", dAp, dAi)
    cdag = ops.dag_build("csc_lower", dCp, dCi)
    x = torch.empty_like(db)
    reps = max(2, min(args.steps, 5))
    out = {}

    def timed(name, fn, result=None, reference=None):
        ms = float(np.median(_time_steps(fn, reps, 1)))
        rec = {"ms": ms}
        if result is not None:
            got = result().cpu().numpy()
            ref = want if reference is None else reference
            rec["max_rel_error"] = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
        if ops.read_status(status)[0] != 0:
            rec["status"] = int(ops.read_status(status)[0])
        out[name] = rec

    timed("csr_syncfree_row_kernel", lambda: ops.sptrsv_csr_syncfree(
        dAp, dAi, dAx, db, x, lanes=1, status=status, sync=False), lambda: x)
    timed("csr_syncfree_kernel<4>", lambda: ops.sptrsv_csr_syncfree(
        dAp, dAi, dAx, db, x, lanes=4, status=status, sync=False), lambda: x)
    counts = ops.csc_edge_count(dCp, dCi)
    timed("csc_syncfree_kernel", lambda: ops.sptrsv_csc_syncfree(
        dCp, dCi, dCx, db, counts.clone(), x, status=status, sync=False), lambda: x)
    timed("wavefront_coop_kernel", lambda: ops.sptrsv_wavefront(
        "csr_lower", dAp, dAi, dAx, db, dag.wavefronts, dag.wavefront_ptr, None, x,
        mode="cooperative", status=status, sync=False), lambda: x)
    timed("wavefront_level_kernel (a launch per level)", lambda: ops.sptrsv_wavefront(
        "csr_lower", dAp, dAi, dAx, db, dag.wavefronts, dag.wavefront_ptr, dag.wavefront_ptr_host, x,
        mode="per_level", status=status, sync=False), lambda: x)
    timed("csc wavefront_coop_kernel", lambda: ops.sptrsv_wavefront(
        "csc_lower", dCp, dCi, dCx, db, cdag.wavefronts, cdag.wavefront_ptr, None, x,
        mode="cooperative", status=status, sync=False), lambda: x)
    plan = ops.OrderedPlan(dag.wavefronts, dag.n_levels)
    timed("csr_ordered_kernel (what the launcher uses)", lambda: ops.sptrsv_csr_ordered(
        dAp, dAi, dAx, db, plan, x, status=status, sync=False), lambda: x)
    # eight right-hand sides
    B = np.random.default_rng(3).uniform(-1, 1, (n, 8))
    dB = up(B)
    X = torch.empty_like(dB)
    want8 = cpu.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(B[:, 5]))
    timed("csr_syncfree_multi_kernel (8 rhs)", lambda: ops.sptrsv_csr_syncfree_multi(
        dAp, dAi, dAx, dB, X, status=status, sync=False), lambda: X[:, 5], want8)
    timed("wavefront_multi_coop_kernel (8 rhs)", lambda: ops.sptrsv_wavefront_multi(
        dAp, dAi, dAx, dB, dag.wavefronts, dag.wavefront_ptr, X, status=status, sync=False),
        lambda: X[:, 5], want8)
    timed("csr_ordered_kernel (8 rhs)", lambda: ops.sptrsv_csr_ordered(
        dAp, dAi, dAx, dB, plan, X, status=status, sync=False), lambda: X[:, 5], want8)
    # ILU0 by index and per level on the matching full matrix
    mat, _ = gen.laplacian3d_ilu0(size, seed=0)
    Fp, Fi, Fx = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    dFp, dFi, dF0 = up(Fp), up(Fi), up(Fx)
    work = dF0.clone()
    pos = ops.diag_positions(dFp, dFi)
    fdag = ops.dag_build("ilu0_csr", dFp, dFi)
    fwant = cpu.ilu0_csr(Fp, Fi, Fx, fast=True)
    done = torch.empty(len(Fp) - 1, dtype=torch.int32, device=dev)
    for name, kw in (("ilu0_lookahead_kernel by index", dict(mode="sync_free")),
                     ("ilu0_level_kernel (a launch per level)", dict(mode="wavefront")),
                     ("ilu0_lookahead_kernel in level order", dict(mode="ordered", scratch=False)),
                     ("ilu0_valueflag_kernel (what the launcher uses)", dict(mode="ordered"))):
        def step():
            work.copy_(dF0)
            ops.spilu0_csr(dFp, dFi, work, pos, wavefronts=fdag.wavefronts,
                           wavefront_ptr_host=fdag.wavefront_ptr_host, done=done, status=status,
                           sync=False, max_row=7, **kw)
        ms = float(np.median(_time_steps(step, reps, 1)))
        out[name] = {"ms_with_restore_of_A": ms,
                     "bit_identical": bool(np.array_equal(work.cpu().numpy(), fwant))}
    return {"workload": f"literal_kernels_lap3d_g{size}", "n": n, "nnz": nnz, "levels": dag.n_levels,
            "kernels": out}


CONFIG_RUNNERS = {"literal": config_literal_kernels, "ilu0": config_ilu0, "supernodal": config_supernodal, "multirhs": config_multirhs,
                  "csc": config_csc_lap2d, "partition": config_partition}


def other_configurations(args, rank, world):
    """The configurations next to the headline one.  One GPU: the CSC demo, ILU0 with its two
    solves, the supernodal solve and the 64 right-hand sides.  Several GPUs: the 64 right-hand
    sides split by column and one large solve partitioned by block rows."""
    import torch
    if world == 1:
        plan = [("cfg1_csc_lap2d_g256", "csc", 256), ("cfg3_ilu0_lap3d_g128", "ilu0", 128),
                ("cfg4_supernodal_n1048576", "supernodal", 1_048_576),
                ("cfg5a_multirhs_lap3d_g192", "multirhs", 192),
                ("cfg5b_partition_lap3d_g256", "partition", 256)]
    else:
        plan = [("cfg5a_multirhs_lap3d_g192", "multirhs", 192),
                ("cfg5b_partition_lap3d_g256", "partition", 256)]
    out = {}
    for name, kind, size in plan:
        t0 = time.time()
        try:
            out[name] = CONFIG_RUNNERS[kind](args, size)
            out[name]["bench_seconds"] = round(time.time() - t0, 1)
        except Exception as error:          # the headline line must still be printed
            if world > 1:
                raise                       # (a rank that stops alone would hang the others)
            out[name] = {"error": f"{type(error).__name__}: {error}"}
        torch.cuda.empty_cache()
        if rank == 0:
            log(f"[bench] {name}: {time.time() - t0:.1f}s")
    return out


def run_side_workload(args):
    """One of the other configurations alone (smaller sizes for profiling runs): prints its
    record as one JSON line."""
    import torch
    import torch.distributed as dist
    kind, size = SIDE_WORKLOADS[args.workload]
    rank, local_rank, world, dev = _context()
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    peak, peak_kind = measured_peak_gbs()
    line = {"data": "synthetic", "dtype": "f64", "steps": args.steps, "peak_gbs": peak,
            "peak_kind": peak_kind}
    line.update(CONFIG_RUNNERS[kind](args, size))
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", default="native", choices=("native", "reference"))
    parser.add_argument("--workload", default=DEFAULT_WORKLOAD,
                        choices=sorted(WORKLOADS) + sorted(SIDE_WORKLOADS))
    parser.add_argument("--lanes", type=int, default=0)
    parser.add_argument("--threads", type=int, default=0)
    parser.add_argument("--skip-extras", action="store_true",
                        help="skip the DAG-build and wavefront side measurements")
    parser.add_argument("--solver", choices=("auto", "row", "chain"), default="auto",
                        help="sync-free kernel: polling rows, block-recurrence chain, or by level count")
    parser.add_argument("--kernel-only", action="store_true",
                        help="time the kernel only (profiling runs): no e2e, CPU baseline, extras")
    parser.add_argument("--skip-configs", action="store_true",
                        help="headline configuration only: skip the records of the other configurations")
    args = parser.parse_args()
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        # the data path uses plain peer stores and NCCL only for gathers and small reductions:
        # no in-switch reduction is needed, and a rank that stops with an error must not leave
        # memory bound to an NVLink multicast object
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    args.warmup = max(args.warmup, 3) if args.impl == "native" else args.warmup
    if args.workload in SIDE_WORKLOADS:
        run_side_workload(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_native(args)


if __name__ == "__main__":
    main()
