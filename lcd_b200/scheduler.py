"""Schedule search space and the level-width scheduler.

Keeps the public interface of the reference's ``compiler/scheduler.py``
(``Schedule`` / ``ScheduleSpace`` / ``SchedulePlan`` / ``WorkloadFeatures`` /
``AnalyticScheduler.schedule`` / ``inspection_fingerprint``, ``:100-303``,
``:306-452``, ``:678-711``) so existing ``parallel(...)`` call sites keep
working, but replaces the cost model.  The reference estimates
``launch_latency * levels`` against ``atomic_cost * rows`` and has no term for
the critical path; here the decision is taken from the level structure the DAG
build measured, with constants measured on B200:

* sync-free:        levels * t_handoff (0.6 us) + rows * 1.1 ns, or, for CSR triangular
                    solves with narrow levels, rows * 7 ns (block-recurrence chain solver)
* level-synchronous, levels that fit one block (<= 512 rows):
                    levels * (2.4 us + 13 ns * width)   (block-level barriers)
* level-synchronous, wide levels:
                    levels * t_grid_barrier (3 us) + rows * 0.5 ns

so a long chain of narrow levels goes to the sync-free kernel (754,679 levels:
0.46 s against 1.8 s), while grids with thousands of rows per level are a near
tie that the level-synchronous kernel wins, clearly so for ILU0 whose sync-free
hand-off is about 8x dearer.
"""

from __future__ import annotations

import hashlib
import itertools
from dataclasses import dataclass, replace

import numpy as np

WAVEFRONT = "wavefront"
SYNC_FREE = "sync_free"
AUTO = "auto"
EXECUTION_MODES = (WAVEFRONT, SYNC_FREE)
BLOCK_SIZES = (32, 64, 128, 256)
UNROLL_FACTORS = (1, 2, 4, 8)
DEFAULT_THREADS_PER_BLOCK = 128
N_WARP_CANDIDATES = (1,)
WARP_SIZE = 32
COUNTER_DEPENDENCE = "counter"
PUSH_DEPENDENCE = "push"
PULL_DEPENDENCE = "pull"


class SchedulerError(Exception):
    pass


@dataclass(frozen=True)
class ArchConstants:
    """Machine model.  The first four fields are the reference's; the last three
    are what the level-width model uses (seconds per grid barrier, per sync-free
    hand-off through L2, per hand-off through shared memory)."""

    launch_latency_s: float
    atomic_cost_s: float
    memory_bandwidth_bytes_per_s: float
    lane_flops_per_s: float
    barrier_s: float = 3.0e-6           # grid-wide barrier after a level that spans the grid
    block_level_s: float = 2.4e-6       # one level walked by a single block (__syncthreads)
    block_level_row_s: float = 1.3e-8   # ... plus this much per row of that level
    wavefront_row_s: float = 0.5e-9     # streaming cost per row in wide levels
    handoff_s: float = 0.6e-6           # sync-free: one dependence hop on the critical chain
    syncfree_row_s: float = 1.1e-9      # sync-free: per-row cost when many rows are in flight
    chain_row_s: float = 7.0e-9         # block-recurrence chain solver: per row, whatever the levels
    chain_min_rows: int = 32768         # ... below this the preparation does not pay
    block_level_width: int = 512        # levels up to this width stay inside one block


FALLBACK_ARCH_CONSTANTS = ArchConstants(
    launch_latency_s=3.0e-6,
    atomic_cost_s=2.0e-9,
    memory_bandwidth_bytes_per_s=6.5e12,
    lane_flops_per_s=1.5e9,
)


@dataclass(frozen=True)
class WorkloadFeatures:
    rows: int
    edges: int
    levels: int
    nonzeros: int
    flops: float
    memory_bytes: int
    thread_work_items: int = 0
    thread_loop_invocations: int = 0
    max_level_width: int = 0
    sync_free_penalty: float = 1.0   # operators whose sync-free kernel does more work per hop
    chain_capable: bool = False      # the operator has a block-recurrence solver (CSR SpTRSV)

    @property
    def average_in_degree(self):
        return self.edges / self.rows if self.rows else 0.0

    @property
    def average_thread_trip_count(self):
        if self.thread_loop_invocations == 0:
            return 0.0
        return self.thread_work_items / self.thread_loop_invocations

    @property
    def average_level_width(self):
        return self.rows / self.levels if self.levels else 0.0


@dataclass(frozen=True)
class CostEstimate:
    launch_s: float
    sync_s: float
    memory_s: float
    compute_s: float

    @property
    def total_s(self):
        return self.launch_s + self.sync_s + self.memory_s + self.compute_s


@dataclass(frozen=True)
class Schedule:
    execution_mode: str
    threads_per_block: int
    thread_unroll: int
    n_warp: int = 1
    dependence_protocol: str = COUNTER_DEPENDENCE
    cost: CostEstimate | None = None

    @property
    def lowering_key(self):
        return (self.execution_mode, self.threads_per_block, self.thread_unroll, self.n_warp,
                self.dependence_protocol)


@dataclass(frozen=True)
class SchedulePlan:
    schedule: Schedule
    execution_data: object
    features: WorkloadFeatures | None = None
    rows: int = 0
    levels: int = 0
    dag: object = None      # device arrays of the inspector (level sets for the launchers)


def normalize_execution_mode(execution_mode):
    if execution_mode is None or execution_mode == AUTO:
        return None
    if execution_mode.replace("-", "_") == SYNC_FREE:
        return SYNC_FREE
    return WAVEFRONT


def task_threads(threads_per_block, n_warp):
    if threads_per_block % WARP_SIZE:
        return threads_per_block
    return min(threads_per_block, WARP_SIZE * n_warp)


def _warp_task(threads_per_block, n_warp):
    return n_warp == 1 and threads_per_block % WARP_SIZE == 0


@dataclass(frozen=True)
class ScheduleSpace:
    execution_modes: tuple
    block_sizes: tuple
    unroll_factors: tuple
    n_warps: tuple = N_WARP_CANDIDATES
    thread_mapped: bool = False
    dependence_protocols: tuple = (COUNTER_DEPENDENCE,)

    @classmethod
    def from_options(cls, execution_mode=None, threads_per_block=None, thread_unroll=None,
                     thread_mapped=False, n_warp=None, direct_protocol=None,
                     dependence_protocol=None):
        mode = normalize_execution_mode(execution_mode)
        if n_warp is not None and (not isinstance(n_warp, int) or n_warp <= 0):
            raise SchedulerError("n_warp must be a positive integer.")
        block_task = n_warp is not None and n_warp > 1
        if block_task and threads_per_block is not None \
                and threads_per_block != n_warp * WARP_SIZE:
            raise SchedulerError(
                f"n_warp={n_warp} maps one task to {n_warp * WARP_SIZE} threads, "
                f"but threads_per_block={threads_per_block}.")
        if n_warp == 1 and thread_mapped and threads_per_block is not None \
                and threads_per_block % WARP_SIZE:
            raise SchedulerError(
                f"n_warp=1 requires threads_per_block to be a multiple of {WARP_SIZE}, "
                f"but threads_per_block={threads_per_block}.")
        if threads_per_block is not None:
            block_sizes = (threads_per_block,)
        elif block_task:
            block_sizes = (n_warp * WARP_SIZE,)
        elif thread_mapped:
            block_sizes = BLOCK_SIZES
        else:
            block_sizes = (DEFAULT_THREADS_PER_BLOCK,)
        if thread_unroll is not None:
            unroll_factors = (thread_unroll,)
        else:
            unroll_factors = UNROLL_FACTORS if thread_mapped else (1,)
        modes = EXECUTION_MODES if mode is None else (mode,)
        n_warps = N_WARP_CANDIDATES if n_warp is None else (n_warp,)
        available = (COUNTER_DEPENDENCE,) + (
            (direct_protocol,) if thread_mapped and direct_protocol is not None else ())
        searched = len(modes) * len(block_sizes) * len(unroll_factors) * len(n_warps) > 1
        if dependence_protocol is not None:
            if dependence_protocol not in available:
                raise SchedulerError(
                    f"Dependence protocol {dependence_protocol!r} is not supported by this "
                    "loop; available protocols: " + ", ".join(available) + ".")
            protocols = (dependence_protocol,)
        elif PUSH_DEPENDENCE in available:
            protocols = (PUSH_DEPENDENCE,)
        elif PULL_DEPENDENCE in available and searched:
            protocols = (COUNTER_DEPENDENCE, PULL_DEPENDENCE)
        else:
            protocols = (COUNTER_DEPENDENCE,)
        return cls(modes, block_sizes, unroll_factors, n_warps, thread_mapped, protocols)

    def configurations(self):
        out = []
        for mode, tpb, unroll, n_warp in itertools.product(
                self.execution_modes, self.block_sizes, self.unroll_factors, self.n_warps):
            direct = mode == SYNC_FREE and self.thread_mapped and _warp_task(tpb, n_warp)
            protocols = self.dependence_protocols if direct else (COUNTER_DEPENDENCE,)
            out.extend((mode, tpb, unroll, n_warp, protocol) for protocol in protocols)
        return out

    @property
    def is_fixed(self):
        return len(self.configurations()) == 1

    def fixed_schedule(self):
        if not self.is_fixed:
            raise SchedulerError("The schedule space has more than one configuration.")
        return Schedule(*self.configurations()[0])


class AnalyticScheduler:
    """Chooses among the configurations of a :class:`ScheduleSpace`.

    The name and call signature are the reference's; the estimate is the
    level-width model described in the module docstring."""

    def __init__(self, arch_constants=None):
        self._arch_constants = arch_constants

    @property
    def arch_constants(self):
        if self._arch_constants is None:
            self._arch_constants = measure_arch_constants()
        return self._arch_constants

    def estimate(self, features, execution_mode, threads_per_block, thread_unroll, n_warp,
                 thread_mapped, dependence_protocol=COUNTER_DEPENDENCE):
        arch = self.arch_constants
        memory_s = features.memory_bytes / arch.memory_bandwidth_bytes_per_s
        lanes = task_threads(threads_per_block, n_warp) * thread_unroll if thread_mapped else 1
        trip = features.average_thread_trip_count if (
            thread_mapped and features.thread_loop_invocations) else features.average_in_degree
        active = min(lanes, max(trip, 1.0))
        compute_s = features.flops / (active * arch.lane_flops_per_s * 148 * 64)
        width = features.average_level_width
        if execution_mode == WAVEFRONT:
            if width <= arch.block_level_width:
                per_level = arch.block_level_s + arch.block_level_row_s * width
                sync_s = features.levels * per_level
            else:
                sync_s = features.levels * arch.barrier_s + features.rows * arch.wavefront_row_s
            return CostEstimate(arch.launch_latency_s, sync_s, memory_s, compute_s)
        if execution_mode == SYNC_FREE:
            # a hand-off is a poll of the operand itself; the chain pays one per level,
            # wide levels add a throughput term
            sync_s = (features.levels * arch.handoff_s + features.rows * arch.syncfree_row_s)
            sync_s *= features.sync_free_penalty
            if features.chain_capable and chain_solver_preferred(features.rows, features.levels,
                                                                 arch):
                sync_s = features.rows * arch.chain_row_s
            if dependence_protocol == PULL_DEPENDENCE:
                sync_s *= 0.99
            return CostEstimate(arch.launch_latency_s, sync_s, memory_s, compute_s)
        raise SchedulerError(f"Unknown execution mode {execution_mode!r}.")

    def candidates(self, features, space):
        return [Schedule(mode, tpb, unroll, n_warp, protocol,
                         cost=self.estimate(features, mode, tpb, unroll, n_warp,
                                            space.thread_mapped, protocol))
                for mode, tpb, unroll, n_warp, protocol in space.configurations()]

    def schedule(self, features, space):
        return min(self.candidates(features, space), key=_schedule_rank)


def chain_solver_preferred(rows, levels, arch=None):
    """True when the block-recurrence chain solver is expected to beat the polling
    sync-free kernel: its time grows with the rows only, the polling kernel's with the
    levels.  The sync-free launcher of CSR triangular solves takes the same decision."""
    arch = arch or FALLBACK_ARCH_CONSTANTS
    if rows < arch.chain_min_rows or levels <= 0:
        return False
    polling_s = levels * arch.handoff_s + rows * arch.syncfree_row_s
    return rows * arch.chain_row_s < polling_s


# Measured on B200: a level costs the one-block solver about 0.2 us (block barrier, operands in
# shared memory) and one SM streams its packed arrays at about 60 GB/s; a hand-off through L2
# (polling kernels, grid barriers) costs about 1 us per level whatever the kernel.
SMALL_LEVEL_S = 0.2e-6
SMALL_STREAM_BYTES_PER_S = 60e9
L2_HANDOFF_S = 1.0e-6
ORDERED_MIN_AVERAGE_WIDTH = 64


def small_solver_preferred(rows, entries, levels):
    """True when one thread block walking the levels is expected to beat the kernels that hand
    values over through L2: few rows, many levels."""
    if rows <= 0 or levels <= 0:
        return False
    small_s = levels * SMALL_LEVEL_S + (12.0 * entries + 32.0 * rows) / SMALL_STREAM_BYTES_PER_S
    return small_s < levels * L2_HANDOFF_S + 10e-6


def ordered_solver_preferred(rows, levels, average_row):
    """True when the level-ordered sync-free kernel (one lane per row, rows of a level side by
    side) is expected to beat the index-ordered one: wide levels, short rows."""
    return levels > 0 and rows / levels >= ORDERED_MIN_AVERAGE_WIDTH and average_row <= 24


def _schedule_rank(schedule):
    return (schedule.cost.total_s,
            task_threads(schedule.threads_per_block, schedule.n_warp) * schedule.thread_unroll,
            abs(schedule.threads_per_block.bit_length()
                - DEFAULT_THREADS_PER_BLOCK.bit_length()),
            schedule.threads_per_block, schedule.n_warp,
            EXECUTION_MODES.index(schedule.execution_mode), schedule.dependence_protocol)


_MEASURED_CONSTANTS = {}
CALIBRATION_NAMES = ("launch_s", "l2_handoff_s", "shared_memory_handoff_s", "block_barrier_s",
                     "contended_atomic_s", "grid_barrier_s", "copy_bytes_per_s", "l2_load_s",
                     "l2_load_p10_s", "l2_load_p90_s")


def calibrate(workspace_bytes=256 << 20):
    """Raw figures of ``lcd_calibrate`` on the current device (a dict by CALIBRATION_NAMES)."""
    import ctypes
    import torch
    from . import _native as nat
    workspace = torch.empty(workspace_bytes, dtype=torch.uint8, device="cuda")
    out = (ctypes.c_double * 16)()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    nat.check(nat.load().lcd_calibrate(nat.ptr(workspace), workspace.numel(), stream, ctypes.byref(out)),
              "lcd_calibrate")
    return {name: float(out[k]) for k, name in enumerate(CALIBRATION_NAMES)}


def measure_arch_constants():
    """Machine constants of the current device, measured on it once per process and device
    (``lcd_calibrate``: launch latency, hand-off through L2, contended atomic, grid barrier, copy
    bandwidth), as the reference measures its own (compiler/scheduler.py:714-775).  Figures that
    could not be measured keep the values observed on B200; without a GPU all of them do."""
    try:
        import torch
        if torch.cuda.is_available():
            device = torch.cuda.current_device()
            if device not in _MEASURED_CONSTANTS:
                raw = calibrate()
                pick = lambda name, default: raw[name] if raw.get(name, 0.0) > 0.0 else default
                base = FALLBACK_ARCH_CONSTANTS
                _MEASURED_CONSTANTS[device] = replace(
                    base,
                    launch_latency_s=pick("launch_s", base.launch_latency_s),
                    atomic_cost_s=pick("contended_atomic_s", base.atomic_cost_s),
                    memory_bandwidth_bytes_per_s=pick("copy_bytes_per_s", base.memory_bandwidth_bytes_per_s),
                    barrier_s=pick("grid_barrier_s", base.barrier_s),
                    handoff_s=pick("l2_handoff_s", base.handoff_s))
            return _MEASURED_CONSTANTS[device]
    except Exception:  # no device, or no library: the cost model still needs numbers
        pass
    return FALLBACK_ARCH_CONSTANTS


def pointer_array_names(function_props):
    return [name for name, properties in (function_props or {}).items()
            if isinstance(name, str) and "monotonically_increasing" in properties]


def _array_nbytes(value):
    if isinstance(value, np.ndarray):
        return value.nbytes
    if hasattr(value, "element_size") and hasattr(value, "numel"):
        return value.element_size() * value.numel()
    return 0


def extract_workload_features(dag, wavefront_list, argument_values, function_props=None,
                              flops_per_iteration=1, thread_trip_counts=None,
                              sync_free_penalty=1.0, chain_capable=False):
    """Features of one concrete input.  ``dag`` is either the reference's list of
    successor lists or a device DAG (then everything is read from its sizes)."""
    if hasattr(dag, "n_edges"):
        if getattr(dag, "capped", False):
            # deep DAG whose level sets were not built: a lower bound of the level count is all
            # the cost model needs to send it to the sync-free schedules
            rows, edges, levels = dag.n, dag.n_edges, dag.levels_at_least
            widths = np.asarray([max(1, rows // max(levels, 1))], dtype=np.int64)
        else:
            rows, edges, levels = dag.n, dag.n_edges, dag.n_levels
            widths = np.diff(dag.wavefront_ptr_host) if levels else np.zeros(0, dtype=np.int64)
    else:
        rows = len(dag)
        edges = sum(len(s) for s in dag)
        levels = len(wavefront_list)
        widths = np.asarray([len(w) for w in wavefront_list], dtype=np.int64)
    nonzeros = None
    for name in pointer_array_names(function_props):
        value = argument_values.get(name)
        if value is not None and len(value) >= 2:
            count = int(value[-1]) - int(value[0])
            nonzeros = count if nonzeros is None else max(nonzeros, count)
    if nonzeros is None:
        nonzeros = rows + edges
    if thread_trip_counts is None:
        work, invocations, items = nonzeros, 0, 0
    else:
        if isinstance(thread_trip_counts, tuple) and len(thread_trip_counts) == 2 \
                and not isinstance(thread_trip_counts[0], (tuple, list)):
            items, invocations = int(thread_trip_counts[0]), int(thread_trip_counts[1])
        else:
            counts = [max(int(c), 0) for c in thread_trip_counts]
            items, invocations = sum(counts), len(counts)
        work = items
    seen = {}
    for value in argument_values.values():
        if _array_nbytes(value):
            seen[id(value)] = _array_nbytes(value)
    return WorkloadFeatures(rows=rows, edges=edges, levels=levels, nonzeros=nonzeros,
                            flops=float(flops_per_iteration * work),
                            memory_bytes=int(sum(seen.values())),
                            thread_work_items=items, thread_loop_invocations=invocations,
                            max_level_width=int(widths.max()) if len(widths) else 0,
                            sync_free_penalty=float(sync_free_penalty),
                            chain_capable=bool(chain_capable))


def _digest(value):
    if isinstance(value, np.ndarray):
        if value.dtype.hasobject:
            return object()
        data = np.ascontiguousarray(value)
        return (data.dtype.str, data.shape,
                hashlib.blake2b(data.reshape(-1).view(np.uint8), digest_size=16).digest())
    if hasattr(value, "data_ptr") and hasattr(value, "cpu"):
        return _digest(value.detach().cpu().numpy())
    if isinstance(value, (list, tuple)):
        try:
            return _digest(np.asarray(value))
        except (TypeError, ValueError):
            return object()
    if value is None or np.isscalar(value):
        return type(value).__name__, value
    return object()


def inspection_fingerprint(values, content_names):
    """Cache key of an inspection: content digests of the structure arrays plus
    dtype/shape of every array argument (same rule as the reference)."""
    content = tuple((name, _digest(values.get(name))) for name in sorted(set(content_names)))
    shapes = tuple((name, value.dtype.str, value.shape)
                   for name, value in sorted(values.items()) if isinstance(value, np.ndarray))
    return content, shapes


if __name__ == "__main__":          # python -m lcd_b200.scheduler --calibrate
    import json
    import sys
    if "--calibrate" in sys.argv:
        print(json.dumps({"raw": calibrate(), "arch_constants": measure_arch_constants().__dict__}, indent=1))
