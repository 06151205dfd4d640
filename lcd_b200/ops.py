"""Torch-tensor front end of the C ABI: one thin function per entry point.

Tensors only provide device memory and the current stream; all work happens in
``liblcd_b200.so``.  Index tensors are ``int32``, values ``float64``, everything
contiguous and on the same CUDA device.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as nat
from ._native import NativeError, check, ptr

OPS = {"csr_lower": nat.OP_CSR_LOWER, "csc_lower": nat.OP_CSC_LOWER,
       "ilu0_csr": nat.OP_ILU0_CSR, "csr_upper": nat.OP_CSR_UPPER,
       "csc_upper": nat.OP_CSC_UPPER, "csr_lower_rows": nat.OP_CSR_LOWER_ROWS,
       "csr_upper_rows": nat.OP_CSR_UPPER_ROWS}


def _op_code(op):
    return OPS[op] if isinstance(op, str) else int(op)


_raw_stream = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream():
    """Handle of the current CUDA stream (the raw-handle getter when this torch has it:
    ``torch.cuda.current_stream()`` builds a Stream object per call)."""
    if _raw_stream is not None:
        return ctypes.c_void_p(_raw_stream(torch.cuda.current_device()))
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _require(t, dtype, name):
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError(f"{name} must be a CUDA tensor (lcd_b200 has no CPU path)")
    if t.dtype != dtype or not t.is_contiguous():
        raise TypeError(f"{name} must be a contiguous {dtype} tensor")
    return t


def new_status(device):
    return torch.zeros(nat.STATUS_WORDS, dtype=torch.int32, device=device)


def read_status(status):
    node = ctypes.c_int32(-1)
    code = nat.load().lcd_read_status(ptr(status), _stream(), ctypes.byref(node))
    return code, node.value


def to_device(array, dtype=None, device="cuda"):
    """Host array -> device tensor through pinned memory."""
    a = np.ascontiguousarray(array, dtype=dtype)
    return torch.from_numpy(a).to(device, non_blocking=False)


class DeviceDag:
    """Outputs of the on-device DAG build (all int32 device tensors).

    Built with a level cap that was reached (``capped``), the level arrays - ``level``,
    ``wavefronts``, ``wavefront_ptr``, ``n_levels`` - are not there yet; reading one of them runs
    the full build once.  ``levels_at_least`` is a lower bound that never triggers that."""

    def __init__(self, n, op, dep_count, edge_count, dag_ptr, dag_index, n_edges, level, wavefronts,
                 wavefront_ptr, n_levels, capped_at=0, complete=None):
        self.n, self.op = n, op
        self.dep_count, self.edge_count = dep_count, edge_count
        self.dag_ptr, self.dag_index, self.n_edges = dag_ptr, dag_index, n_edges
        self._level, self._wavefronts, self._wavefront_ptr = level, wavefronts, wavefront_ptr
        self._n_levels = n_levels
        self._wavefront_ptr_host = None
        self.capped_at = int(capped_at)
        self._complete = complete

    @property
    def capped(self):
        return self.capped_at > 0

    @property
    def levels_at_least(self):
        return self.capped_at + 1 if self.capped else self._n_levels

    def _levels(self):
        if self.capped:
            full = self._complete()
            self._level, self._wavefronts = full._level, full._wavefronts
            self._wavefront_ptr, self._n_levels = full._wavefront_ptr, full._n_levels
            self.capped_at, self._complete = 0, None
        return self

    level = property(lambda self: self._levels()._level)
    wavefronts = property(lambda self: self._levels()._wavefronts)
    wavefront_ptr = property(lambda self: self._levels()._wavefront_ptr)
    n_levels = property(lambda self: self._levels()._n_levels)

    @property
    def wavefront_ptr_host(self):
        if self._wavefront_ptr_host is None:
            self._wavefront_ptr_host = self.wavefront_ptr.cpu().numpy()
        return self._wavefront_ptr_host


def dag_build(op, ptr_t, idx_t, n=None, timeout_ms=0, level_cap=0):
    """Dependence DAG, level sets and topological order of one operator.  ``level_cap`` > 0 stops
    the level propagation (the sequential part) once a node reaches that level: the result then
    is ``capped`` and completes itself when its level arrays are read."""
    op = _op_code(op)
    _require(ptr_t, torch.int32, "ptr")
    _require(idx_t, torch.int32, "idx")
    n = ptr_t.numel() - 1 if n is None else int(n)
    nnz = idx_t.numel()
    dev = ptr_t.device
    lib = nat.load()
    need = ctypes.c_int64(0)
    check(lib.lcd_dag_workspace_bytes(op, n, nnz, ctypes.byref(need)), "lcd_dag_workspace_bytes")
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    dep = torch.empty(n, **i32)
    edge = torch.empty(n, **i32)
    dag_ptr = torch.empty(n + 1, **i32)
    dag_index = torch.empty(max(nnz, 1), **i32)
    level = torch.empty(n, **i32)
    waves = torch.empty(n, **i32)
    wptr = torch.empty(n + 1, **i32)
    n_edges = ctypes.c_int64(0)
    n_levels = ctypes.c_int32(0)
    rc = lib.lcd_dag_build_capped(op, n, ptr(ptr_t), ptr(idx_t), nnz, ptr(dep), ptr(edge), ptr(dag_ptr),
                                  ptr(dag_index), ctypes.byref(n_edges), ptr(level), ptr(waves),
                                  ptr(wptr), ctypes.byref(n_levels), int(level_cap), ptr(ws), need.value,
                                  int(timeout_ms), _stream())
    check(rc, "lcd_dag_build")
    del ws
    if n_levels.value < 0:          # the cap was reached: level arrays on demand
        return DeviceDag(n, op, dep, edge, dag_ptr, dag_index[:n_edges.value], n_edges.value, None, None,
                         None, 0, capped_at=-n_levels.value,
                         complete=lambda: dag_build(op, ptr_t, idx_t, n=n, timeout_ms=timeout_ms))
    return DeviceDag(n, op, dep, edge, dag_ptr, dag_index[:n_edges.value], n_edges.value, level, waves,
                     wptr[:n_levels.value + 1], n_levels.value)


def band_chains(dag, band_width):
    """(task_nodes, task_ptr, band_ptr) of the warp executor's tasks for ``band_width`` > 1:
    int32 device tensors, element-wise the reference's ``_band_chains``."""
    lib = nat.load()
    n, dev = dag.n, dag.wavefronts.device
    need = ctypes.c_int64(0)
    check(lib.lcd_band_chains_workspace_bytes(n, ctypes.byref(need)), "lcd_band_chains_workspace_bytes")
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    n_bands = (dag.n_levels + band_width - 1) // band_width
    task_nodes = torch.empty(max(n, 1), **i32)
    task_ptr = torch.empty(n + 1, **i32)
    band_ptr = torch.empty(n_bands + 1, **i32)
    n_tasks = ctypes.c_int32(0)
    check(lib.lcd_band_chains(n, ptr(dag.dag_ptr), ptr(dag.dag_index), ptr(dag.level),
                              ptr(dag.wavefronts), ptr(dag.wavefront_ptr), dag.n_levels,
                              int(band_width), ptr(task_nodes), ptr(task_ptr), ptr(band_ptr),
                              ctypes.byref(n_tasks), ptr(ws), need.value, _stream()),
          "lcd_band_chains")
    return task_nodes[:n], task_ptr[:n_tasks.value + 1], band_ptr


def diag_positions(ptr_t, idx_t, status=None):
    _require(ptr_t, torch.int32, "ptr")
    _require(idx_t, torch.int32, "idx")
    n = ptr_t.numel() - 1
    pos = torch.empty(n, dtype=torch.int32, device=ptr_t.device)
    status = new_status(ptr_t.device) if status is None else status
    host = ctypes.c_int(0)
    rc = nat.load().lcd_diag_positions(n, ptr(ptr_t), ptr(idx_t), idx_t.numel(), ptr(pos),
                                       ptr(status), _stream(), ctypes.byref(host))
    check(rc, "lcd_diag_positions")
    return pos


def _solve_flags(upper, unit_diag, of_full, exact):
    return ((nat.SOLVE_UPPER if upper else 0) | (nat.SOLVE_UNIT_DIAG if unit_diag else 0)
            | (nat.SOLVE_OF_FULL if of_full else 0) | (nat.SOLVE_EXACT if exact else 0))


@dataclass
class GaussSeidelLayout:
    """Diagonal-last rows of a Gauss-Seidel sweep over a lower-triangular matrix."""

    Ap: torch.Tensor
    Ai: torch.Tensor
    perm: torch.Tensor
    nnz: int
    separate_diagonal: bool


def gs_layout(Ap, Ai, *, separate_diagonal):
    """Structure part of the conversion (once per matrix): rows whose diagonal is kept in a
    separate array (``separate_diagonal``) or stored somewhere in the row become rows with
    the diagonal last, which is what the CSR solvers read."""
    _require(Ap, torch.int32, "Ap")
    _require(Ai, torch.int32, "Ai")
    n, nnz, dev = Ap.numel() - 1, Ai.numel(), Ap.device
    lib = nat.load()
    need = ctypes.c_int64(0)
    check(lib.lcd_gs_layout_workspace_bytes(n, ctypes.byref(need)), "lcd_gs_layout_workspace_bytes")
    ws = torch.empty(need.value, dtype=torch.uint8, device=dev)
    Ap_out = torch.empty(n + 1, dtype=torch.int32, device=dev)
    Ai_out = torch.empty(max(nnz + n, 1), dtype=torch.int32, device=dev)
    perm = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    status = new_status(dev)
    total, host = ctypes.c_int64(0), ctypes.c_int(0)
    rc = lib.lcd_gs_layout(n, nnz, ptr(Ap), ptr(Ai), 0 if separate_diagonal else 1, ptr(Ap_out),
                           ptr(Ai_out), ptr(perm), ctypes.byref(total), ptr(ws), ws.numel(),
                           ptr(status), _stream(), ctypes.byref(host))
    check(rc, "lcd_gs_layout")
    if n == 0:
        Ap_out.zero_()
    return GaussSeidelLayout(Ap_out, Ai_out[:max(total.value, 0)].contiguous() if total.value else Ai_out[:0],
                             perm, int(total.value), bool(separate_diagonal))


def gs_values(layout, Ax, diagonal=None, out=None):
    """Value part of the conversion (every call): scatter the stored values to their slots and
    fill the diagonal slots from ``diagonal`` (separate array), the row's own entry, or 1.0."""
    _require(Ax, torch.float64, "Ax")
    if layout.separate_diagonal:
        _require(diagonal, torch.float64, "diagonal")
    n = layout.Ap.numel() - 1
    out = torch.empty(max(layout.nnz, 1), dtype=torch.float64, device=Ax.device) if out is None else out
    check(nat.load().lcd_gs_values(n, Ax.numel(), ptr(layout.Ap), ptr(layout.perm), ptr(Ax),
                                   ptr(diagonal) if layout.separate_diagonal else None, ptr(out),
                                   _stream()), "lcd_gs_values")
    return out[:layout.nnz]


def chain_workspace(n, device):
    """Scratch for the block-recurrence chain solver (56 KiB per 64 rows)."""
    need = ctypes.c_int64(0)
    check(nat.load().lcd_chain_workspace_bytes(int(n), ctypes.byref(need)), "lcd_chain_workspace_bytes")
    return torch.empty((need.value + 7) // 8, dtype=torch.float64, device=device)


CHAIN_PREPARE_ROWS = 64      # granularity of the row ranges of chain_prepare
CHAIN_SOLVE_ROWS = 512       # ... and of sptrsv_csr_chain


def chain_prepare(Ap, Ai, Ax, workspace, *, upper=False, unit_diag=False, diag_pos=None, rows=None):
    """Build the block tiles (inverse of each 64-row diagonal block and its product with the
    coupling to the block before) into ``workspace``; repeat when Ax changes.  ``rows`` =
    (begin, end) restricts the call to those rows in solve order (begin a multiple of 64, end
    too unless it is n): only their entries of Ax are read."""
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, False)
    n = Ap.numel() - 1
    begin, end = (0, n) if rows is None else rows
    check(nat.load().lcd_chain_prepare_rows(n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax),
                                            ptr(diag_pos), flags, ptr(workspace),
                                            workspace.numel() * 8, int(begin), int(end), _stream()),
          "lcd_chain_prepare_rows")
    return workspace


def chain_growth(workspace, n):
    """Growth figure of the block inverses in ``workspace`` (synchronises the stream): compare
    with ``CHAIN_MAX_GROWTH``; above it the chain solver loses accuracy that substitution keeps."""
    out = ctypes.c_double(0.0)
    check(nat.load().lcd_chain_growth(int(n), ptr(workspace), workspace.numel() * 8, _stream(),
                                      ctypes.byref(out)), "lcd_chain_growth")
    return float(out.value)


CHAIN_MAX_GROWTH = nat.CHAIN_MAX_GROWTH


def sptrsv_csr_chain(Ap, Ai, Ax, b, workspace, x=None, *, upper=False, unit_diag=False,
                     diag_pos=None, status=None, timeout_ms=0, sync=True, rows=None):
    """Block-recurrence chain solve (for matrices whose levels hold only a few rows).
    ``workspace`` must have been filled by ``chain_prepare`` for the same matrix.

    ``rows`` = (begin, end) solves only those rows in solve order (begin a multiple of 512,
    end too unless it is n); the ranges of one solve are issued in order on one stream, with
    the same ``x`` and ``status``, starting at 0 and ending at n.  A range needs the tiles and
    the matrix entries of its own rows only, so a solve can start while later rows are still
    being uploaded or prepared.  The status is read back (``sync``) by the range that ends at n."""
    _require(b, torch.float64, "b")
    n = Ap.numel() - 1
    x = torch.empty(n, dtype=torch.float64, device=b.device) if x is None else x
    status = new_status(b.device) if status is None else status
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, False)
    begin, end = (0, n) if rows is None else rows
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_csr_chain_rows(
        n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(b), ptr(x), flags,
        ptr(workspace), workspace.numel() * 8, int(begin), int(end), ptr(status), int(timeout_ms),
        _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_csr_chain_rows")
    return x


def sptrsv_csr_syncfree(Ap, Ai, Ax, b, x=None, *, upper=False, unit_diag=False, diag_pos=None,
                        exact=False, lanes=0, threads=0, status=None, timeout_ms=0, sync=True):
    """Sync-free CSR triangular solve; returns x (a new tensor unless given)."""
    _require(Ap, torch.int32, "Ap")
    _require(Ai, torch.int32, "Ai")
    _require(Ax, torch.float64, "Ax")
    _require(b, torch.float64, "b")
    n = Ap.numel() - 1
    x = torch.empty(n, dtype=torch.float64, device=b.device) if x is None else x
    status = new_status(b.device) if status is None else status
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, exact)
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_csr_syncfree(
        n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(b), ptr(x), flags,
        int(lanes), int(threads), ptr(status), int(timeout_ms), _stream(),
        ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_csr_syncfree")
    return x


def sptrsv_csr_syncfree_multi(Ap, Ai, Ax, B, X=None, *, upper=False, unit_diag=False,
                              diag_pos=None, status=None, timeout_ms=0, sync=True):
    """Multi-RHS solve on a row-major n x nrhs block (nrhs <= 64)."""
    _require(B, torch.float64, "B")
    n = Ap.numel() - 1
    if B.dim() != 2 or B.shape[0] != n:
        raise ValueError("B must be a row-major n x nrhs tensor")
    nrhs = B.shape[1]
    X = torch.empty_like(B) if X is None else X
    status = new_status(B.device) if status is None else status
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, False)
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_csr_syncfree_multi(
        n, Ai.numel(), nrhs, ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(B), ptr(X), nrhs,
        flags, ptr(status), int(timeout_ms), _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_csr_syncfree_multi")
    return X


def sptrsv_wavefront_multi(Ap, Ai, Ax, B, wavefronts, wavefront_ptr, X=None, *, upper=False,
                           unit_diag=False, diag_pos=None, status=None, timeout_ms=0, sync=True):
    """Level-synchronous multi-RHS solve on a row-major n x nrhs block (nrhs <= 64).
    ``wavefronts`` / ``wavefront_ptr`` come from ``dag_build`` of the matching operator
    (``csr_lower`` or ``csr_upper``)."""
    _require(B, torch.float64, "B")
    n = Ap.numel() - 1
    if B.dim() != 2 or B.shape[0] != n:
        raise ValueError("B must be a row-major n x nrhs tensor")
    nrhs = B.shape[1]
    X = torch.empty_like(B) if X is None else X
    status = new_status(B.device) if status is None else status
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, False)
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_wavefront_multi(
        n, Ai.numel(), nrhs, ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(B), ptr(X), nrhs, flags,
        ptr(wavefronts), ptr(wavefront_ptr), wavefront_ptr.numel() - 1, ptr(status),
        int(timeout_ms), _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_wavefront_multi")
    return X


_side_streams = {}


CHAIN_PIPELINE_PIECES = 16   # measured on the 4,194,304-row benchmark matrix: 28.6 ms in two steps,
                             # 28.3 / 27.7 / 26.9 / 27.7 ms with 4 / 8 / 16 / 32 pieces


CHAIN_PIPELINE_MIN_ROWS = 262144   # a range's launches cost ~0.1 ms: smaller pieces do not pay


def chain_pipeline_bounds(n, pieces=None):
    """Row ranges (in solve order, multiples of 512 rows) of the pipelined chain solve; by
    default up to 16 pieces of at least 262,144 rows."""
    if pieces is None:
        pieces = min(CHAIN_PIPELINE_PIECES, n // CHAIN_PIPELINE_MIN_ROWS)
    step = max(CHAIN_SOLVE_ROWS, -(-n // max(int(pieces), 1) // CHAIN_SOLVE_ROWS) * CHAIN_SOLVE_ROWS)
    return list(range(0, n, step)) + [n]


def side_stream(device):
    """The second stream of a device, for throughput work that runs beside a latency-bound
    kernel on the current stream."""
    key = torch.device(device).index
    side = _side_streams.get(key)
    if side is None:
        side = _side_streams[key] = torch.cuda.Stream(device=device, priority=0)
    return side


def chain_prepare_and_solve(Ap, Ai, Ax, b, workspace, x=None, *, upper=False, unit_diag=False,
                            diag_pos=None, status=None, timeout_ms=0, sync=True, pieces=None):
    """Numeric preparation and solve of the chain solver as one pipelined step.  The solve runs
    on one SM at a time and the preparation is throughput work, so the two overlap: the tiles
    are prepared in ``pieces`` row ranges on a second (low-priority) stream, and the solve of a
    range starts on the current stream as soon as its own tiles are there."""
    n = Ap.numel() - 1
    x = torch.empty(n, dtype=torch.float64, device=b.device) if x is None else x
    status = new_status(b.device) if status is None else status
    bounds = chain_pipeline_bounds(n, pieces)
    if len(bounds) < 3:
        chain_prepare(Ap, Ai, Ax, workspace, upper=upper, unit_diag=unit_diag, diag_pos=diag_pos)
        return sptrsv_csr_chain(Ap, Ai, Ax, b, workspace, x, upper=upper, unit_diag=unit_diag,
                                diag_pos=diag_pos, status=status, timeout_ms=timeout_ms, sync=sync)
    main = torch.cuda.current_stream(b.device)
    side = side_stream(b.device)
    side.wait_stream(main)                      # the inputs are complete
    ready = []
    with torch.cuda.stream(side):
        for begin, end in zip(bounds[:-1], bounds[1:]):
            chain_prepare(Ap, Ai, Ax, workspace, upper=upper, unit_diag=unit_diag, diag_pos=diag_pos,
                          rows=(begin, end))
            event = torch.cuda.Event()
            event.record(side)
            ready.append(event)
    for (begin, end), event in zip(zip(bounds[:-1], bounds[1:]), ready):
        main.wait_event(event)
        sptrsv_csr_chain(Ap, Ai, Ax, b, workspace, x, upper=upper, unit_diag=unit_diag,
                         diag_pos=diag_pos, status=status, timeout_ms=timeout_ms,
                         sync=sync and end == n, rows=(begin, end))
    return x


class OrderedPlan:
    """Per-task records of an ordered solve (structure only): reusable while the pattern, the
    flags and the order stay.  ``levels`` (when known) sizes the window of rows in flight."""

    def __init__(self, order, levels=0):
        _require(order, torch.int32, "order")
        self.order = order
        self.levels = int(levels)
        self.records = torch.empty(order.numel() * 4 + 512, dtype=torch.int32, device=order.device)
        self.key = None          # (Ap, diag_pos, flags) the records were built for

    def window(self, nrhs):
        n = self.order.numel()
        if self.levels <= 0:
            return 0
        # about four average levels, never fewer rows than keep every SM busy
        lanes = 2 if nrhs <= 2 else 4 if nrhs <= 4 else 8 if nrhs <= 32 else 16
        floor = 148 * 8 * (32 // lanes)
        return max(4 * n // self.levels, floor)


def sptrsv_csr_ordered(Ap, Ai, Ax, B, order, X=None, *, upper=False, unit_diag=False,
                       diag_pos=None, row_flags=None, use_flags=False, window_rows=None,
                       status=None, timeout_ms=0, sync=True):
    """Sync-free CSR solve with rows handed out in ``order``: node ids in a topological order
    (``dag_build(...).wavefronts``), or an ``OrderedPlan`` around it that keeps the per-task
    records between calls.  ``B``: a vector of n doubles or a row-major ``n x nrhs`` block
    (nrhs <= 64).  ``use_flags``: per-row ready flags instead of the NaN pre-fill of X;
    ``row_flags`` is the scratch for them (n int32)."""
    _require(B, torch.float64, "B")
    plan = order if isinstance(order, OrderedPlan) else OrderedPlan(order)
    n = Ap.numel() - 1
    if B.dim() == 1:
        nrhs = 1
        if B.numel() != n:
            raise ValueError("B must hold n doubles")
    elif B.dim() == 2 and B.shape[0] == n:
        nrhs = B.shape[1]
    else:
        raise ValueError("B must be a vector of n doubles or a row-major n x nrhs tensor")
    if plan.order.numel() != n:
        raise ValueError("order must list every node once")
    X = torch.empty_like(B) if X is None else X
    status = new_status(B.device) if status is None else status
    use_flags = use_flags or row_flags is not None
    if use_flags and row_flags is None:
        row_flags = torch.empty(max(n, 1), dtype=torch.int32, device=B.device)
    flags = _solve_flags(upper, unit_diag, diag_pos is not None, False)
    key = (Ap.data_ptr(), diag_pos.data_ptr() if diag_pos is not None else 0, flags, n)
    ready = plan.key == key
    window = plan.window(nrhs) if window_rows is None else int(window_rows)
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_csr_ordered(
        n, Ai.numel(), nrhs, ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(B), ptr(X), nrhs, flags,
        ptr(plan.order), ptr(plan.records), 1 if ready else 0, ptr(row_flags) if use_flags else None,
        window, ptr(status), int(timeout_ms), _stream(), ctypes.byref(host) if sync else None)
    plan.key = None
    check(rc, "lcd_sptrsv_csr_ordered")
    plan.key = key
    return X


class SmallPlan:
    """Level-ordered task records of a triangular matrix (structure only, built on the device)
    and the per-solve scratch of the level walk with shared-memory hand-off.  ``blocks`` = 1:
    the one-block solver for small systems.  ``blocks`` > 1: the nodes are cut into that many
    ranges and one thread block walks the tasks of each range level by level (at most one block
    per SM; ``blocks`` = 0 picks a number from the average level width).  A block's tasks of a
    level are padded to whole warps of task slots."""

    def __init__(self, op, Ap, Ai, dag, *, diag_pos=None, unit_diag=False, blocks=1):
        op = _op_code(op)
        _require(Ap, torch.int32, "Ap")
        _require(Ai, torch.int32, "Ai")
        lib = nat.load()
        dev = Ap.device
        n = Ap.numel() - 1
        self.op, self.n = op, n
        flags = _solve_flags(False, unit_diag, diag_pos is not None, False)
        i32 = dict(dtype=torch.int32, device=dev)
        self.n_levels = levels = dag.n_levels
        widths = np.diff(dag.wavefront_ptr_host.astype(np.int64))
        if blocks == 0:
            blocks = sliced_blocks(n, levels, dev)
        self.blocks = blocks = max(1, int(blocks))
        if blocks * (levels + 1) > SLICED_MAX_TABLE:
            raise NativeError(nat.ERR_TOO_LARGE, "SmallPlan",
                              f"{blocks} blocks x {levels} levels: slot table too large")
        # slot table: block b owns the nodes [n b / blocks, n (b + 1) / blocks); its tasks of a
        # level are consecutive in the level's (node-sorted) task list; every such slice is padded
        # to whole warps and the slots are numbered block by block
        if blocks > 1:
            self.cuts = torch.empty(blocks * max(levels, 1), **i32)
            check(lib.lcd_small_level_cuts(n, blocks, levels, ptr(dag.wavefronts), ptr(dag.wavefront_ptr),
                                           ptr(self.cuts), _stream()), "lcd_small_level_cuts")
            cuts = np.empty((blocks + 1, levels), dtype=np.int64)
            cuts[:blocks] = self.cuts.cpu().numpy().reshape(blocks, levels)
            cuts[blocks] = widths
        else:
            self.cuts = None
            cuts = np.stack([np.zeros(levels, dtype=np.int64), widths])
        padded = (np.diff(cuts, axis=0) + 31) // 32 * 32              # blocks x levels
        local = np.zeros((blocks, levels + 1), dtype=np.int64)
        np.cumsum(padded, axis=1, out=local[:, 1:])
        base = np.zeros(blocks + 1, dtype=np.int64)
        np.cumsum(local[:, -1], out=base[1:])
        table = local + base[:-1, None]
        self.n_slots = int(base[-1])
        limit = SMALL_MAX_SLOTS if blocks == 1 else SLICED_MAX_SLOTS
        if self.n_slots > limit:
            raise NativeError(nat.ERR_TOO_LARGE, "SmallPlan",
                              f"{self.n_slots} task slots after padding to whole warps; "
                              f"the level walk serves up to {limit}")
        self.slot_ptr = torch.from_numpy(np.ascontiguousarray(table.astype(np.int32)).reshape(-1)).to(dev)
        m = max(self.n_slots, 1)
        pos = torch.empty(max(n, 1), **i32)
        cursor = torch.empty(m, **i32)
        info_dev = torch.zeros(4, **i32)
        self.status = status = new_status(dev)
        info = (ctypes.c_int32 * 4)()
        check(lib.lcd_small_plan_measure(op, flags, n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(diag_pos),
                                         ptr(dag.wavefronts), ptr(dag.level), ptr(dag.wavefront_ptr),
                                         ptr(self.slot_ptr), ptr(self.cuts), levels, blocks, self.n_slots,
                                         ptr(pos),
                                         ptr(cursor), ptr(info_dev), ptr(status), _stream(),
                                         ctypes.byref(info)), "lcd_small_plan_measure")
        longest, self.max_width = int(info[0]), int(info[1])
        if longest > lib.lcd_small_max_entries():
            raise NativeError(nat.ERR_TOO_LARGE, "SmallPlan",
                              f"a task has {longest} operands; the level walk "
                              f"serves up to {lib.lcd_small_max_entries()}")
        self.entries = 2 if longest <= 2 else (4 if longest <= 4 else 8)
        self.rec_pc = torch.empty(self.entries * m, **i32)
        self.rec_src = torch.empty(self.entries * m, **i32)
        self.row_of = torch.empty(m, **i32)
        self.diag_src = torch.empty(m, **i32)
        far = ctypes.c_int32(0)
        check(lib.lcd_small_plan_fill(op, flags, n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(diag_pos),
                                      ptr(dag.wavefronts), ptr(dag.level), ptr(self.slot_ptr), levels,
                                      blocks, ptr(pos), self.n_slots, self.entries,
                                      ptr(self.rec_pc), ptr(self.rec_src), ptr(self.row_of),
                                      ptr(self.diag_src), ptr(cursor), ptr(info_dev), ptr(status),
                                      _stream(), ctypes.byref(far)), "lcd_small_plan_fill")
        self.far = int(far.value)
        self.scratch, self.scratch_rhs = None, 0
        self.scratch_for(1)

    def scratch_for(self, nrhs):
        """Scratch of the solve (coefficients in slot order, x by position) for ``nrhs``
        right-hand sides; growing it loses the gathered coefficients."""
        if nrhs > self.scratch_rhs:
            need = ctypes.c_int64(0)
            check(nat.load().lcd_small_scratch_bytes_multi(self.n_slots, self.entries, nrhs,
                                                           ctypes.byref(need)),
                  "lcd_small_scratch_bytes_multi")
            self.scratch = torch.empty(need.value, dtype=torch.uint8, device=self.slot_ptr.device)
            self.scratch_rhs = nrhs
            self.gathered = False
        return self.scratch

    @staticmethod
    def serves(n, nnz):
        """Cheap size test before a one-block plan is attempted."""
        return 0 < n <= SMALL_MAX_ROWS and nnz - n <= nat.load().lcd_small_max_entries() * n


SMALL_MAX_ROWS = 1 << 18
SMALL_MAX_SLOTS = 1 << 21
SLICED_MAX_SLOTS = 1 << 27         # slots x 8 operand entries stay below 2^31
SLICED_MAX_TABLE = 1 << 24         # blocks x (levels + 1) entries of the slot table
SLICED_ROWS_PER_SLICE = 64         # average tasks of a slice of a level worth a block of its own


def sliced_blocks(n, levels, device=None):
    """Thread blocks for the shared level walk: one per SM at most, and no more than give every
    block about 64 tasks of an average level."""
    count = ctypes.c_int(0)
    check(nat.load().lcd_device_sm_count(ctypes.byref(count)), "lcd_device_sm_count")
    return int(max(1, min(count.value, n // max(levels, 1) // SLICED_ROWS_PER_SLICE)))


SMALL_MAX_RHS = 16


def sptrsv_small(plan, Ax, b, x=None, *, status=None, timeout_ms=0, sync=False, same_values=False):
    """Level walk of a ``SmallPlan`` (asynchronous on the current stream unless ``sync``).
    ``b``: one right-hand side, or - for a plan with several blocks - a row-major ``n x k`` block
    with k = 1, 2, 4, 8 or 16 (the walk then runs on k interleaved copies of the pattern).
    ``same_values``: Ax holds what the previous solve with this plan had (one matrix, many
    right-hand sides) - its coefficients are not gathered into slot order again."""
    _require(Ax, torch.float64, "Ax")
    if b.dim() == 1:
        _require(b, torch.float64, "b")
        x = torch.empty_like(b) if x is None else x
        nrhs, ld = 1, 1
    else:
        # a row-major block, or columns [c0, c1) of one (leading dimension = its row stride)
        x = torch.empty(b.shape, dtype=b.dtype, device=b.device) if x is None else x
        for name, t in (("b", b), ("x", x)):
            if not (isinstance(t, torch.Tensor) and t.is_cuda and t.dtype == torch.float64 and t.dim() == 2
                    and t.stride(1) == 1 and t.stride(0) >= t.shape[1]):
                raise TypeError(f"{name} must be a row-major float64 CUDA block of right-hand sides")
        if x.shape != b.shape or x.stride() != b.stride():
            raise ValueError("x must have the shape and leading dimension of b")
        nrhs, ld = int(b.shape[1]), int(b.stride(0))
    status = plan.status if status is None else status
    host = ctypes.c_int(0)
    scratch = plan.scratch_for(nrhs)
    gather = not (same_values and plan.gathered)
    check(nat.load().lcd_sptrsv_small_multi(plan.n, plan.n_slots, plan.entries, ptr(Ax), ptr(b), ptr(x),
                                            nrhs, ld, ptr(plan.rec_pc), ptr(plan.rec_src),
                                            ptr(plan.row_of), ptr(plan.diag_src), ptr(plan.slot_ptr),
                                            plan.n_levels, plan.blocks, plan.max_width,
                                            1 if gather else 0, ptr(scratch), scratch.numel(),
                                            ptr(status), int(timeout_ms), _stream(),
                                            ctypes.byref(host) if sync else None),
          "lcd_sptrsv_small_multi")
    plan.gathered = True
    return x


def transpose(src, rows, cols, out=None):
    """out[c, r] = src[r, c] for a row-major rows x cols block."""
    out = torch.empty(cols, rows, dtype=torch.float64, device=src.device) if out is None else out
    check(nat.load().lcd_transpose_f64(rows, cols, ptr(src), cols, ptr(out), rows, _stream()),
          "lcd_transpose_f64")
    return out


def csc_edge_count(Ap, Ai, upper=False):
    n = Ap.numel() - 1
    out = torch.empty(n, dtype=torch.int32, device=Ap.device)
    check(nat.load().lcd_csc_edge_count(n, ptr(Ap), ptr(Ai), nat.SOLVE_UPPER if upper else 0,
                                        ptr(out), _stream()), "lcd_csc_edge_count")
    return out


def sptrsv_csc_syncfree(Ap, Ai, Ax, b, dep_count, x=None, *, upper=False, exact=False, lanes=0,
                        status=None, timeout_ms=0, sync=True):
    """Sync-free CSC solve (push protocol).  ``dep_count`` is consumed."""
    _require(dep_count, torch.int32, "dep_count")
    n = Ap.numel() - 1
    x = torch.empty(n, dtype=torch.float64, device=b.device) if x is None else x
    status = new_status(b.device) if status is None else status
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_csc_syncfree(
        n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(b), ptr(x), ptr(dep_count),
        _solve_flags(upper, False, False, exact), int(lanes), ptr(status), int(timeout_ms),
        _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_csc_syncfree")
    return x


def sptrsv_wavefront(op, Ap, Ai, Ax, b, wavefronts, wavefront_ptr, wavefront_ptr_host=None,
                     x=None, *, mode="cooperative", diag_pos=None, unit_diag=False, exact=False,
                     lanes=1, status=None, timeout_ms=0, sync=True, task_ptr=None):
    """Level-synchronous solve over the level sets of ``dag_build``.  With ``task_ptr`` the
    items of a level are chains of nodes (band chains of ``preprocess_warp_tasks`` with
    ``band_width > 1``): ``wavefronts`` then holds the task nodes, ``wavefront_ptr`` the
    band pointer."""
    op = _op_code(op)
    n = Ap.numel() - 1
    x = torch.empty(n, dtype=torch.float64, device=b.device) if x is None else x
    status = new_status(b.device) if status is None else status
    n_levels = wavefront_ptr.numel() - 1
    mode_code = nat.WAVEFRONT_COOPERATIVE if mode == "cooperative" else nat.WAVEFRONT_PER_LEVEL
    host_ptr = None
    if mode_code == nat.WAVEFRONT_PER_LEVEL:
        if wavefront_ptr_host is None:
            wavefront_ptr_host = wavefront_ptr.cpu().numpy()
        wavefront_ptr_host = np.ascontiguousarray(wavefront_ptr_host, dtype=np.int32)
        host_ptr = wavefront_ptr_host.ctypes.data_as(ctypes.c_void_p)
    flags = _solve_flags(False, unit_diag, diag_pos is not None, exact)
    host = ctypes.c_int(0)
    if task_ptr is None:
        rc = nat.load().lcd_sptrsv_wavefront(
            op, n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(b), ptr(x), flags,
            ptr(wavefronts), ptr(wavefront_ptr), host_ptr, n_levels, mode_code, int(lanes),
            ptr(status), int(timeout_ms), _stream(), ctypes.byref(host) if sync else None)
    else:
        _require(task_ptr, torch.int32, "task_ptr")
        rc = nat.load().lcd_sptrsv_wavefront_tasks(
            op, n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(b), ptr(x), flags,
            ptr(wavefronts), ptr(task_ptr), ptr(wavefront_ptr), host_ptr, n_levels, mode_code,
            int(lanes), ptr(status), int(timeout_ms), _stream(),
            ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_wavefront")
    return x


def spilu0_csr(Ap, Ai, Ax, diag_pos, *, mode="sync_free", wavefronts=None,
               wavefront_ptr_host=None, done=None, lanes=0, status=None, timeout_ms=0, sync=True,
               skip_stored_zeros=False, scratch=None, max_row=None):
    """In-place ILU(0) of a sorted CSR matrix; returns Ax.  ``mode``: "sync_free" (rows by
    index), "ordered" (sync-free, rows in the order of ``wavefronts``) or "wavefront" (a launch
    per level).  ``scratch`` (ordered mode): nnz doubles for the kernel that uses the factor's
    entries as their own ready flags, allocated when None; False selects the flag-based kernel.
    ``max_row`` (longest row, when the caller knows it) picks the lanes per row and skips that
    kernel for rows of more than 64 entries; without it and without ``sync`` a row too long for
    the kernel shows up in ``status`` (A unchanged)."""
    _require(Ax, torch.float64, "Ax")
    _require(diag_pos, torch.int32, "diag_pos")
    n = Ap.numel() - 1
    status = new_status(Ax.device) if status is None else status
    host = ctypes.c_int(0)
    extra = nat.ILU0_SKIP_STORED_ZEROS if skip_stored_zeros else 0   # the column loop's rule
    if mode.replace("-", "_") == "sync_free":
        done = torch.empty(n, dtype=torch.int32, device=Ax.device) if done is None else done
        rc = nat.load().lcd_spilu0_csr(n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), 0 + extra,
                                       ptr(done), None, None, 0, int(lanes), ptr(status),
                                       int(timeout_ms), _stream(),
                                       ctypes.byref(host) if sync else None)
    elif mode == "ordered":
        # sync-free, rows handed out in the order of the level sets
        _require(wavefronts, torch.int32, "wavefronts")
        if (max_row is not None and max_row > 64) or lanes in (1, 2):
            scratch = False
        if scratch is not False:
            # the factor's entries as their own ready flags (rows must fit the lanes' registers)
            if max_row is not None and not lanes:
                lanes = 4 if max_row <= 8 else 8 if max_row <= 16 else 16 if max_row <= 32 else 32
            if scratch is None or scratch.numel() < Ai.numel():
                scratch = torch.empty(max(Ai.numel(), 1), dtype=torch.float64, device=Ax.device)
            rc = nat.load().lcd_spilu0_csr_ordered(
                n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), ptr(wavefronts), ptr(scratch),
                extra, int(lanes), ptr(status), int(timeout_ms), _stream(),
                ctypes.byref(host) if sync else None)
            if rc != nat.ERR_TOO_LARGE and not (sync and host.value == nat.ERR_TOO_LARGE):
                check(rc, "lcd_spilu0_csr_ordered")
                return Ax
        done = torch.empty(n, dtype=torch.int32, device=Ax.device) if done is None else done
        rc = nat.load().lcd_spilu0_csr(n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), 2 + extra,
                                       ptr(done), ptr(wavefronts), None, 0, int(lanes), ptr(status),
                                       int(timeout_ms), _stream(),
                                       ctypes.byref(host) if sync else None)
    else:
        wph = np.ascontiguousarray(wavefront_ptr_host, dtype=np.int32)
        rc = nat.load().lcd_spilu0_csr(n, Ai.numel(), ptr(Ap), ptr(Ai), ptr(Ax), ptr(diag_pos), 1 + extra,
                                       None, ptr(wavefronts), wph.ctypes.data_as(ctypes.c_void_p),
                                       len(wph) - 1, int(lanes), ptr(status), int(timeout_ms),
                                       _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_spilu0_csr")
    return Ax


class CscRowView:
    """Row-ordered view of a CSC pattern: CSR pointers, column indices, diagonal positions and
    ``position`` (place in the column-ordered arrays of the k-th entry in row order)."""

    def __init__(self, ptr_, idx, diag_pos, position):
        self.Ap, self.Ai, self.diag_pos, self.position = ptr_, idx, diag_pos, position


def csc_row_view(Ap, Ai):
    """Build the row-ordered view of a CSC pattern on the device (structure only: once per
    pattern).  Entries of a row come out by ascending column; entries of one position keep
    their storage order."""
    _require(Ap, torch.int32, "Ap")
    _require(Ai, torch.int32, "Ai")
    n = Ap.numel() - 1
    counts = (Ap[1:] - Ap[:-1]).to(torch.int64)
    cols = torch.repeat_interleave(torch.arange(n, device=Ap.device, dtype=torch.int64), counts)
    rows = Ai.to(torch.int64)
    if rows.numel() and (int(rows.min()) < 0 or int(rows.max()) >= n):
        raise nat.NativeError(nat.ERR_INDEX_RANGE, "csc_row_view: row index outside the matrix")
    order = torch.sort(rows * n + cols, stable=True).indices
    ptr_ = torch.zeros(n + 1, dtype=torch.int64, device=Ap.device)
    ptr_[1:] = torch.cumsum(torch.bincount(rows, minlength=n), 0)
    ptr_, idx = ptr_.to(torch.int32), cols[order].to(torch.int32).contiguous()
    return CscRowView(ptr_, idx, diag_positions(ptr_, idx), order.to(torch.int32).contiguous())


def permute(position, values, out=None, *, scatter=False):
    """out[k] = values[position[k]] (gather) or out[position[k]] = values[k] (scatter)."""
    _require(values, torch.float64, "values")
    out = torch.empty_like(values) if out is None else out
    check(nat.load().lcd_permute_f64(position.numel(), ptr(position), ptr(values), ptr(out),
                                     1 if scatter else 0, _stream()), "lcd_permute_f64")
    return out


def spilu0_csc(Ap, Ai, Ax, view=None, *, mode="sync_free", wavefronts=None, wavefront_ptr_host=None,
               lanes=0, status=None, timeout_ms=0):
    """In-place ILU(0) of a matrix stored by columns (the loop of compiler/demo/spilu0.py:50-82);
    returns Ax.  The column loop applies the same updates to the same entries in the same order
    as the row loop, so the values are gathered into row order (``view`` = ``csc_row_view(Ap,
    Ai)``, reusable while the pattern stays), factored by the row kernel and scattered back.
    ``wavefronts`` are level sets of the row view's DAG."""
    _require(Ax, torch.float64, "Ax")
    view = csc_row_view(Ap, Ai) if view is None else view
    by_rows = permute(view.position, Ax)
    spilu0_csr(view.Ap, view.Ai, by_rows, view.diag_pos, mode=mode, wavefronts=wavefronts,
               wavefront_ptr_host=wavefront_ptr_host, lanes=lanes, status=status, timeout_ms=timeout_ms,
               skip_stored_zeros=True)
    return permute(view.position, by_rows, Ax, scatter=True)


_checksum_scratch = {}
_FINGERPRINT_SLOTS = 8


def fingerprints(tensors):
    """Fingerprints of up to eight int32 device tensors with one synchronisation: the checksum
    kernels are queued back to back and their results come back in one copy."""
    tensors = list(tensors)
    if not tensors:
        return []
    if len(tensors) > _FINGERPRINT_SLOTS:
        return [fingerprint(t) for t in tensors]
    device = tensors[0].device
    key = (device, "batch")
    scratch = _checksum_scratch.get(key)
    if scratch is None:
        scratch = _checksum_scratch[key] = torch.zeros(2 * _FINGERPRINT_SLOTS, dtype=torch.int64, device=device)
    lib = nat.load()
    for k, t in enumerate(tensors):
        _require(t, torch.int32, "fingerprint input")
        check(lib.lcd_checksum_i32(ptr(t), t.numel(), ctypes.c_void_p(scratch.data_ptr() + 16 * k), None,
                                   _stream()), "lcd_checksum_i32")
    words = scratch[:2 * len(tensors)].cpu().tolist()       # one copy, one synchronisation
    mask = (1 << 64) - 1
    return [(t.numel(), words[2 * k] & mask, words[2 * k + 1] & mask) for k, t in enumerate(tensors)]


def fingerprint(t):
    """(length, checksum_lo, checksum_hi) of an int32 device tensor."""
    _require(t, torch.int32, "fingerprint input")
    scratch = _checksum_scratch.get(t.device)
    if scratch is None:
        scratch = _checksum_scratch[t.device] = torch.zeros(2, dtype=torch.int64, device=t.device)
    out = (ctypes.c_uint64 * 2)()
    check(nat.load().lcd_checksum_i32(ptr(t), t.numel(), ptr(scratch), ctypes.byref(out),
                                      _stream()), "lcd_checksum_i32")
    return t.numel(), int(out[0]), int(out[1])


def fill_u64(t, value):
    check(nat.load().lcd_fill_u64(ptr(t), t.numel() * t.element_size() // 8, value, _stream()),
          "lcd_fill_u64")
    return t


__all__ = [name for name in dir() if not name.startswith("_")] + ["NativeError"]
