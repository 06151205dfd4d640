"""Supernodal lower-triangular solve on the reference's supernodal layout.

Layout (``utils/symbolic_cholesky_csc.py:950-1021`` of the reference): supernode
``s`` owns columns ``[sn[s], sn[s+1])``; ``Li[Lip[s]:Lip[s+1]]`` lists its rows,
own columns first; its values form a column-major ``len x width`` panel at
``Lx[Lp[sn[s]]:]`` with leading dimension ``len``.  ``Lp`` is widened to int64.

The solve mirrors ``benchmark/sptrsv_supernodal.py:12-28`` (sequential) and
``:55-94`` (the sync-free CUDA kernel): dense triangular solve of the diagonal
block, panel product, scatter-subtract into ``x``.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _native as nat
from ._native import check, ptr
from .ops import _stream, new_status

MAX_WIDTH = 1024


class SupernodalError(ValueError):
    """The supernodal arrays are inconsistent."""


@dataclass
class SupernodalPlan:
    """Device-resident matrix plus the task list and initial dependency counters."""

    n: int
    n_super: int
    n_tasks: int
    sn: torch.Tensor
    Lip: torch.Tensor
    Li: torch.Tensor
    Lp: torch.Tensor
    Lx: torch.Tensor
    col_to_super: torch.Tensor
    task_super: torch.Tensor
    task_strip: torch.Tensor
    initial_pending: torch.Tensor
    pending: torch.Tensor
    solved: torch.Tensor
    status: torch.Tensor
    panel_values: int
    flops: float
    block_inverses: torch.Tensor | None = None      # inverse diagonal blocks, column-major
    inverse_ptr: torch.Tensor | None = None         # int64 start of each supernode's inverse
    inverse_growth: float = 0.0    # max |inverse entry| x max |diagonal| over the supernodes (the
                                   # inverses are dropped when it exceeds the stability bound)

    @property
    def algorithmic_bytes(self):
        """8 bytes per panel value, 4 per row index, 16 per unknown."""
        return 8 * self.panel_values + 4 * int(self.Li.numel()) + 16 * self.n


def _host(a, dtype):
    if isinstance(a, torch.Tensor):
        a = a.cpu().numpy()
    return np.ascontiguousarray(a, dtype=dtype)


def _level_order(sn_h, Lip_h, Li_h, cts_h, n_super):
    """Supernodes sorted by (level, index), level(t) = 1 + max level of the supernodes whose
    panels have a row in t's columns (``utils/symbolic_cholesky_csc.py:1024-1050`` builds the
    same dependence graph)."""
    if n_super == 0:
        return np.zeros(0, dtype=np.int64)
    width = np.diff(sn_h)
    length = np.diff(Lip_h)
    # off-diagonal rows of every panel -> (source supernode, target supernode), distinct pairs
    positions = np.arange(int(Lip_h[-1]), dtype=np.int64)
    owner = np.repeat(np.arange(n_super, dtype=np.int64), length)
    off = positions - Lip_h[owner] >= width[owner]
    src = owner[off]
    dst = cts_h[Li_h[off]].astype(np.int64)
    keep = dst > src
    pair = np.unique(src[keep] * n_super + dst[keep])
    src, dst = pair // n_super, pair % n_super
    by_target = np.argsort(dst, kind="stable")
    src, dst = src[by_target], dst[by_target]
    start = np.searchsorted(dst, np.arange(n_super + 1))
    level = np.zeros(n_super, dtype=np.int64)
    for t in range(n_super):          # sources have smaller indices: one pass in index order
        a, b = start[t], start[t + 1]
        if b > a:
            level[t] = level[src[a:b]].max() + 1
    return np.lexsort((np.arange(n_super), level))


def analyse(sn, Lip, Li, Lp, Lx, col_to_super=None, n=None, device="cuda", invert_triangles=True):
    """Validate the layout, upload it and build the task list.  With ``invert_triangles`` the
    triangular diagonal block of every supernode is inverted once (numeric: analyse again
    when the values change; 8 * sum(width^2) bytes), which turns the dependent chain of each
    diagonal solve into one pass of independent multiply-adds.

    Host work is O(n_super + n); the per-row counters are accumulated on the
    device.  ``Lx`` may already be a CUDA tensor (it is the large array).
    """
    sn_h = _host(sn, np.int64)
    Lip_h = _host(Lip, np.int64)
    Lp_h = _host(Lp, np.int64)
    n_super = len(sn_h) - 1
    n = int(sn_h[-1]) if n is None else int(n)
    width = np.diff(sn_h)
    length = np.diff(Lip_h)
    if n_super < 0 or len(Lip_h) != n_super + 1 or len(Lp_h) < n + 1:
        raise SupernodalError("sn, Lip and Lp have inconsistent lengths")
    if n_super and (width.min() <= 0 or (length < width).any()):
        raise SupernodalError("every supernode needs width > 0 and at least width rows")
    if n_super and width.max() > MAX_WIDTH:
        raise SupernodalError(f"supernode wider than {MAX_WIDTH} columns")
    if col_to_super is None:
        col_to_super = np.repeat(np.arange(n_super, dtype=np.int32), width)
    strip_rows = nat.load().lcd_supernodal_strip_rows()
    strips = np.maximum(1, -(-(length - width) // strip_rows))
    # Tasks are handed out by ticket; a task whose inputs are not there yet keeps its block
    # waiting.  In index order a supernode often follows one it depends on closely; in level
    # order (a topological order too) the tasks around it in the queue are independent of it.
    order = _level_order(sn_h, Lip_h, _host(Li, np.int32), _host(col_to_super, np.int32), n_super)
    task_super = np.repeat(order.astype(np.int32), strips[order])
    first = np.zeros(n_super + 1, dtype=np.int64)
    np.cumsum(strips[order], out=first[1:])
    task_strip = (np.arange(int(first[-1]), dtype=np.int64) - np.repeat(first[:-1], strips[order]))
    dev = torch.device(device)

    def up(a, dtype):
        if isinstance(a, torch.Tensor) and a.is_cuda:
            kind = {np.int32: torch.int32, np.int64: torch.int64, np.float64: torch.float64}[dtype]
            return a.to(kind).contiguous()
        return torch.from_numpy(_host(a, dtype)).to(dev)

    t_sn, t_Lip = up(sn_h, np.int32), up(Lip_h, np.int32)
    t_Li = up(Li, np.int32)
    t_Lp = up(Lp_h, np.int64)
    t_Lx = Lx if isinstance(Lx, torch.Tensor) and Lx.is_cuda else up(Lx, np.float64)
    t_cts = up(col_to_super, np.int32)
    if t_Li.numel() != int(Lip_h[-1]):
        raise SupernodalError("Li does not match Lip")
    if t_Li.numel() and (int(t_Li.min()) < 0 or int(t_Li.max()) >= n):
        raise SupernodalError("row index out of range")
    pending = torch.empty(n_super, dtype=torch.int32, device=dev)
    check(nat.load().lcd_supernodal_pending(n_super, ptr(t_sn), ptr(t_Lip), ptr(t_Li), ptr(t_cts),
                                            ptr(pending), _stream()), "lcd_supernodal_pending")
    panel_values = int((width * length).sum())
    flops = float((width * width + 2 * width * (length - width)).sum())
    inv = inv_ptr = None
    inverse_growth = 0.0
    if invert_triangles and n_super:
        starts = np.zeros(n_super + 1, dtype=np.int64)
        np.cumsum(width * width, out=starts[1:])
        inv_ptr = up(starts, np.int64)
        inv = torch.empty(int(starts[-1]), dtype=torch.float64, device=dev)
        growth = torch.zeros(1, dtype=torch.float64, device=dev)
        check(nat.load().lcd_supernodal_prepare(n_super, ptr(t_sn), ptr(t_Lip), ptr(t_Lp), ptr(t_Lx),
                                                ptr(inv_ptr), ptr(inv), ptr(growth), _stream()),
              "lcd_supernodal_prepare")
        inverse_growth = float(growth.item())
        if not inverse_growth <= nat.CHAIN_MAX_GROWTH:
            # ill-conditioned diagonal blocks: substitution keeps the digits an explicit
            # inverse would lose
            inv = inv_ptr = None
    return SupernodalPlan(
        n=n, n_super=n_super, n_tasks=int(first[-1]), sn=t_sn, Lip=t_Lip, Li=t_Li, Lp=t_Lp,
        Lx=t_Lx, col_to_super=t_cts, task_super=up(task_super, np.int32),
        task_strip=up(task_strip, np.int32), initial_pending=pending,
        pending=torch.empty_like(pending),
        solved=torch.empty(max(n, 1), dtype=torch.float64, device=dev), status=new_status(dev),
        panel_values=panel_values, flops=flops, block_inverses=inv, inverse_ptr=inv_ptr,
        inverse_growth=inverse_growth)


def solve(plan: SupernodalPlan, b, x=None, timeout_ms=0, sync=True):
    """x = L^{-1} b.  ``b`` is a CUDA float64 tensor; x is returned (device)."""
    if x is None:
        x = torch.empty_like(b)
    x.copy_(b)
    plan.pending.copy_(plan.initial_pending)
    host = ctypes.c_int(0)
    rc = nat.load().lcd_sptrsv_supernodal(
        plan.n, plan.n_super, plan.n_tasks, ptr(plan.task_super), ptr(plan.task_strip),
        ptr(plan.sn), ptr(plan.Lip), ptr(plan.Li), ptr(plan.Lp), ptr(plan.Lx),
        ptr(plan.col_to_super), ptr(plan.pending), ptr(plan.solved), ptr(x),
        ptr(plan.inverse_ptr), ptr(plan.block_inverses), ptr(plan.status),
        int(timeout_ms), _stream(), ctypes.byref(host) if sync else None)
    check(rc, "lcd_sptrsv_supernodal")
    return x


def sptrsv_csc_supernodal(sn_begin, col_to_sup, Lip, Li, Lp, Lx, x, flag_thread=None,
                          max_width=None):
    """Drop-in for ``sptrsv_csc_supernodal_numba_cuda`` of the reference
    (``benchmark/sptrsv_supernodal.py:89-94``): solves in place on ``x`` (which
    holds the right-hand side).  ``flag_thread`` / ``max_width`` are accepted for
    signature compatibility; the counters are recomputed on the device."""
    plan = analyse(sn_begin, Lip, Li, Lp, Lx, col_to_sup, n=len(x))
    if isinstance(x, torch.Tensor) and x.is_cuda:
        b = x.clone()
        solve(plan, b, x)
        return x
    xd = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float64)).to(plan.Lx.device)
    out = solve(plan, xd).cpu().numpy()
    x[...] = out
    return x


@dataclass
class SupernodalLayout:
    """Supernodal arrays of a CSC matrix as device tensors (the reference's ``Ls`` dictionary of
    ``convert_csc_to_supernodal``: ``sn`` = 'supernodes', ``Li`` = 'i', ``Lip`` = 'ip', ``Lp`` =
    'p' widened to int64, ``Lx`` = 'x')."""

    n: int
    n_super: int
    max_width: int
    sn: torch.Tensor
    Lip: torch.Tensor
    Li: torch.Tensor
    Lp: torch.Tensor
    Lx: torch.Tensor
    col_to_super: torch.Tensor

    def fill(self, Cp, Ci, Cx, status=None):
        """New values of the same pattern into the same panels."""
        status = new_status(Cx.device) if status is None else status
        host = ctypes.c_int(0)
        check(nat.load().lcd_supernodal_fill(
            self.n, Ci.numel(), ptr(Cp), ptr(Ci), ptr(Cx), ptr(self.col_to_super), ptr(self.Lip),
            ptr(self.Li), ptr(self.Lp), ptr(self.Lx), self.Lx.numel(), ptr(status), _stream(),
            ctypes.byref(host)), "lcd_supernodal_fill")
        return self


def from_csc(Cp, Ci, Cx, relaxation=0, device="cuda"):
    """Supernodal layout of a lower-triangular matrix stored by columns with sorted rows
    (``convert_csc_to_supernodal(L, relaxation)`` of the reference,
    utils/symbolic_cholesky_csc.py:950-1021), built on the device.  Arguments may be NumPy arrays
    or device tensors; returns a ``SupernodalLayout`` whose fields feed ``analyse``."""
    dev = torch.device(device)

    def up(a, dtype):
        if isinstance(a, torch.Tensor):
            return a.to(device=dev, dtype=dtype).contiguous()
        return torch.from_numpy(np.ascontiguousarray(a, dtype={torch.int32: np.int32,
                                                               torch.float64: np.float64}[dtype])).to(dev)
    Cp, Ci, Cx = up(Cp, torch.int32), up(Ci, torch.int32), up(Cx, torch.float64)
    n, nnz = Cp.numel() - 1, Ci.numel()
    if n < 0 or Cx.numel() != nnz:
        raise SupernodalError("indptr, indices and data have inconsistent lengths")
    need = ctypes.c_int64(0)
    check(nat.load().lcd_supernodal_layout_workspace_bytes(n, nnz, ctypes.byref(need)),
          "lcd_supernodal_layout_workspace_bytes")
    workspace = torch.empty(need.value, dtype=torch.uint8, device=dev)
    col_to_super = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    begin = torch.empty(n + 1, dtype=torch.int32, device=dev)
    Lip = torch.empty(n + 1, dtype=torch.int32, device=dev)
    Li = torch.empty(max(nnz, 1), dtype=torch.int32, device=dev)
    Lp = torch.empty(n + 1, dtype=torch.int64, device=dev)
    summary = (ctypes.c_int64 * 4)()
    check(nat.load().lcd_supernodal_layout(
        n, nnz, ptr(Cp), ptr(Ci), int(relaxation), ptr(col_to_super), ptr(begin), ptr(Lip), ptr(Li),
        ptr(Lp), summary, ptr(workspace), workspace.numel(), _stream()), "lcd_supernodal_layout")
    n_super, n_rows, max_width, panel_values = (int(v) for v in summary)
    layout = SupernodalLayout(
        n=n, n_super=n_super, max_width=max_width, sn=begin[:n_super + 1].clone(),
        Lip=Lip[:n_super + 1].clone(), Li=Li[:n_rows].clone(), Lp=Lp,
        Lx=torch.empty(max(panel_values, 1), dtype=torch.float64, device=dev)[:panel_values],
        col_to_super=col_to_super[:n])
    return layout.fill(Cp, Ci, Cx)
