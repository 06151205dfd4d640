"""ctypes front end of the CPU oracle (``oracle/lcd_oracle.c``).

TEST INFRASTRUCTURE ONLY.  Imported by ``tests/``, by the smoke check and by the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``; never by the
product package.  Parity status: pinned against fixtures produced by the
reference's own Python pipeline (``tests/golden/``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from dataclasses import dataclass

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liblcd_oracle.so")

CSR_LOWER, CSC_LOWER, ILU0_CSR, CSR_UPPER, CSC_UPPER, CSR_LOWER_ROWS, CSR_UPPER_ROWS = range(7)
KINDS = {"csr_lower": CSR_LOWER, "csc_lower": CSC_LOWER, "ilu0_csr": ILU0_CSR,
         "csr_upper": CSR_UPPER, "csc_upper": CSC_UPPER, "csr_lower_rows": CSR_LOWER_ROWS,
         "csr_upper_rows": CSR_UPPER_ROWS}


def build(force=False):
    """Compile the oracle library next to its source."""
    src = os.path.join(_HERE, "lcd_oracle.c")
    if (force or not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.check_call(["make", "-s", "-C", _HERE, "-B", "liblcd_oracle.so"])
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        _lib.orc_dag_count_edges.restype = ctypes.c_int64
        _lib.orc_residual_csr.restype = ctypes.c_double
    return _lib


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _f64(a):
    return np.ascontiguousarray(a, dtype=np.float64)


@dataclass
class DagArrays:
    dep_count: np.ndarray
    edge_count: np.ndarray
    dag_ptr: np.ndarray
    dag_index: np.ndarray
    level: np.ndarray
    wavefronts: np.ndarray
    wavefront_ptr: np.ndarray
    cyclic: bool


def dag_build(kind, ptr, idx, n=None):
    """All preprocessing arrays of one operator (``kind`` is a key of KINDS)."""
    kind = KINDS[kind] if isinstance(kind, str) else kind
    ptr, idx = _i32(ptr), _i32(idx)
    n = len(ptr) - 1 if n is None else int(n)
    L = lib()
    cap = L.orc_dag_count_edges(kind, n, _p(ptr), _p(idx))
    dep = np.zeros(n, np.int32)
    edge = np.zeros(n, np.int32)
    dag_ptr = np.zeros(n + 1, np.int32)
    dag_index = np.zeros(max(cap, 1), np.int32)
    level = np.zeros(n, np.int32)
    waves = np.zeros(n, np.int32)
    wptr = np.zeros(n + 2, np.int32)
    n_edges = ctypes.c_int64(0)
    n_levels = ctypes.c_int32(0)
    rc = L.orc_dag_build(kind, n, _p(ptr), _p(idx), _p(dep), _p(edge),
                         _p(dag_ptr), _p(dag_index), ctypes.byref(n_edges),
                         _p(level), _p(waves), _p(wptr), ctypes.byref(n_levels))
    return DagArrays(dep, edge, dag_ptr, dag_index[:n_edges.value].copy(), level,
                     waves, wptr[:n_levels.value + 1].copy(), bool(rc))


def diag_positions(ptr, idx):
    ptr, idx = _i32(ptr), _i32(idx)
    n = len(ptr) - 1
    pos = np.full(n, -1, np.int32)
    rc = lib().orc_diag_positions(n, _p(ptr), _p(idx), ctypes.c_int64(len(idx)), _p(pos))
    return pos, rc


def _solve(name, Ap, Ai, Ax, b, extra=()):
    Ap, Ai, Ax, b = _i32(Ap), _i32(Ai), _f64(Ax), _f64(b)
    n = len(Ap) - 1
    x = np.zeros(n)
    args = [n, _p(Ap), _p(Ai), _p(Ax)] + [_p(e) for e in extra] + [_p(b), _p(x)]
    getattr(lib(), name)(*args)
    return x


def sptrsv_csr_lower(Ap, Ai, Ax, b):
    return _solve("orc_sptrsv_csr_lower", Ap, Ai, Ax, b)


def gauss_seidel_simple_csr(Ap, Ai, Ax, D, b, x0, max_iter):
    """Sweeps over strictly lower rows with a separate diagonal; returns the new x."""
    Ap, Ai, Ax, D, b = _i32(Ap), _i32(Ai), _f64(Ax), _f64(D), _f64(b)
    x = np.array(x0, dtype=np.float64)
    lib().orc_gauss_seidel_simple_csr(len(Ap) - 1, _p(Ap), _p(Ai), _p(Ax), _p(D), _p(b), _p(x),
                                      ctypes.c_int32(int(max_iter)))
    return x


def gauss_seidel_full_csr(Ap, Ai, Ax, b, x0, max_iter):
    """Sweeps over lower rows that store their diagonal; returns the new x."""
    Ap, Ai, Ax, b = _i32(Ap), _i32(Ai), _f64(Ax), _f64(b)
    x = np.array(x0, dtype=np.float64)
    lib().orc_gauss_seidel_full_csr(len(Ap) - 1, _p(Ap), _p(Ai), _p(Ax), _p(b), _p(x),
                                    ctypes.c_int32(int(max_iter)))
    return x


def sptrsv_csr_upper(Ap, Ai, Ax, b):
    return _solve("orc_sptrsv_csr_upper", Ap, Ai, Ax, b)


def sptrsv_csc_lower(Ap, Ai, Ax, b):
    return _solve("orc_sptrsv_csc_lower", Ap, Ai, Ax, b)


def sptrsv_csc_upper(Ap, Ai, Ax, b):
    return _solve("orc_sptrsv_csc_upper", Ap, Ai, Ax, b)


def sptrsv_unit_lower_of_full(Ap, Ai, Ax, dpos, b):
    return _solve("orc_sptrsv_csr_unit_lower_of_full", Ap, Ai, Ax, b, (_i32(dpos),))


def sptrsv_upper_of_full(Ap, Ai, Ax, dpos, b):
    return _solve("orc_sptrsv_csr_upper_of_full", Ap, Ai, Ax, b, (_i32(dpos),))


def ilu0_csr(Ap, Ai, Ax, fast=False):
    """Returns the factored copy of Ax (the input is not modified)."""
    Ap, Ai = _i32(Ap), _i32(Ai)
    out = _f64(Ax).copy()
    n = len(Ap) - 1
    if fast:
        dpos, rc = diag_positions(Ap, Ai)
        if rc:
            raise ValueError("ilu0_csr(fast=True) needs sorted rows")
        lib().orc_ilu0_csr_fast(n, _p(Ap), _p(Ai), _p(out), _p(dpos))
    else:
        lib().orc_ilu0_csr(n, _p(Ap), _p(Ai), _p(out))
    return out


def ilu0_csc(Ap, Ai, Ax):
    """ILU0 on CSC storage (compiler/demo/spilu0.py:50-82); returns the factored copy of Ax."""
    Ap, Ai = _i32(Ap), _i32(Ai)
    out = _f64(Ax).copy()
    n = len(Ap) - 1
    work = np.zeros(n + 1 + len(Ai), dtype=np.int32)
    lib().orc_ilu0_csc(n, _p(Ap), _p(Ai), _p(out), _p(work))
    return out


def sptrsv_supernodal(sn, Lip, Li, Lp, Lx, b):
    sn, Lip, Li = _i32(sn), _i32(Lip), _i32(Li)
    Lp = np.ascontiguousarray(Lp, dtype=np.int64)
    Lx = _f64(Lx)
    x = _f64(b).copy()
    ns = len(sn) - 1
    work = np.zeros(int(np.max(np.diff(Lip))) + 1)
    lib().orc_sptrsv_supernodal(ns, _p(sn), _p(Lip), _p(Li), _p(Lp), _p(Lx), _p(x), _p(work))
    return x


def csc_to_supernodal(indptr, indices, data, relaxation=0):
    """Supernodal layout of a lower-triangular CSC matrix: restatement (NumPy, small inputs) of
    the reference's converter, utils/symbolic_cholesky_csc.py:883-921 (column i joins column
    i + 1 when the symmetric difference of their row patterns has at most relaxation + 1
    elements) and :950-1021 (row structure of a supernode = sorted union of its columns'
    patterns; every column stores a value per row of that union, zero where it has none).
    Returns a dict with the reference's keys: x, i, ip, p, supernodes, col_to_super, nSuper,
    max_width."""
    indptr, indices = _i32(indptr), _i32(indices)
    data = _f64(data)
    n = len(indptr) - 1
    pattern = [indices[indptr[j]:indptr[j + 1]] for j in range(n)]
    begins = [0] if n else []
    for j in range(n - 1):
        differ = len(np.setxor1d(pattern[j], pattern[j + 1]))
        if differ > relaxation + 1:
            begins.append(j + 1)
    supernodes = np.asarray(begins + [n], dtype=np.int32)
    n_super = len(begins)
    col_to_super = np.zeros(n, dtype=np.int32)
    rows, ip, p = [], [0], [0]
    for s in range(n_super):
        first, last = supernodes[s], supernodes[s + 1]
        col_to_super[first:last] = s
        union = np.unique(np.concatenate([pattern[j] for j in range(first, last)]))
        rows.append(union)
        ip.append(ip[-1] + len(union))
        for _ in range(first, last):
            p.append(p[-1] + len(union))
    x = np.zeros(p[-1], dtype=np.float64)
    for j in range(n):
        union = rows[col_to_super[j]]
        x[p[j] + np.searchsorted(union, pattern[j])] = data[indptr[j]:indptr[j + 1]]
    return {"x": x, "i": np.concatenate(rows).astype(np.int32) if rows else np.zeros(0, np.int32),
            "ip": np.asarray(ip, dtype=np.int32), "p": np.asarray(p, dtype=np.int64),
            "supernodes": supernodes, "col_to_super": col_to_super, "nSuper": n_super,
            "max_width": int(np.max(np.diff(supernodes))) if n_super else 0}


def relative_residual_csr(Ap, Ai, Ax, x, b):
    """||A x - b||_2 / ||b||_2 for a CSR matrix that stores its diagonal."""
    Ap, Ai, Ax, x, b = _i32(Ap), _i32(Ai), _f64(Ax), _f64(x), _f64(b)
    b2 = ctypes.c_double(0.0)
    r2 = lib().orc_residual_csr(len(Ap) - 1, _p(Ap), _p(Ai), _p(Ax), _p(x), _p(b),
                                ctypes.byref(b2))
    return float(np.sqrt(r2) / np.sqrt(b2.value))
