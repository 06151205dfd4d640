"""Seeded synthetic inputs with the shapes of the benchmark configurations.

The reference evaluates on SuiteSparse matrices that it does not ship
(``matrix_list.txt``, ``compiler/demo/matrix.py:11-13``); these generators are the
stand-ins.  Every generator is a pure function of its arguments and a seed
(``numpy.random.default_rng``), returns ``int32`` index arrays and ``float64``
values, and keeps indices sorted inside each row / column.

Storage conventions required by the operators being served
(``compiler/demo/sptrsv.py:26-43``):

* lower-triangular CSR keeps the diagonal **last** in each row,
* lower-triangular CSC keeps the diagonal **first** in each column,
* upper-triangular CSR keeps the diagonal **first**, CSC keeps it **last**.

With sorted indices all four follow from the triangle itself.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import scipy.sparse as sp


@dataclass
class Triangular:
    """A triangular matrix in both compressed layouts plus a right-hand side."""

    n: int
    csr: sp.csr_matrix
    b: np.ndarray

    @property
    def nnz(self):
        return int(self.csr.nnz)

    def csr_arrays(self):
        m = self.csr
        return (m.indptr.astype(np.int32), m.indices.astype(np.int32),
                m.data.astype(np.float64))

    def csc_arrays(self):
        m = sp.csc_matrix(self.csr)
        m.sort_indices()
        return (m.indptr.astype(np.int32), m.indices.astype(np.int32),
                m.data.astype(np.float64))


def _rhs(n, rng, nrhs=None):
    if nrhs is None:
        return rng.uniform(-1.0, 1.0, n)
    # column-major n x nrhs block of right-hand sides
    return np.asfortranarray(rng.uniform(-1.0, 1.0, (n, nrhs)))


def _tridiag(g, lo, d, up):
    return sp.diags([lo, d, up], [-1, 0, 1], shape=(g, g), format="csr")


def laplacian2d_tril(g=256, seed=0):
    """Lower triangle of the 2-D 5-point Laplacian on a g x g grid.

    Diagonal 4.0, off-diagonals -1.0; n = g*g, about 3 entries per row.
    """
    rng = np.random.default_rng(seed)
    eye = sp.identity(g, format="csr")
    full = sp.kron(eye, _tridiag(g, -1.0, 4.0, -1.0)) + sp.kron(
        _tridiag(g, -1.0, 0.0, -1.0), eye)
    lower = sp.tril(full, format="csr")
    lower.sort_indices()
    n = g * g
    return Triangular(n, lower, _rhs(n, rng))


def laplacian3d(g, seed=0, perturb=0.0):
    """Full 3-D 7-point Laplacian (CSR, sorted).  Diagonal 6.0; every stored
    off-diagonal is ``-1 + U[-perturb, perturb]`` drawn independently, so the
    perturbed matrix is structurally symmetric but not numerically symmetric."""
    rng = np.random.default_rng(seed)
    n = g * g * g
    idx = np.arange(n, dtype=np.int64)
    x = idx % g
    y = (idx // g) % g
    z = idx // (g * g)
    rows, cols = [idx], [idx]
    for cond, off in ((z > 0, -g * g), (y > 0, -g), (x > 0, -1),
                      (x < g - 1, 1), (y < g - 1, g), (z < g - 1, g * g)):
        rows.append(idx[cond])
        cols.append(idx[cond] + off)
    rows = np.concatenate(rows)
    cols = np.concatenate(cols)
    vals = np.full(rows.shape, -1.0)
    vals[:n] = 6.0
    mat = sp.csr_matrix((vals, (rows, cols)), shape=(n, n))
    mat.sort_indices()
    if perturb:
        off = mat.data != 6.0
        mat.data[off] += rng.uniform(-perturb, perturb, int(off.sum()))
    return mat, rng


def laplacian3d_ilu0(g=128, seed=0):
    """Input of the ILU0 configuration: perturbed 3-D Laplacian and a RHS."""
    mat, rng = laplacian3d(g, seed, perturb=0.05)
    b = rng.uniform(-1.0, 1.0, mat.shape[0])
    return mat, b


def laplacian3d_tril(g, seed=0, nrhs=None):
    """Lower triangle of the unperturbed 3-D Laplacian with 1 or nrhs RHS."""
    mat, rng = laplacian3d(g, seed, perturb=0.0)
    lower = sp.tril(mat, format="csr")
    lower.sort_indices()
    n = lower.shape[0]
    return Triangular(n, lower, _rhs(n, rng, nrhs))


_BAND_CHUNK_ROWS = 131072


def _band_chunk(args):
    """Rows [r0, r1) of the random banded matrix: (counts, cols, vals, absum)."""
    seed, chunk, r0, r1, mean_degree, band = args
    rng = np.random.default_rng([seed, chunk])
    m = r1 - r0
    rows_all = np.arange(r0, r1, dtype=np.int64)
    k = np.minimum(rng.poisson(mean_degree, m), rows_all)
    rows = np.repeat(rows_all, k)
    total = rows.shape[0]
    near = rng.random(total) < 0.5
    lo = np.where(near, np.maximum(rows - band, 0), 0)
    cols = lo + (rng.random(total) * (rows - lo)).astype(np.int64)
    np.minimum(cols, rows - 1, out=cols)
    key = (rows - r0) * np.int64(r1) + cols      # cols < r1
    key.sort()
    if total:
        keep = np.empty(total, dtype=bool)
        keep[0] = True
        np.not_equal(key[1:], key[:-1], out=keep[1:])
        key = key[keep]
    local = key // r1
    cols = (key - local * r1).astype(np.int32)
    vals = rng.uniform(-1.0, 1.0, cols.shape[0]) / 16.0
    counts = np.bincount(local, minlength=m).astype(np.int64)
    absum = np.bincount(local, weights=np.abs(vals), minlength=m)
    return counts, local.astype(np.int32), cols, vals, absum


def random_band_lower(n=4_194_304, seed=0, mean_degree=15.0, band=64, workers=None):
    """Random lower-triangular CSR matrix of the sync-free/wavefront configuration.

    Row i draws ``k = min(Poisson(mean_degree), i)`` strictly-lower columns:
    each with probability 1/2 uniform in ``[max(0, i-band), i)`` and otherwise
    uniform in ``[0, i)``; duplicates are removed.  Off-diagonal values are
    ``U[-1,1]/16``, the diagonal is ``1 + sum |offdiag|`` and is stored last.
    Rows are generated in fixed blocks of 131072 with one random stream per
    block, so the result does not depend on the number of worker threads.
    """
    from concurrent.futures import ThreadPoolExecutor
    import os
    jobs = [(seed, c, r0, min(r0 + _BAND_CHUNK_ROWS, n), mean_degree, band)
            for c, r0 in enumerate(range(0, n, _BAND_CHUNK_ROWS))]
    workers = workers or min(len(jobs), os.cpu_count() or 1)
    if workers > 1:
        with ThreadPoolExecutor(workers) as pool:
            parts = list(pool.map(_band_chunk, jobs))
    else:
        parts = [_band_chunk(j) for j in jobs]
    counts = np.concatenate([p[0] for p in parts])
    indptr = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(counts + 1, out=indptr[1:])
    nnz = int(indptr[-1])
    indices = np.empty(nnz, dtype=np.int32)
    data = np.empty(nnz, dtype=np.float64)
    for (seed_, c, r0, r1, _, _), (cnt, local, cols, vals, absum) in zip(jobs, parts):
        base = int(indptr[r0])
        # entry e of local row l lands at base + e + l (one diagonal slot per earlier row)
        dst = base + np.arange(cols.shape[0], dtype=np.int64) + local
        indices[dst] = cols
        data[dst] = vals
        dpos = indptr[r0 + 1:r1 + 1] - 1
        indices[dpos] = np.arange(r0, r1, dtype=np.int32)
        data[dpos] = 1.0 + absum
    mat = sp.csr_matrix((data, indices, indptr.astype(np.int32)), shape=(n, n))
    mat.has_sorted_indices = True
    b = np.random.default_rng([seed, 1 << 30]).uniform(-1.0, 1.0, n)
    return Triangular(n, mat, b)


@dataclass
class Supernodal:
    """Block lower-triangular matrix in the reference's supernodal layout
    (``utils/symbolic_cholesky_csc.py:1008-1017``): supernode s owns columns
    ``[sn[s], sn[s+1])``; its row list is ``Li[Lip[s]:Lip[s+1]]`` (its own
    columns first); its values are a column-major ``len x width`` panel starting
    at ``Lx[Lp[sn[s]]]`` with leading dimension ``len``.  ``Lp`` is int64."""

    n: int
    sn: np.ndarray
    Lip: np.ndarray
    Li: np.ndarray
    Lp: np.ndarray
    Lx: np.ndarray
    col_to_super: np.ndarray
    b: np.ndarray

    @property
    def n_super(self):
        return len(self.sn) - 1

    def to_csc(self):
        """Expand to an ordinary CSC lower-triangular matrix (explicit zeros of
        the strict upper part of each diagonal block are dropped)."""
        rows, cols, vals = [], [], []
        for s in range(self.n_super):
            c0, c1 = int(self.sn[s]), int(self.sn[s + 1])
            r = self.Li[self.Lip[s]:self.Lip[s + 1]].astype(np.int64)
            ln = len(r)
            for c in range(c0, c1):
                col = self.Lx[self.Lp[c]:self.Lp[c] + ln]
                keep = r >= c
                rows.append(r[keep])
                cols.append(np.full(int(keep.sum()), c, dtype=np.int64))
                vals.append(col[keep])
        mat = sp.csc_matrix((np.concatenate(vals),
                             (np.concatenate(rows), np.concatenate(cols))),
                            shape=(self.n, self.n))
        mat.sort_indices()
        return mat


def supernodal_random(n=1_048_576, seed=0, widths=(16, 32, 64, 128),
                      min_targets=8, max_targets=32):
    """Block lower-triangular matrix of the supernodal configuration.

    Supernode widths are i.i.d. from ``widths`` until n is covered (last one
    clipped).  Diagonal blocks are dense lower triangular (diagonal
    ``2 + U[0,1]``, strict lower ``U[-0.1, 0.1]``, strict upper stored as
    zeros).  The off-diagonal panel of a supernode covers the full column
    ranges of ``k ~ UniformInt[min_targets, max_targets]`` distinct later
    supernodes (fewer near the end), entries ``U[-0.1, 0.1]``.
    """
    rng = np.random.default_rng(seed)
    draws = rng.choice(np.asarray(widths), size=n // min(widths) + 1)
    ends = np.cumsum(draws)
    n_super = int(np.searchsorted(ends, n)) + 1
    sn = np.zeros(n_super + 1, dtype=np.int64)
    sn[1:] = np.minimum(ends[:n_super], n)
    width = np.diff(sn)
    col_to_super = np.repeat(np.arange(n_super, dtype=np.int32), width)
    targets = []
    lens = np.zeros(n_super, dtype=np.int64)
    for s in range(n_super):
        later = n_super - 1 - s
        k = min(int(rng.integers(min_targets, max_targets + 1)), later)
        t = (np.sort(rng.choice(later, size=k, replace=False)) + s + 1
             if k else np.zeros(0, dtype=np.int64))
        targets.append(t)
        lens[s] = width[s] + int(width[t].sum()) if k else width[s]
    Lip = np.zeros(n_super + 1, dtype=np.int64)
    np.cumsum(lens, out=Lip[1:])
    Li = np.empty(int(Lip[-1]), dtype=np.int32)
    Lp = np.zeros(n + 1, dtype=np.int64)
    np.cumsum(np.repeat(lens, width), out=Lp[1:])
    Lx = np.empty(int(Lp[-1]), dtype=np.float64)
    for s in range(n_super):
        w, ln = int(width[s]), int(lens[s])
        c0 = int(sn[s])
        rows = [np.arange(c0, c0 + w)]
        rows += [np.arange(sn[t], sn[t + 1]) for t in targets[s]]
        Li[Lip[s]:Lip[s + 1]] = np.concatenate(rows)
        panel = rng.uniform(-0.1, 0.1, (w, ln))  # panel[c, r]: column-major
        top = panel[:, :w]
        top[np.triu_indices(w, 1)[::-1]] = 0.0  # (col, row) with row < col
        top[np.arange(w), np.arange(w)] = 2.0 + rng.uniform(0.0, 1.0, w)
        Lx[Lp[c0]:Lp[c0] + w * ln] = panel.ravel()
    b = rng.uniform(-1.0, 1.0, n)
    return Supernodal(n, sn.astype(np.int32), Lip.astype(np.int32), Li, Lp, Lx,
                      col_to_super, b)


def upper_from_lower(tri: Triangular):
    """Transpose of a lower-triangular system: an upper-triangular CSR matrix
    (diagonal first in each row) with the same right-hand side."""
    up = sp.csr_matrix(tri.csr.T)
    up.sort_indices()
    return Triangular(tri.n, up, tri.b)
