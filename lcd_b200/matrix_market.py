"""Matrix Market ingestion and the regularisation the reference's demos apply.

Mirrors ``compiler/demo/matrix.py:26-81`` (``load_matrix_market``): a square real
coordinate file is read, cut to its leading principal ``max_size`` block, values are
scaled by the largest magnitude, the diagonal is replaced by ``1 + sum |off-diagonal|`` of
its row (strictly dominant, so no zero pivots), indices end up sorted.  Same argument
meaning, same exceptions, same result type (``scipy.sparse.csr_matrix``, float64 values);
the file is parsed here instead of going through ``scipy.io.mmread``.

No matrix collection is shipped: ``matrix_path`` has no default file.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import scipy.sparse as sp

DEFAULT_MAX_N = 128   # leading principal sample the reference's demos use (matrix.py:14)

_FIELDS = ("real", "double", "integer", "pattern", "complex")
_SYMMETRIES = ("general", "symmetric", "skew-symmetric", "hermitian")


class MatrixMarketError(ValueError):
    """The file is not a Matrix Market file this reader understands."""


def read_matrix_market(path):
    """(rows, cols, values, shape) of a coordinate Matrix Market file, symmetric storage
    expanded, indices zero-based.  ``array`` (dense) files raise ``ValueError`` with the
    reference's wording, complex ones too."""
    path = Path(path)
    with open(path, "r") as handle:
        header = handle.readline().split()
        if len(header) != 5 or header[0].lower() != "%%matrixmarket" or header[1].lower() != "matrix":
            raise MatrixMarketError(f"Not a Matrix Market matrix file: {path}")
        layout, field, symmetry = (word.lower() for word in header[2:])
        if field not in _FIELDS or symmetry not in _SYMMETRIES:
            raise MatrixMarketError(f"Unknown Matrix Market qualifiers {field!r} / {symmetry!r}: {path}")
        if layout != "coordinate":
            raise ValueError(f"Expected a sparse Matrix Market input: {path}")
        line = handle.readline()
        while line and (line.startswith("%") or not line.strip()):
            line = handle.readline()
        try:
            n_rows, n_cols, count = (int(word) for word in line.split())
        except ValueError as error:
            raise MatrixMarketError(f"Bad size line in {path}: {line!r}") from error
        tokens = handle.read().split()
    if field == "complex":
        raise ValueError("Complex Matrix Market inputs are not supported yet.")
    width = 2 if field == "pattern" else 3
    if len(tokens) != count * width:
        raise MatrixMarketError(
            f"{path}: expected {count} entries of {width} numbers, found {len(tokens)} numbers")
    table = np.asarray(tokens, dtype=np.float64).reshape(count, width) if count else np.zeros((0, width))
    rows = table[:, 0].astype(np.int64) - 1
    cols = table[:, 1].astype(np.int64) - 1
    values = np.ones(count) if field == "pattern" else table[:, 2].copy()
    if count and (rows.min() < 0 or cols.min() < 0 or rows.max() >= n_rows or cols.max() >= n_cols):
        raise MatrixMarketError(f"{path}: an entry lies outside the {n_rows} x {n_cols} matrix")
    if symmetry != "general":
        off = rows != cols
        mirrored = -values[off] if symmetry == "skew-symmetric" else values[off]
        rows, cols = np.concatenate([rows, cols[off]]), np.concatenate([cols, rows[off]])
        values = np.concatenate([values, mirrored])
    return rows, cols, values, (n_rows, n_cols)


def _combine(rows, cols, values):
    """Sorted by (row, column), repeated positions summed, zeros dropped."""
    order = np.lexsort((cols, rows))
    rows, cols, values = rows[order], cols[order], values[order]
    if len(rows):
        first = np.concatenate([[True], (rows[1:] != rows[:-1]) | (cols[1:] != cols[:-1])])
        starts = np.flatnonzero(first)
        values = np.add.reduceat(values, starts)
        rows, cols = rows[starts], cols[starts]
    keep = values != 0.0
    return rows[keep], cols[keep], values[keep]


def load_matrix_market(matrix_path=None, max_size=DEFAULT_MAX_N):
    """Load and regularise a square real Matrix Market input (see the module docstring).

    ``max_size`` is the size of the leading principal sample, 0 for the whole matrix."""
    if max_size < 0:
        raise ValueError("max_size must be nonnegative.")
    if matrix_path is None:
        raise FileNotFoundError("Matrix Market input not found: no matrix collection is shipped, "
                                "pass a path")
    path = Path(matrix_path).expanduser()
    if not path.is_file():
        raise FileNotFoundError(f"Matrix Market input not found: {path}")
    rows, cols, values, shape = read_matrix_market(path)
    if shape[0] != shape[1]:
        raise ValueError(f"Matrix Market input must be square, got {shape}.")
    size = min(max_size, shape[0]) if max_size else shape[0]
    inside = (rows < size) & (cols < size)
    rows, cols, values = _combine(rows[inside], cols[inside], values[inside])
    if not len(values):
        raise ValueError(f"Matrix Market sample is empty: {path}")
    scale = float(np.max(np.abs(values)))
    if scale:
        values = values / scale
    off = rows != cols
    rows, cols, values = rows[off], cols[off], values[off]
    dominant = np.bincount(rows, weights=np.abs(values), minlength=size) + 1.0
    diagonal = np.arange(size, dtype=np.int64)
    rows, cols, values = _combine(np.concatenate([rows, diagonal]), np.concatenate([cols, diagonal]),
                                  np.concatenate([values, dominant]))
    indptr = np.zeros(size + 1, dtype=np.int32)
    np.cumsum(np.bincount(rows, minlength=size), out=indptr[1:])
    matrix = sp.csr_matrix((values, cols.astype(np.int32), indptr), shape=(size, size))
    matrix.has_sorted_indices = True
    return matrix


def write_matrix_market(path, matrix, symmetric=False, pattern=False, comment=None):
    """Small writer for tests and demos (coordinate, real or pattern, general or symmetric:
    the symmetric form stores the lower triangle)."""
    coo = sp.coo_matrix(matrix)
    rows, cols, values = coo.row, coo.col, coo.data
    if symmetric:
        keep = rows >= cols
        rows, cols, values = rows[keep], cols[keep], values[keep]
    with open(path, "w") as handle:
        handle.write("%%MatrixMarket matrix coordinate "
                     f"{'pattern' if pattern else 'real'} {'symmetric' if symmetric else 'general'}\n")
        if comment:
            handle.write(f"% {comment}\n")
        handle.write(f"{coo.shape[0]} {coo.shape[1]} {len(values)}\n")
        for r, c, v in zip(rows, cols, values):
            handle.write(f"{r + 1} {c + 1}\n" if pattern else f"{r + 1} {c + 1} {float(v)!r}\n")
