"""Executable demos on a Matrix Market input, as the reference ships them.

One module for what the reference spreads over ``compiler/demo/sptrsv.py:45-107``,
``compiler/demo/spilu0.py:117-211`` and ``compiler/demo/gauss_seidel.py:70-170``: the
decorated operators of those files (same loop nests, decorated with
:func:`lcd_b200.decorator.parallel`) and a ``run_*`` function each that loads the matrix with
:func:`lcd_b200.matrix_market.load_matrix_market`, runs the operators on the GPU and prints
the largest deviation from the sequential result.

    python -m lcd_b200.demos sptrsv       matrix.mtx [--max-n 128] [--storage csr|csc|both]
    python -m lcd_b200.demos spilu0       matrix.mtx [--execution-mode wavefront|sync_free] [--storage csr|csc|both]
    python -m lcd_b200.demos gauss-seidel matrix.mtx [--variant simple|full|both] [--iterations 2]

ILU0 in CSC form (``compiler/demo/spilu0.py:50-82``) runs on the row kernels through the
row-ordered view of the pattern (same updates in the same order: bit-identical values).
"""

from __future__ import annotations

import argparse

import numpy as np
import scipy.sparse as sp
from scipy.sparse.linalg import spsolve_triangular

from .decorator import parallel
from .matrix_market import DEFAULT_MAX_N, load_matrix_market

PROPS_CSR = {"Ap": ["monotonically_increasing"], "Ai": []}
PROPS_CSC = {"Ap": ["monotonically_increasing"], "Ai": [], ("Ap", "Ai"): ["triangularity"]}
PROPS_ILU0 = {"A_indptr": ["monotonically_increasing"], "A_indices": [],
              ("A_indptr", "A_indices"): [("segmented_monotonically_increasing", "n")]}


@parallel(block_map="i", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def simple_sptrsv_csr(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(block_map="i", function_props=PROPS_CSC, execution_mode="wavefront", threads_per_block=128)
def simple_sptrsv_csc(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


def ilu0_csr(A_data, A_indices, A_indptr):
    n = len(A_indptr) - 1
    for i in range(n):
        row_start = A_indptr[i]
        row_end = A_indptr[i + 1]
        for k_ptr in range(row_start, row_end):
            k = A_indices[k_ptr]
            if k >= i:
                break
            diag_val = 0.0
            for diag_ptr in range(A_indptr[k], A_indptr[k + 1]):
                if A_indices[diag_ptr] == k:
                    diag_val = A_data[diag_ptr]
                    break
            if diag_val != 0.0:
                A_data[k_ptr] = A_data[k_ptr] / diag_val
                l_ik = A_data[k_ptr]
                for j_ptr in range(k_ptr + 1, row_end):
                    j = A_indices[j_ptr]
                    for kj_ptr in range(A_indptr[k], A_indptr[k + 1]):
                        if A_indices[kj_ptr] == j:
                            u_kj = A_data[kj_ptr]
                            A_data[j_ptr] = A_data[j_ptr] - l_ik * u_kj
                            break
    return A_data


def ilu0_csc(A_data, A_indices, A_indptr):
    n = len(A_indptr) - 1
    for k in range(n):
        col_start = A_indptr[k]
        col_end = A_indptr[k + 1]
        diag_val = 0.0
        for dptr in range(col_start, col_end):
            if A_indices[dptr] == k:
                diag_val = A_data[dptr]
                break
        for i_ptr in range(col_start, col_end):
            i = A_indices[i_ptr]
            if i <= k:
                continue
            if diag_val != 0.0:
                A_data[i_ptr] = A_data[i_ptr] / diag_val
                l_ik = A_data[i_ptr]
                for j in range(k + 1, n):
                    j_start = A_indptr[j]
                    j_end = A_indptr[j + 1]
                    u_kj = 0.0
                    for kj_ptr in range(j_start, j_end):
                        if A_indices[kj_ptr] == k:
                            u_kj = A_data[kj_ptr]
                            break
                    if u_kj != 0.0:
                        for ij_ptr in range(j_start, j_end):
                            if A_indices[ij_ptr] == i:
                                A_data[ij_ptr] = A_data[ij_ptr] - l_ik * u_kj
                                break
    return A_data


def compile_ilu0_csc(execution_mode="wavefront", threads_per_block=128):
    """CSC ILU0 with the requested executor settings, as ``compiler/demo/spilu0.py:101-108``."""
    return parallel(block_map="k", function_props=PROPS_ILU0, execution_mode=execution_mode,
                    threads_per_block=threads_per_block)(ilu0_csc)


def compile_ilu0_csr(execution_mode="wavefront", threads_per_block=128, thread_unroll=None):
    """CSR ILU0 with the requested executor settings (the unroll factor is scheduled unless
    given), as ``compiler/demo/spilu0.py:85-99``."""
    return parallel(block_map="i", thread_map="j_ptr", function_props=PROPS_ILU0,
                    execution_mode=execution_mode, threads_per_block=threads_per_block,
                    thread_unroll=thread_unroll)(ilu0_csr)


@parallel(block_map="i", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def simple_gauss_seidel_csr(Ap, Ai, Ax, D, b, x, n, max_iter):
    for sweep in range(max_iter):
        for i in range(n):
            x[i] = b[i]
            for j in range(Ap[i], Ap[i + 1]):
                x[i] -= Ax[j] * x[Ai[j]]
            x[i] /= D[i]
    return x


@parallel(block_map="i", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def full_gauss_seidel_csr(Ap, Ai, Ax, b, x, n, max_iter):
    for sweep in range(max_iter):
        for i in range(n):
            sigma = 0.0
            diag = 1.0
            for j in range(Ap[i], Ap[i + 1]):
                if Ai[j] == i:
                    diag = Ax[j]
                else:
                    sigma += Ax[j] * x[Ai[j]]
            x[i] = (b[i] - sigma) / diag
    return x


def _triangle(source, strict=False):
    lower = sp.tril(source, k=-1 if strict else 0, format="csr")
    lower.sort_indices()
    return lower


def _arrays(matrix):
    return matrix.indptr.astype(np.int32), matrix.indices.astype(np.int32), matrix.data.copy()


def run_sptrsv(matrix_path, max_size=DEFAULT_MAX_N, storage="both"):
    """Lower-triangular solves in CSR and/or CSC form against SciPy."""
    lower = _triangle(load_matrix_market(matrix_path, max_size))
    n = lower.shape[0]
    rhs = np.asarray(lower @ np.linspace(1.0, 2.0, n)).ravel()
    results = {}
    for name in (("csr", "csc") if storage == "both" else (storage,)):
        matrix = sp.csr_matrix(lower) if name == "csr" else sp.csc_matrix(lower)
        matrix.sort_indices()
        solver = simple_sptrsv_csr if name == "csr" else simple_sptrsv_csc
        results[name] = solver(*_arrays(matrix), rhs, n)
        error = float(np.max(np.abs(results[name] - spsolve_triangular(matrix, rhs, lower=True))))
        print(f"SpTRSV {name.upper()}: n={n}, nnz={matrix.nnz}, max_abs_error={error:.3e}")
    return results


def run_spilu0(matrix_path, max_size=DEFAULT_MAX_N, execution_mode="wavefront",
               threads_per_block=128, thread_unroll=None, storage="csr"):
    """In-place ILU(0) of the regularised matrix (CSR and/or CSC storage) against the sequential
    loops."""
    source = load_matrix_market(matrix_path, max_size)
    results = {}
    for name in (("csr", "csc") if storage == "both" else (storage,)):
        matrix = sp.csr_matrix(source) if name == "csr" else sp.csc_matrix(source)
        matrix.sort_indices()
        indptr, indices, data = _arrays(matrix)
        if name == "csr":
            factor, loop = compile_ilu0_csr(execution_mode, threads_per_block, thread_unroll), ilu0_csr
        else:
            factor, loop = compile_ilu0_csc(execution_mode, threads_per_block), ilu0_csc
        results[name] = factor(data.copy(), indices, indptr)
        error = float(np.max(np.abs(results[name] - loop(data.copy(), indices, indptr))))
        schedule = factor.current_schedule
        print(f"ILU0 {name.upper()}: n={matrix.shape[0]}, nnz={matrix.nnz}, mode={schedule.execution_mode}, "
              f"threads={schedule.threads_per_block}, unroll={schedule.thread_unroll}, "
              f"max_abs_error={error:.3e}")
    return results


def run_gauss_seidel(matrix_path, max_size=DEFAULT_MAX_N, variant="both", iterations=2):
    """Gauss-Seidel sweeps over the lower triangle against the undecorated loops."""
    source = load_matrix_market(matrix_path, max_size)
    full, strict = _triangle(source), _triangle(source, strict=True)
    n = source.shape[0]
    rhs = np.asarray(full @ np.linspace(1.0, 2.0, n)).ravel()
    results = {}
    if variant in ("simple", "both"):
        args = (*_arrays(strict), source.diagonal().copy(), rhs)
        results["simple"] = simple_gauss_seidel_csr(*args, np.zeros(n), n, iterations)
        want = simple_gauss_seidel_csr.original_function(*args, np.zeros(n), n, iterations)
        print(f"Gauss-Seidel simple CSR: n={n}, nnz={strict.nnz}, sweeps={iterations}, "
              f"max_abs_error={float(np.max(np.abs(results['simple'] - want))):.3e}")
    if variant in ("full", "both"):
        args = (*_arrays(full), rhs)
        results["full"] = full_gauss_seidel_csr(*args, np.zeros(n), n, iterations)
        want = full_gauss_seidel_csr.original_function(*args, np.zeros(n), n, iterations)
        print(f"Gauss-Seidel full CSR: n={n}, nnz={full.nnz}, sweeps={iterations}, "
              f"max_abs_error={float(np.max(np.abs(results['full'] - want))):.3e}")
    return results


def main(argv=None):
    parser = argparse.ArgumentParser(description="Run the lcd_b200 demos on a Matrix Market input.")
    commands = parser.add_subparsers(dest="demo", required=True)
    for name in ("sptrsv", "spilu0", "gauss-seidel"):
        sub = commands.add_parser(name)
        sub.add_argument("matrix", help="path to a square real Matrix Market file")
        sub.add_argument("--max-n", type=int, default=DEFAULT_MAX_N,
                         help="leading principal sample size; use 0 for the full matrix")
        if name == "sptrsv":
            sub.add_argument("--storage", choices=("csr", "csc", "both"), default="both")
        elif name == "spilu0":
            sub.add_argument("--execution-mode", choices=("wavefront", "sync_free"), default="wavefront")
            sub.add_argument("--threads-per-block", type=int, default=128)
            sub.add_argument("--thread-unroll", type=int, choices=(1, 2, 4, 8))
            sub.add_argument("--storage", choices=("csr", "csc", "both"), default="csr")
        else:
            sub.add_argument("--variant", choices=("simple", "full", "both"), default="both")
            sub.add_argument("--iterations", type=int, default=2)
    args = parser.parse_args(argv)
    if args.max_n < 0:
        parser.error("--max-n must be nonnegative")
    if args.demo == "sptrsv":
        return run_sptrsv(args.matrix, args.max_n, args.storage)
    if args.demo == "spilu0":
        if args.threads_per_block <= 0:
            parser.error("--threads-per-block must be positive")
        return run_spilu0(args.matrix, args.max_n, args.execution_mode, args.threads_per_block,
                          args.thread_unroll, args.storage)
    if args.iterations <= 0:
        parser.error("--iterations must be positive")
    return run_gauss_seidel(args.matrix, args.max_n, args.variant, args.iterations)


if __name__ == "__main__":
    main()
