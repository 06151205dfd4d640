"""Operators decorated with lcd_b200's ``parallel`` exactly as a user of the
reference writes them (module level, decorator on one line)."""
import numpy as np

from lcd_b200.decorator import parallel

PROPS_CSR = {"Ap": ["monotonically_increasing"], "Ai": []}
PROPS_CSC = {"Ap": ["monotonically_increasing"], "Ai": [], ("Ap", "Ai"): ["triangularity"]}
PROPS_ILU = {"A_indptr": ["monotonically_increasing"], "A_indices": [], ("A_indptr", "A_indices"): [("segmented_monotonically_increasing", "n")]}


@parallel(loop="i", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def simple_sptrsv_csr(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(loop="i", function_props=PROPS_CSC, execution_mode="wavefront", threads_per_block=128)
def simple_sptrsv_csc(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


@parallel(block_map="i", thread_map="j", function_props=PROPS_CSR, execution_mode="sync_free", threads_per_block=128, thread_unroll=1)
def csr_warp_syncfree(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(loop="i", function_props=PROPS_CSR, execution_mode="sync_free", threads_per_block=128)
def csr_plain_syncfree(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(block_map="i", thread_map="j", function_props=PROPS_CSC, execution_mode="sync_free", threads_per_block=128, thread_unroll=1)
def csc_warp_push(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


@parallel(block_map="i", thread_map="j", function_props=PROPS_CSR)
def csr_auto(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(loop="ii", function_props=PROPS_CSR, execution_mode="sync_free", threads_per_block=128)
def csr_upper_reversed(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for ii in range(n):
        x[n - 1 - ii] = b[n - 1 - ii]
        for j in range(Ap[n - 1 - ii] + 1, Ap[n - ii]):
            x[n - 1 - ii] -= Ax[j] * x[Ai[j]]
        x[n - 1 - ii] /= Ax[Ap[n - 1 - ii]]
    return x


# band chains: tasks are chains of nodes connected inside two consecutive levels
@parallel(block_map="i", thread_map="j", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128, thread_unroll=1, band_width=2)
def csr_warp_wavefront_band2(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(block_map="i", thread_map="j", function_props=PROPS_CSC, execution_mode="wavefront", threads_per_block=128, thread_unroll=1, band_width=3)
def csc_warp_wavefront_band3(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


# the reference's Gauss-Seidel demo operators (compiler/demo/gauss_seidel.py:18-41)
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


@parallel(block_map="i", function_props=PROPS_CSR, execution_mode="sync_free", threads_per_block=128)
def full_gauss_seidel_csr_syncfree(Ap, Ai, Ax, b, x, n, max_iter):
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
                            A_data[j_ptr] = (
                                A_data[j_ptr] - l_ik * u_kj
                            )
                            break
    return A_data


def compile_ilu0_csr(execution_mode="wavefront", threads_per_block=128, thread_unroll=None):
    return parallel(block_map="i", thread_map="j_ptr", function_props=PROPS_ILU, execution_mode=execution_mode, threads_per_block=threads_per_block, thread_unroll=thread_unroll)(ilu0_csr)


def not_served(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i] * 2.0
    return x


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
    """As compiler/demo/spilu0.py:101-108 (no thread map: the column loop has none)."""
    return parallel(block_map="k", function_props=PROPS_ILU, execution_mode=execution_mode, threads_per_block=threads_per_block)(ilu0_csc)
