"""Operators decorated with the REFERENCE's ``parallel`` (needs the reference on
PYTHONPATH).  Only ``make_golden.py`` imports this file; tests never do."""
import numpy as np
from compiler.decorator import parallel

PROPS_CSR = {"Ap": ["monotonically_increasing"], "Ai": []}
PROPS_CSC = {"Ap": ["monotonically_increasing"], "Ai": [], ("Ap", "Ai"): ["triangularity"]}


@parallel(block_map="i", thread_map="j", function_props=PROPS_CSR, execution_mode="sync_free", threads_per_block=128, thread_unroll=1)
def csr_warp_syncfree(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = b[i]
        for j in range(Ap[i], Ap[i + 1] - 1):
            x[i] -= Ax[j] * x[Ai[j]]
        x[i] /= Ax[Ap[i + 1] - 1]
    return x


@parallel(loop="i", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def csr_plain_wavefront(Ap, Ai, Ax, b, n):
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


@parallel(loop="i", function_props=PROPS_CSC, execution_mode="wavefront", threads_per_block=128)
def csc_plain_wavefront(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x


@parallel(loop="ii", function_props=PROPS_CSR, execution_mode="wavefront", threads_per_block=128)
def csr_upper_reversed(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for ii in range(n):
        x[n - 1 - ii] = b[n - 1 - ii]
        for j in range(Ap[n - 1 - ii] + 1, Ap[n - ii]):
            x[n - 1 - ii] -= Ax[j] * x[Ai[j]]
        x[n - 1 - ii] /= Ax[Ap[n - 1 - ii]]
    return x
