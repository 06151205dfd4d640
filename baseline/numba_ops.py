"""The demo operator decorated with the REFERENCE's ``parallel`` (needs ``baseline/_ref`` on the
path; imported only by ``numba_wavefront.py``).  The reference reads the function's source, so it
has to stand at module level of a real file."""
import numpy as np
from compiler.decorator import parallel     # the reference's decorator

PROPS_CSC = {"Ap": ["monotonically_increasing"], "Ai": [], ("Ap", "Ai"): ["triangularity"]}


@parallel(loop="i", function_props=PROPS_CSC, execution_mode="wavefront", threads_per_block=128)
def sptrsv_csc(Ap, Ai, Ax, b, n):
    x = np.zeros(n)
    for i in range(n):
        x[i] = (b[i] - x[i]) / Ax[Ap[i]]
        for j in range(Ap[i] + 1, Ap[i + 1]):
            x[Ai[j]] += Ax[j] * x[i]
    return x
