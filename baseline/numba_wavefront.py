"""Times the reference's own Numba-CUDA path for the wavefront (level-by-level) variant of the
CSC triangular solve on the 256 x 256 grid matrix (the first benchmark configuration).

Runs the UNMODIFIED reference from ``baseline/_ref`` (see ``install_reference.py``): its decorator,
SMT-based dependence analysis, generated inspector, Numba-CUDA kernel and generated launcher
(compiler/cuda_lowering.py:855-1016 - one launch plus ``cuda.synchronize()`` per level, no
device-side waits).  ``prepared = op.prepare_cuda_arguments(...)`` once, then
``op.cuda_launcher(*prepared.launcher_arguments)`` + ``cuda.synchronize()`` per repetition, with
``x`` zeroed in between (it doubles as the accumulator of the push form).  Every schedule knob is
fixed, so the scheduler's Python trip-count probe is skipped (compiler/decorator.py:378-401).

Only the wavefront variants are run: the reference's sync-free kernels spin on device flags without
a bound (compiler/cuda_lowering.py:1373, 2036), which is not run on a shared GPU.

Prints one JSON line.  Meant to be started as a child process from a scratch directory (the
reference writes ``smt_file.smt2`` into the current directory).
"""
import contextlib
import io
import json
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, REF)

def _device_name(cuda):
    try:
        name = cuda.get_current_device().name
        return name.decode() if isinstance(name, bytes) else str(name)
    except Exception:                               # (the CUDA simulator has no device object)
        return "unknown"


def main(grid=256, repetitions=20):
    out = {"workload": f"sptrsv_csc_lap2d_g{grid}", "variant": "wavefront, threads_per_block=128"}
    if not os.path.isdir(os.path.join(REF, "compiler")):
        out["unavailable"] = "baseline/_ref is absent (no reference checkout where the library was built)"
        return out
    try:
        from numba import cuda
        if not cuda.is_available():
            out["unavailable"] = "numba.cuda reports no usable device"
            return out
    except Exception as error:                      # numba missing or its CUDA binding unusable
        out["unavailable"] = f"numba.cuda cannot be imported: {type(error).__name__}: {error}"
        return out
    sink = io.StringIO()
    with contextlib.redirect_stdout(sink):       # the reference's pipeline prints a lot
        sys.path.insert(0, HERE)
        from numba_ops import sptrsv_csc        # decorated with the reference's parallel(...)
    from lcd_b200 import generators as gen
    tri = gen.laplacian2d_tril(grid, seed=0)
    Ap, Ai, Ax = tri.csc_arrays()
    t0 = time.perf_counter()
    with contextlib.redirect_stdout(sink):
        prepared = sptrsv_csc.prepare_cuda_arguments(Ap, Ai, Ax, tri.b, tri.n)
    out["inspector_and_compile_s"] = time.perf_counter() - t0
    names = list(prepared.launcher_argument_names)
    arguments = list(prepared.launcher_arguments)
    x_dev = arguments[names.index("x")]
    zeros = np.zeros(tri.n)
    launcher = sptrsv_csc.cuda_launcher

    def solve():
        x_dev.copy_to_device(zeros)
        cuda.synchronize()
        t = time.perf_counter()
        launcher(*arguments)
        cuda.synchronize()
        return (time.perf_counter() - t) * 1e3
    solve()
    solve()
    times = [solve() for _ in range(repetitions)]
    x = x_dev.copy_to_host()
    import scipy.sparse as sp
    A = sp.csc_matrix((Ax, Ai, Ap), shape=(tri.n, tri.n))
    out.update(ms=float(np.median(times)), ms_p20=float(np.percentile(times, 20)),
               ms_p80=float(np.percentile(times, 80)), repetitions=repetitions,
               relative_residual=float(np.linalg.norm(A @ x - tri.b) / np.linalg.norm(tri.b)),
               device=_device_name(cuda))
    return out


if __name__ == "__main__":
    try:
        result = main()
    except Exception as error:                      # report, never crash the benchmark that started us
        result = {"unavailable": f"{type(error).__name__}: {error}"[:400]}
    print(json.dumps(result), flush=True)
