"""Regenerates tests/golden/*.npz by running the REFERENCE's own pipeline.

Run where the reference checkout is available:

    cd <scratch dir> && PYTHONDONTWRITEBYTECODE=1 \
      PYTHONPATH=<reference>:<this repo> python <this repo>/tests/golden/make_golden.py

(the reference writes ``smt_file.smt2`` into the current directory, hence the
scratch directory).  The fixtures hold, for small seeded inputs, the arrays the
reference's inspector / preprocessing / undecorated operators produce; the
tests compare the CPU oracle and the CUDA path against them.
"""
import ast
import contextlib
import io
import os
import sys

import numpy as np
import scipy.sparse as sp

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
REF = next(p for p in sys.path if os.path.isdir(os.path.join(p, "compiler", "demo")))

from lcd_b200 import generators as gen  # noqa: E402

_sink = io.StringIO()
with contextlib.redirect_stdout(_sink):
    import ref_ops  # noqa: E402
    from compiler.demo.spilu0 import compile_ilu0_csr, ilu0_csc, ilu0_csr  # noqa: E402
    from compiler.demo.gauss_seidel import (  # noqa: E402
        full_gauss_seidel_csr, simple_gauss_seidel_csr)
    ilu_syncfree = compile_ilu0_csr("sync_free", 128, 1)
    ilu_wavefront = compile_ilu0_csr("wavefront", 128, 1)
from compiler.dag_preprocessing import (  # noqa: E402
    preprocess_sync_free, preprocess_wavefront, preprocess_warp_tasks, wavefronts_from_dag)
from compiler.structural_lookups import materialize_structural_lookups  # noqa: E402
import utils.dense_blas as dense_blas  # noqa: E402
from utils.symbolic_cholesky_csc import convert_csc_to_supernodal  # noqa: E402


def ragged(lists):
    flat = np.asarray([v for l in lists for v in l], dtype=np.int32)
    ptr = np.zeros(len(lists) + 1, dtype=np.int32)
    ptr[1:] = np.cumsum([len(l) for l in lists])
    return ptr, flat


def dag_record(prefix, op, args, out):
    """Inspector + every preprocessing format for one decorated operator."""
    with contextlib.redirect_stdout(_sink):
        succ, sched = op.build_dag(*args)
        plan = op.schedule_plan(*args)
    data = plan.execution_data
    out[prefix + "succ_ptr"], out[prefix + "succ_idx"] = ragged(succ)
    for name in ("dep_count", "initial_dep_count", "dag_ptr", "dag_index", "wavefronts",
                 "wavefront_ptr", "task_nodes", "task_ptr", "band_ptr"):
        value = getattr(data, name, None)
        if value is not None:
            out[prefix + name] = np.asarray(value)
    for name, value in getattr(data, "auxiliary_values", {}).items():
        out[prefix + "aux_" + name] = np.asarray(value)
    out[prefix + "schedule"] = np.asarray(list(map(str, plan.schedule.lowering_key)))
    return succ, sched


def triangular_cases():
    cases = {}
    cases["lap2d_g8"] = gen.laplacian2d_tril(8, seed=0)
    cases["band_n300"] = gen.random_band_lower(300, seed=1, mean_degree=6.0, band=16)
    cases["band_n600"] = gen.random_band_lower(600, seed=2, mean_degree=15.0, band=64)
    cases["lap3d_g5"] = gen.laplacian3d_tril(5, seed=3)
    return cases


def ilu0_inputs():
    inputs = {"lap3d_g4": gen.laplacian3d_ilu0(4, seed=5)[0]}
    rnd = sp.random(90, 90, density=0.08, random_state=6, format="csr")
    rnd = rnd + rnd.T + sp.identity(90) * 4.0
    rnd = sp.csr_matrix(rnd)
    rnd.sort_indices()
    inputs["random_n90"] = rnd
    nodiag = sp.csr_matrix(rnd.copy())
    nodiag = nodiag.tolil()
    nodiag[5, 5] = 0.0
    nodiag = sp.csr_matrix(nodiag)
    nodiag.eliminate_zeros()
    nodiag.sort_indices()
    inputs["missing_diag_n90"] = nodiag
    return inputs


def write_ilu0_csc(out_dir):
    """ILU0 on CSC storage: the undecorated loop of compiler/demo/spilu0.py:50-82 on the ILU0
    inputs, plus an unsymmetric matrix (columns differ from rows)."""
    inputs = dict(ilu0_inputs())
    uns = sp.random(70, 70, density=0.1, random_state=8, format="csr") + sp.identity(70) * 3.0
    inputs["unsymmetric_n70"] = sp.csr_matrix(uns)
    # explicitly stored zeros right of the diagonal (the column loop skips them: `if u_kj != 0.0`),
    # among them a negative zero, and one huge sub-diagonal entry over a tiny pivot, so that a
    # multiplier overflows to inf where a stored zero sits in the pivot row
    zeros = sp.csr_matrix(sp.random(60, 60, density=0.12, random_state=11, format="csr")
                          + sp.identity(60) * 3.0).tolil()
    zeros[3, 3] = 1e-200
    zeros[7, 3] = 1e200
    zeros[3, 9] = 5.0
    zeros[7, 9] = 2.0
    zeros = sp.csr_matrix(zeros)
    zeros.sort_indices()
    upper = np.flatnonzero(zeros.indices > np.repeat(np.arange(60), np.diff(zeros.indptr)))
    zeros.data[upper[::3]] = 0.0
    zeros.data[upper[1::9]] = -0.0
    zeros.data[[p for p in range(zeros.indptr[3], zeros.indptr[4]) if zeros.indices[p] == 9]] = 0.0
    inputs["stored_zeros_n60"] = zeros
    for name, mat in inputs.items():
        csc = sp.csc_matrix(mat)
        csc.sort_indices()
        data = csc.data.astype(np.float64)
        indices = csc.indices.astype(np.int32)
        indptr = csc.indptr.astype(np.int32)
        out = dict(data=data, indices=indices, indptr=indptr,
                   factored=ilu0_csc(data.copy(), indices, indptr))
        np.savez_compressed(os.path.join(out_dir, f"csc_ilu0_{name}.npz"), **out)
        print("wrote ilu0_csc", name)


def write_band_chains(out_dir):
    """Tasks of the warp executor with band_width > 1: the reference's preprocess_warp_tasks
    (compiler/dag_preprocessing.py:207-298) on the successor lists and level sets of its own
    inspector, for band widths 2, 3 and 5."""
    out = {}
    for name, tri in triangular_cases().items():
        Ap, Ai, Ax = tri.csr_arrays()
        with contextlib.redirect_stdout(_sink):
            succ, dep = ref_ops.csr_warp_syncfree.build_dag(Ap, Ai, Ax, tri.b, tri.n)
        waves = wavefronts_from_dag(succ, dep)
        for width in (2, 3, 5):
            data = preprocess_warp_tasks(succ, waves, band_width=width)
            for field in ("task_nodes", "task_ptr", "band_ptr"):
                out[f"{name}/w{width}/{field}"] = np.asarray(getattr(data, field))
    np.savez_compressed(os.path.join(out_dir, "band_chains.npz"), **out)
    print("wrote band chains", len(out))


def supernodal_conversion_cases():
    """Lower-triangular CSC matrices (sorted columns, diagonal stored) for the converter."""
    rng = np.random.default_rng(17)
    cases = {}
    # Cholesky factor of the 2-D Laplacian on a 9 x 9 grid: real fill, nested column patterns
    g = 9
    T = sp.diags([-1.0, 4.0, -1.0], [-1, 0, 1], shape=(g, g))
    A = (sp.kron(sp.identity(g), T) + sp.kron(sp.diags([-1.0, -1.0], [-1, 1], shape=(g, g)),
                                               sp.identity(g))).toarray()
    L = np.linalg.cholesky(A)
    L[np.abs(L) < 1e-14] = 0.0
    cases["chol_lap2d_g9"] = sp.csc_matrix(np.tril(L))
    # the generator's supernodal matrices, taken back to CSC
    cases["generated_n200"] = gen.supernodal_random(n=200, seed=8, widths=(2, 3, 4, 8),
                                                    min_targets=1, max_targets=4).to_csc()
    # random lower triangle: hardly any column pairs merge
    R = sp.tril(sp.random(150, 150, 0.05, random_state=rng, format="csc"), -1) + sp.identity(150)
    cases["random_n150"] = sp.csc_matrix(R)
    cases["diagonal_n40"] = sp.csc_matrix(sp.identity(40) * 2.0)
    cases["dense_n24"] = sp.csc_matrix(np.tril(rng.uniform(0.5, 1.5, (24, 24))))
    for m in cases.values():
        m.sort_indices()
    return cases


def write_supernodal_conversion(out_dir):
    """convert_csc_to_supernodal (utils/symbolic_cholesky_csc.py:883-1021) of the reference on
    small matrices, relaxation 0, 1 and 3: supernode partition, row structure, column pointers,
    panel values."""
    out = {}
    for name, L in supernodal_conversion_cases().items():
        out[f"{name}/indptr"] = L.indptr.astype(np.int32)
        out[f"{name}/indices"] = L.indices.astype(np.int32)
        out[f"{name}/data"] = L.data.astype(np.float64)
        for relaxation in (0, 1, 3):
            with contextlib.redirect_stdout(_sink):
                Ls = convert_csc_to_supernodal(L, relaxation=relaxation)
            for field in ("x", "i", "ip", "p", "supernodes", "col_to_super"):
                out[f"{name}/r{relaxation}/{field}"] = np.asarray(Ls[field])
            out[f"{name}/r{relaxation}/nSuper"] = np.int64(Ls["nSuper"])
            out[f"{name}/r{relaxation}/max_width"] = np.int64(Ls["max_width"])
    np.savez_compressed(os.path.join(out_dir, "csc_to_supernodal.npz"), **out)
    print("wrote csc_to_supernodal", len(out))


def main():
    out_dir = HERE
    if sys.argv[1:] == ["csc_to_supernodal"]:
        return write_supernodal_conversion(out_dir)
    if sys.argv[1:] == ["ilu0_csc"]:        # only these fixtures
        return write_ilu0_csc(out_dir)
    if sys.argv[1:] == ["band_chains"]:
        return write_band_chains(out_dir)
    # ---- SpTRSV, lower, CSR and CSC -------------------------------------
    for name, tri in triangular_cases().items():
        out = {}
        Ap, Ai, Ax = tri.csr_arrays()
        Cp, Ci, Cx = tri.csc_arrays()
        n, b = tri.n, tri.b
        out.update(csr_Ap=Ap, csr_Ai=Ai, csr_Ax=Ax, csc_Ap=Cp, csc_Ai=Ci, csc_Ax=Cx, b=b)
        succ, dep = dag_record("csr_warp_syncfree/", ref_ops.csr_warp_syncfree, (Ap, Ai, Ax, b, n), out)
        dag_record("csr_plain_wavefront/", ref_ops.csr_plain_wavefront, (Ap, Ai, Ax, b, n), out)
        dag_record("csr_plain_syncfree/", ref_ops.csr_plain_syncfree, (Ap, Ai, Ax, b, n), out)
        dag_record("csc_warp_push/", ref_ops.csc_warp_push, (Cp, Ci, Cx, b, n), out)
        dag_record("csc_plain_wavefront/", ref_ops.csc_plain_wavefront, (Cp, Ci, Cx, b, n), out)
        waves = wavefronts_from_dag(succ, dep)
        out["levels_ptr"], out["levels_idx"] = ragged(waves)
        out["x_csr"] = ref_ops.csr_warp_syncfree.original_function(Ap, Ai, Ax, b, n)
        out["x_csc"] = ref_ops.csc_warp_push.original_function(Cp, Ci, Cx, b, n)
        np.savez_compressed(os.path.join(out_dir, f"sptrsv_{name}.npz"), **out)
        print("wrote", name, "n", n, "levels", len(waves))

    # ---- inspector on unsorted rows with repeated entries -----------------
    rng = np.random.default_rng(7)
    n = 60
    rows = []
    for i in range(n):
        k = int(min(rng.integers(0, 9), i))
        cols = list(rng.integers(0, max(i, 1), size=k)) if i else []
        rows.append([int(c) for c in cols] + [i])          # duplicates, unsorted, diag last
    Ap, Ai = ragged(rows)
    Ax = rng.uniform(0.5, 1.5, len(Ai))
    b = rng.uniform(-1, 1, n)
    out = dict(csr_Ap=Ap, csr_Ai=Ai, csr_Ax=Ax, b=b)
    dag_record("csr_warp_syncfree/", ref_ops.csr_warp_syncfree, (Ap, Ai, Ax, b, n), out)
    dag_record("csr_plain_wavefront/", ref_ops.csr_plain_wavefront, (Ap, Ai, Ax, b, n), out)
    cols = [[] for _ in range(n)]
    for i, r in enumerate(rows):
        for c in r[:-1]:
            cols[c].append(i)
    cols = [[c] + list(rng.permutation(v)) for c, v in enumerate(cols)]  # diag first, unsorted
    Cp, Ci = ragged(cols)
    Cx = rng.uniform(0.5, 1.5, len(Ci))
    out.update(csc_Ap=Cp, csc_Ai=Ci, csc_Ax=Cx)
    dag_record("csc_warp_push/", ref_ops.csc_warp_push, (Cp, Ci, Cx, b, n), out)
    dag_record("csc_plain_wavefront/", ref_ops.csc_plain_wavefront, (Cp, Ci, Cx, b, n), out)
    out["x_csr"] = ref_ops.csr_warp_syncfree.original_function(Ap, Ai, Ax, b, n)
    out["x_csc"] = ref_ops.csc_warp_push.original_function(Cp, Ci, Cx, b, n)
    np.savez_compressed(os.path.join(out_dir, "sptrsv_unsorted_dups.npz"), **out)

    # ---- upper triangular through the reversed-index loop -----------------
    tri = gen.upper_from_lower(gen.random_band_lower(48, seed=4, mean_degree=4.0, band=8))
    Ap, Ai, Ax = tri.csr_arrays()
    out = dict(csr_Ap=Ap, csr_Ai=Ai, csr_Ax=Ax, b=tri.b)
    dag_record("csr_upper_reversed/", ref_ops.csr_upper_reversed, (Ap, Ai, Ax, tri.b, tri.n), out)
    out["x_csr"] = ref_ops.csr_upper_reversed.original_function(Ap, Ai, Ax, tri.b, tri.n)
    np.savez_compressed(os.path.join(out_dir, "sptrsv_upper_n48.npz"), **out)

    # ---- Gauss-Seidel sweeps (the reference's demo operators, inputs as its E2E test builds them)
    for name, tri in (("lap2d_g8", gen.laplacian2d_tril(8, seed=0)),
                      ("band_n300", gen.random_band_lower(300, seed=1, mean_degree=6.0, band=16))):
        full = tri.csr.tocsr()
        full.sort_indices()
        strict = sp.tril(full, k=-1, format="csr")
        strict.sort_indices()
        n = tri.n
        D = full.diagonal().copy()
        b = np.asarray(full @ np.linspace(1.0, 2.0, n)).ravel()
        x0 = np.zeros(n)
        sAp, sAi, sAx = strict.indptr.astype(np.int32), strict.indices.astype(np.int32), strict.data.copy()
        fAp, fAi, fAx = full.indptr.astype(np.int32), full.indices.astype(np.int32), full.data.copy()
        out = dict(simple_Ap=sAp, simple_Ai=sAi, simple_Ax=sAx, D=D, full_Ap=fAp, full_Ai=fAi,
                   full_Ax=fAx, b=b, x0=x0, max_iter=np.int32(2))
        dag_record("simple/", simple_gauss_seidel_csr, (sAp, sAi, sAx, D, b, x0.copy(), n, 2), out)
        dag_record("full/", full_gauss_seidel_csr, (fAp, fAi, fAx, b, x0.copy(), n, 2), out)
        out["simple/launcher_arguments"] = np.asarray(simple_gauss_seidel_csr.cuda_lowering.launcher_arguments)
        out["full/launcher_arguments"] = np.asarray(full_gauss_seidel_csr.cuda_lowering.launcher_arguments)
        out["x_simple"] = simple_gauss_seidel_csr.original_function(sAp, sAi, sAx, D, b, x0.copy(), n, 2)
        out["x_full"] = full_gauss_seidel_csr.original_function(fAp, fAi, fAx, b, x0.copy(), n, 2)
        np.savez_compressed(os.path.join(out_dir, f"gauss_seidel_{name}.npz"), **out)
        print("wrote gauss_seidel", name)

    # ---- Matrix Market ingestion + regularisation (compiler/demo/matrix.py:26-81) ------
    # Synthetic files (no matrix collection is shipped): the file text and what the
    # reference's loader makes of it.
    from compiler.demo.matrix import load_matrix_market as reference_loader
    from lcd_b200.matrix_market import write_matrix_market
    import tempfile
    rng = np.random.default_rng(11)
    base = sp.random(40, 40, density=0.12, random_state=12, format="coo")
    base.data = rng.uniform(-3.0, 3.0, base.nnz)
    sym = sp.random(30, 30, density=0.15, random_state=13, format="csr")
    sym = sym + sym.T + sp.diags(rng.uniform(0.0, 1.0, 30))
    files = {"general": dict(matrix=base, comment="synthetic, with an explicit zero"),
             "symmetric": dict(matrix=sym, symmetric=True),
             "pattern": dict(matrix=sp.csr_matrix(np.tril(rng.uniform(0, 1, (12, 12)) < 0.4)), pattern=True)}
    out = {}
    with tempfile.TemporaryDirectory() as tmp:
        for name, options in files.items():
            path = os.path.join(tmp, name + ".mtx")
            write_matrix_market(path, **options)
            text = open(path).read()
            if name == "general":       # repeated position and an explicit zero entry
                lines = text.splitlines()
                head, entries = lines[:3], lines[3:]
                entries += [entries[0], "5 7 0.0"]
                head[2] = f"40 40 {len(entries)}"
                text = "\n".join(head + entries) + "\n"
                open(path, "w").write(text)
            out[name + "/text"] = np.frombuffer(text.encode(), dtype=np.uint8)
            for size in (0, 16):
                got = reference_loader(path, size)
                out[f"{name}/n{size}/indptr"] = got.indptr
                out[f"{name}/n{size}/indices"] = got.indices
                out[f"{name}/n{size}/data"] = got.data
    np.savez_compressed(os.path.join(out_dir, "matrix_market_cases.npz"), **out)
    print("wrote matrix_market_cases")

    # ---- ILU0 CSR ---------------------------------------------------------
    ilu_inputs = ilu0_inputs()
    for name, mat in ilu_inputs.items():
        data = mat.data.astype(np.float64)
        indices = mat.indices.astype(np.int32)
        indptr = mat.indptr.astype(np.int32)
        out = dict(data=data, indices=indices, indptr=indptr)
        dag_record("ilu_syncfree/", ilu_syncfree, (data.copy(), indices, indptr), out)
        dag_record("ilu_wavefront/", ilu_wavefront, (data.copy(), indices, indptr), out)
        lookups = materialize_structural_lookups(
            ilu_syncfree.structural_lookups, dict(A_indptr=indptr, A_indices=indices))
        (out["diag_pos"],) = [np.asarray(v) for v in lookups.values()]
        out["factored"] = ilu0_csr(data.copy(), indices, indptr)
        np.savez_compressed(os.path.join(out_dir, f"ilu0_{name}.npz"), **out)
        print("wrote ilu0", name)

    write_ilu0_csc(out_dir)
    write_band_chains(out_dir)
    write_supernodal_conversion(out_dir)

    # ---- supernodal solve ------------------------------------------------
    source = open(os.path.join(REF, "benchmark", "sptrsv_supernodal.py")).read()
    fn = next(node for node in ast.parse(source).body
              if isinstance(node, ast.FunctionDef) and node.name == "sptrv_csc_supernodal")
    ns = dict(lsolve_dense_col_order=dense_blas.lsolve_dense_col_order,
              dense_matvec_col_order=dense_blas.dense_matvec_col_order)
    exec(compile(ast.Module(body=[fn], type_ignores=[]), "<supernodal>", "exec"), ns)
    for name, kw in {"n200": dict(n=200, seed=8, widths=(2, 3, 4, 8), min_targets=1, max_targets=4),
                     "n360": dict(n=360, seed=9, widths=(16, 32), min_targets=2, max_targets=4)}.items():
        s = gen.supernodal_random(**kw)
        x = s.b.copy()
        ns["sptrv_csc_supernodal"](s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.b, x)
        out = dict(sn=s.sn, Lip=s.Lip, Li=s.Li, Lp=s.Lp, Lx=s.Lx, b=s.b, x=x,
                   col_to_super=s.col_to_super)
        # layout cross-check: the reference's own CSC -> supernodal converter
        with contextlib.redirect_stdout(_sink):
            Ls = convert_csc_to_supernodal(s.to_csc(), relaxation=0)
        out["conv_supernodes"] = Ls["supernodes"]
        out["conv_i"], out["conv_ip"], out["conv_p"], out["conv_x"] = Ls["i"], Ls["ip"], Ls["p"], Ls["x"]
        np.savez_compressed(os.path.join(out_dir, f"supernodal_{name}.npz"), **out)
        print("wrote supernodal", name, s.n_super)


if __name__ == "__main__":
    main()
