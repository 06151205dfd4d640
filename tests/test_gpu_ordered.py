"""Parity of the level-ordered sync-free kernels (through the C ABI) with the CPU oracle:
triangular solves with one and many right-hand sides in both hand-off forms, ILU0 with rows
handed out in level order (bit-identical to the sequential loop), the solves on ILU0 factors
kept in place, and the DAG rule for the U part of a full matrix."""
import numpy as np
import pytest
import scipy.sparse as sp

from conftest import golden, golden_names

pytestmark = pytest.mark.gpu

RESIDUAL_TOL = 1e-12     # relative residual ||Lx - b|| / ||b||, fp64


def dev(a, dtype, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(device)


def host(t):
    return t.cpu().numpy()


def csr_residual(Ap, Ai, Ax, x, b):
    n = len(Ap) - 1
    A = sp.csr_matrix((Ax, Ai, Ap), shape=(n, n))
    return float(np.linalg.norm(A @ x - b) / np.linalg.norm(b))


def test_upper_rows_dag_rule(cuda, oracle):
    """Edge rule "entries right of the diagonal of a full row" = the upper-triangular rule on
    the upper triangle of the same matrix (all arrays element-wise)."""
    from lcd_b200 import generators as gen, ops
    mat, _ = gen.laplacian3d_ilu0(9, seed=3)
    rng = np.random.default_rng(5)
    R = sp.random(700, 700, 0.01, random_state=rng, format="csr") + sp.identity(700, format="csr")
    R.sort_indices()
    for A in (mat, R):
        A = sp.csr_matrix(A)
        A.sort_indices()
        Ap, Ai = A.indptr.astype(np.int32), A.indices.astype(np.int32)
        d = ops.dag_build("csr_upper_rows", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
        ref = oracle.dag_build("csr_upper_rows", Ap, Ai)
        U = sp.triu(A, 0, format="csr")
        U.sort_indices()
        tri = oracle.dag_build("csr_upper", U.indptr.astype(np.int32), U.indices.astype(np.int32))
        for name in ("dep_count", "dag_ptr", "dag_index", "level", "wavefronts", "wavefront_ptr"):
            np.testing.assert_array_equal(host(getattr(d, name)), getattr(ref, name))
            np.testing.assert_array_equal(getattr(ref, name), getattr(tri, name))


@pytest.mark.parametrize("use_flags", [False, True])
@pytest.mark.parametrize("nrhs", [1, 2, 3, 8, 13, 16, 31, 32, 33, 64])
def test_ordered_solve_lower_grid(cuda, oracle, nrhs, use_flags):
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian3d_tril(19, seed=1, nrhs=nrhs)
    Ap, Ai, Ax = tri.csr_arrays()
    B = np.ascontiguousarray(tri.b).reshape(tri.n, nrhs)
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    dag = ops.dag_build("csr_lower", dAp, dAi)
    X = host(ops.sptrsv_csr_ordered(dAp, dAi, dev(Ax, np.float64, cuda), dev(B, np.float64, cuda),
                                    dag.wavefronts, use_flags=use_flags))
    for q in range(nrhs):
        want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(B[:, q]))
        np.testing.assert_allclose(X[:, q], want, rtol=1e-10, atol=1e-12)
        assert csr_residual(Ap, Ai, Ax, X[:, q], B[:, q]) <= RESIDUAL_TOL


@pytest.mark.parametrize("use_flags", [False, True])
def test_ordered_solve_vector_forms_and_orders(cuda, oracle, use_flags):
    """A plain vector (nrhs = 1, one-dimensional tensors); rows longer than one staged chunk;
    narrow levels (rows of one batch depend on each other); index order as the order; upper."""
    import torch
    from lcd_b200 import generators as gen, ops
    lower = gen.random_band_lower(6000, seed=4, mean_degree=11.0, band=50)
    for tri, upper in ((lower, False), (gen.upper_from_lower(lower), True)):
        Ap, Ai, Ax = tri.csr_arrays()
        b = np.random.default_rng(9).uniform(-1, 1, tri.n)
        dAp, dAi, dAx, db = (dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda),
                             dev(Ax, np.float64, cuda), dev(b, np.float64, cuda))
        dag = ops.dag_build("csr_upper" if upper else "csr_lower", dAp, dAi)
        want = (oracle.sptrsv_csr_upper if upper else oracle.sptrsv_csr_lower)(Ap, Ai, Ax, b)
        by_index = torch.arange(tri.n, dtype=torch.int32, device=cuda)
        for order in (dag.wavefronts, by_index, ops.OrderedPlan(dag.wavefronts, dag.n_levels)):
            x = host(ops.sptrsv_csr_ordered(dAp, dAi, dAx, db, order, upper=upper, use_flags=use_flags))
            if isinstance(order, ops.OrderedPlan):        # second call reuses the task records
                x = host(ops.sptrsv_csr_ordered(dAp, dAi, dAx, db, order, upper=upper,
                                                use_flags=use_flags, window_rows=64))
            assert x.shape == (tri.n,)
            np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
            assert csr_residual(Ap, Ai, Ax, x, b) <= RESIDUAL_TOL


def test_ordered_solve_config1_matrix_and_empty(cuda, oracle):
    import torch
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian2d_tril(256, seed=0)              # the 65,536-row grid of the first configuration
    Ap, Ai, Ax = tri.csr_arrays()
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    dag = ops.dag_build("csr_lower", dAp, dAi)
    x = host(ops.sptrsv_csr_ordered(dAp, dAi, dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda),
                                    dag.wavefronts))
    assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b), rtol=1e-10, atol=1e-12)
    # n = 0
    e32 = torch.zeros(1, dtype=torch.int32, device=cuda)
    empty = ops.sptrsv_csr_ordered(e32, torch.zeros(0, dtype=torch.int32, device=cuda),
                                   torch.zeros(0, dtype=torch.float64, device=cuda),
                                   torch.zeros(0, dtype=torch.float64, device=cuda),
                                   torch.zeros(0, dtype=torch.int32, device=cuda))
    assert empty.numel() == 0


def test_ordered_solve_reports_bad_orders_without_hanging(cuda):
    """An order that lacks a node, an entry on the wrong side of the diagonal and a node id
    outside the matrix: the bounded waits / the checks report, the context stays usable."""
    import torch
    from lcd_b200 import _native as nat, generators as gen, ops
    tri = gen.laplacian2d_tril(12, seed=0)
    Ap, Ai, Ax = tri.csr_arrays()
    dAp, dAi, dAx, db = (dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda),
                         dev(tri.b, np.float64, cuda))
    order = np.arange(tri.n, dtype=np.int32)
    order[5] = 4                                          # row 5 is never solved: row 6 waits in vain
    with pytest.raises(nat.NativeError) as err:
        ops.sptrsv_csr_ordered(dAp, dAi, dAx, db, dev(order, np.int32, cuda), timeout_ms=200)
    assert err.value.code == nat.ERR_TIMEOUT
    bad = Ai.copy()
    bad[Ap[5]] = 7                                        # row 5 names a later row
    with pytest.raises(nat.NativeError) as err:
        ops.sptrsv_csr_ordered(dAp, dev(bad, np.int32, cuda), dAx, db,
                               torch.arange(tri.n, dtype=torch.int32, device=cuda), timeout_ms=200)
    assert err.value.code == nat.ERR_INDEX_RANGE
    order[:] = np.arange(tri.n)
    order[3] = tri.n + 5                                  # a node id outside the matrix
    with pytest.raises(nat.NativeError) as err:
        ops.sptrsv_csr_ordered(dAp, dAi, dAx, db, dev(order, np.int32, cuda), timeout_ms=200)
    assert err.value.code == nat.ERR_INDEX_RANGE
    x = host(ops.sptrsv_csr_ordered(dAp, dAi, dAx, db, torch.arange(tri.n, dtype=torch.int32, device=cuda)))
    assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL


@pytest.mark.parametrize("name", golden_names("ilu0_"))
def test_ilu0_ordered_is_bit_identical_to_reference(cuda, name):
    from lcd_b200 import ops
    g = golden(name)
    Ap, Ai = dev(g["indptr"], np.int32, cuda), dev(g["indices"], np.int32, cuda)
    pos = ops.diag_positions(Ap, Ai)
    d = ops.dag_build("ilu0_csr", Ap, Ai)
    for lanes in (1, 2, 4, 8, 16, 32):
        out = ops.spilu0_csr(Ap, Ai, dev(g["data"], np.float64, cuda), pos, mode="ordered",
                             wavefronts=d.wavefronts, lanes=lanes)
        np.testing.assert_array_equal(host(out), g["factored"])


def test_ilu0_ordered_then_ordered_solves_on_the_factors(cuda, oracle):
    from lcd_b200 import generators as gen, ops
    mat, b = gen.laplacian3d_ilu0(26, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    pos = ops.diag_positions(dAp, dAi)
    lower = ops.dag_build("ilu0_csr", dAp, dAi)          # operands of the L solve = pivots of ILU0
    upper = ops.dag_build("csr_upper_rows", dAp, dAi)
    fac = ops.spilu0_csr(dAp, dAi, dev(Ax, np.float64, cuda), pos, mode="ordered",
                         wavefronts=lower.wavefronts)
    want = oracle.ilu0_csr(Ap, Ai, Ax, fast=True)
    np.testing.assert_array_equal(host(fac), want)
    hp = host(pos)
    for nrhs in (1, 6):
        B = np.random.default_rng(nrhs).uniform(-1, 1, (len(b), nrhs))
        dB = dev(B if nrhs > 1 else B[:, 0], np.float64, cuda)
        Y = ops.sptrsv_csr_ordered(dAp, dAi, fac, dB, lower.wavefronts, diag_pos=pos, unit_diag=True)
        X = host(ops.sptrsv_csr_ordered(dAp, dAi, fac, Y, upper.wavefronts, diag_pos=pos, upper=True))
        X = X.reshape(len(b), nrhs)
        for q in range(nrhs):
            y_ref = oracle.sptrsv_unit_lower_of_full(Ap, Ai, want, hp, np.ascontiguousarray(B[:, q]))
            x_ref = oracle.sptrsv_upper_of_full(Ap, Ai, want, hp, y_ref)
            np.testing.assert_allclose(X[:, q], x_ref, rtol=1e-10, atol=1e-12)


def test_ilu0_value_flag_kernel_matches_flag_kernel_and_falls_back(cuda, oracle):
    """Ordered ILU0 with the factor's entries as their own ready flags: same bits as the
    flag-based kernel and the sequential loop; a row too long for the lanes' registers is
    reported with A untouched, and the wrapper then takes the flag-based kernel."""
    import torch
    from lcd_b200 import _native as nat, generators as gen, ops
    mat, _ = gen.laplacian3d_ilu0(21, seed=2)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    pos = ops.diag_positions(dAp, dAi)
    d = ops.dag_build("ilu0_csr", dAp, dAi)
    want = oracle.ilu0_csr(Ap, Ai, Ax, fast=True)
    scratch = torch.empty(len(Ai), dtype=torch.float64, device=cuda)
    for lanes in (0, 4, 8, 16, 32):
        got = ops.spilu0_csr(dAp, dAi, dev(Ax, np.float64, cuda), pos, mode="ordered",
                             wavefronts=d.wavefronts, lanes=lanes, scratch=scratch, max_row=7)
        np.testing.assert_array_equal(host(got), want)
    flagged = ops.spilu0_csr(dAp, dAi, dev(Ax, np.float64, cuda), pos, mode="ordered",
                             wavefronts=d.wavefronts, scratch=False)
    np.testing.assert_array_equal(host(flagged), want)
    # a dense-ish banded matrix: rows of up to 81 entries do not fit 2 x 32 registers
    rng = np.random.default_rng(3)
    n = 400
    B = sp.diags([rng.uniform(0.01, 0.1, n - abs(k)) for k in range(-40, 41)], list(range(-40, 41)),
                 format="csr") + 10.0 * sp.identity(n, format="csr")
    B = sp.csr_matrix(B)
    B.sort_indices()
    Bp, Bi, Bx = B.indptr.astype(np.int32), B.indices.astype(np.int32), B.data.copy()
    dBp, dBi = dev(Bp, np.int32, cuda), dev(Bi, np.int32, cuda)
    bpos = ops.diag_positions(dBp, dBi)
    bd = ops.dag_build("ilu0_csr", dBp, dBi)
    work = dev(Bx, np.float64, cuda)
    status = ops.new_status(cuda)
    factor = torch.empty(len(Bi), dtype=torch.float64, device=cuda)
    rc = nat.load().lcd_spilu0_csr_ordered(
        n, len(Bi), nat.ptr(dBp), nat.ptr(dBi), nat.ptr(work), nat.ptr(bpos), nat.ptr(bd.wavefronts),
        nat.ptr(factor), 0, 32, nat.ptr(status), 500, None, None)
    assert rc == nat.OK
    assert ops.read_status(status)[0] == nat.ERR_TOO_LARGE
    np.testing.assert_array_equal(host(work), Bx)            # A is only replaced by a complete factor
    got = ops.spilu0_csr(dBp, dBi, work, bpos, mode="ordered", wavefronts=bd.wavefronts)
    np.testing.assert_array_equal(host(got), oracle.ilu0_csr(Bp, Bi, Bx, fast=True))


def test_ilu0_reports_corrupted_pointers(cuda):
    """A pivot row whose pointers are not monotone is reported, not searched."""
    from lcd_b200 import _native as nat, generators as gen, ops
    mat, _ = gen.laplacian3d_ilu0(6, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    pos = ops.diag_positions(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
    bad = Ap.copy()
    bad[41] = len(Ai) + 1000                              # row 40 ends / row 41 starts past the arrays
    for mode in ("sync_free", "ordered"):
        d = ops.dag_build("ilu0_csr", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
        with pytest.raises(nat.NativeError) as err:
            ops.spilu0_csr(dev(bad, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda),
                           pos, mode=mode, wavefronts=d.wavefronts, timeout_ms=300)
        assert err.value.code in (nat.ERR_BAD_POINTERS, nat.ERR_INDEX_RANGE)


# ------------------------------------------------------------- one-block solver ----
def _small_case(kind, cuda):
    from lcd_b200 import generators as gen
    if kind == "lap2d":
        return gen.laplacian2d_tril(40, seed=2)
    if kind == "lap3d":
        return gen.laplacian3d_tril(13, seed=2)
    if kind == "band":              # narrow levels, rows of up to 8 entries, operands far back
        return gen.random_band_lower(3000, seed=6, mean_degree=3.0, band=9)
    raise ValueError(kind)


@pytest.mark.parametrize("kind", ["lap2d", "lap3d", "band"])
@pytest.mark.parametrize("op", ["csr_lower", "csr_upper", "csc_lower", "csc_upper"])
def test_small_solver_all_forms(cuda, oracle, kind, op):
    from lcd_b200 import _native as nat, generators as gen, ops
    tri = _small_case(kind, cuda)
    upper = op.endswith("upper")
    if upper:
        tri = gen.upper_from_lower(tri)
    b = np.random.default_rng(11).uniform(-1, 1, tri.n)
    Ap, Ai, Ax = tri.csc_arrays() if op.startswith("csc") else tri.csr_arrays()
    dAp, dAi, dAx, db = (dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda),
                         dev(b, np.float64, cuda))
    dag = ops.dag_build(op, dAp, dAi)
    try:
        plan = ops.SmallPlan(op, dAp, dAi, dag)
    except nat.NativeError as error:                    # a row longer than the solver serves
        assert error.code == nat.ERR_TOO_LARGE and kind == "band"
        return
    want = getattr(oracle, "sptrsv_" + op)(Ap, Ai, Ax, b)
    for _ in range(2):                                  # the ring and the scratch are reused
        x = host(ops.sptrsv_small(plan, dAx, db))
        np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    A = sp.csc_matrix((Ax, Ai, Ap), shape=(tri.n, tri.n)) if op.startswith("csc") else \
        sp.csr_matrix((Ax, Ai, Ap), shape=(tri.n, tri.n))
    assert float(np.linalg.norm(A @ x - b) / np.linalg.norm(b)) <= RESIDUAL_TOL


def test_small_solver_config1_csc_and_far_operands(cuda, oracle):
    """The 65,536-row grid of the first configuration in CSC form against SciPy and the oracle;
    then a matrix with operands 10,000 rows back (far outside the shared-memory
    ring) in a chain of 20,000 levels (level offsets staged in several pieces)."""
    from scipy.sparse.linalg import spsolve_triangular
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian2d_tril(256, seed=0)
    for fmt in ("csc", "csr"):
        Ap, Ai, Ax = tri.csc_arrays() if fmt == "csc" else tri.csr_arrays()
        dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
        dag = ops.dag_build(fmt + "_lower", dAp, dAi)
        plan = ops.SmallPlan(fmt + "_lower", dAp, dAi, dag)
        assert plan.entries == 2 and plan.far == 0 and plan.max_width == 256
        x = host(ops.sptrsv_small(plan, dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda)))
        want = getattr(oracle, f"sptrsv_{fmt}_lower")(Ap, Ai, Ax, tri.b)
        np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    A = sp.csr_matrix((Ax, Ai, Ap), shape=(tri.n, tri.n))
    np.testing.assert_allclose(x, spsolve_triangular(A, tri.b, lower=True), rtol=1e-10, atol=1e-12)
    assert float(np.linalg.norm(A @ x - tri.b) / np.linalg.norm(tri.b)) <= RESIDUAL_TOL
    # chain with long-range operands: row i holds columns i - 10000 and i - 1 and the diagonal
    n = 20000
    i = np.arange(n)
    rows = np.concatenate([i[1:], i[10000:], i])
    cols = np.concatenate([i[1:] - 1, i[10000:] - 10000, i])
    rng = np.random.default_rng(3)
    vals = np.concatenate([rng.uniform(-0.3, 0.3, n - 1), rng.uniform(-0.3, 0.3, n - 10000),
                           2.0 + rng.uniform(0, 1, n)])
    L = sp.csr_matrix((vals, (rows, cols)), shape=(n, n))
    L.sort_indices()
    b = rng.uniform(-1, 1, n)
    for fmt in ("csr", "csc"):
        M = L if fmt == "csr" else sp.csc_matrix(L)
        M.sort_indices()
        Ap, Ai, Ax = M.indptr.astype(np.int32), M.indices.astype(np.int32), M.data
        dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
        dag = ops.dag_build(fmt + "_lower", dAp, dAi)
        plan = ops.SmallPlan(fmt + "_lower", dAp, dAi, dag)
        assert dag.n_levels == n and plan.far > 0
        x = host(ops.sptrsv_small(plan, dev(Ax, np.float64, cuda), dev(b, np.float64, cuda)))
        np.testing.assert_allclose(x, getattr(oracle, f"sptrsv_{fmt}_lower")(Ap, Ai, Ax, b),
                                   rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("blocks", [2, 7, 40, 148])
@pytest.mark.parametrize("op", ["csr_lower", "csr_upper", "csc_lower", "csc_upper"])
def test_level_walk_shared_by_many_blocks(cuda, oracle, op, blocks):
    """The level walk cut into node ranges, one thread block each: operands of the own range
    through shared memory, the others polled in global memory.  Same results as the one-block
    form bit for bit (the operands of a task are taken in the same order); repeated solves keep
    the gathered coefficients; levels narrower than the number of blocks leave blocks idle."""
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian3d_tril(17, seed=4)
    if op.endswith("upper"):
        tri = gen.upper_from_lower(tri)
    b = np.random.default_rng(5).uniform(-1, 1, tri.n)
    Ap, Ai, Ax = tri.csc_arrays() if op.startswith("csc") else tri.csr_arrays()
    dAp, dAi, dAx, db = (dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda),
                         dev(b, np.float64, cuda))
    dag = ops.dag_build(op, dAp, dAi)
    one = host(ops.sptrsv_small(ops.SmallPlan(op, dAp, dAi, dag), dAx, db, sync=True))
    plan = ops.SmallPlan(op, dAp, dAi, dag, blocks=blocks)
    assert plan.blocks == blocks and plan.n_slots >= tri.n
    x = host(ops.sptrsv_small(plan, dAx, db, sync=True))
    np.testing.assert_array_equal(x, one)
    np.testing.assert_allclose(x, getattr(oracle, "sptrsv_" + op)(Ap, Ai, Ax, b), rtol=1e-10, atol=1e-12)
    b2 = np.random.default_rng(6).uniform(-1, 1, tri.n)
    x2 = host(ops.sptrsv_small(plan, dAx, dev(b2, np.float64, cuda), sync=True, same_values=True))
    np.testing.assert_allclose(x2, getattr(oracle, "sptrsv_" + op)(Ap, Ai, Ax, b2), rtol=1e-10, atol=1e-12)
    scaled = 3.0 * Ax                                    # new values: gathered again
    x3 = host(ops.sptrsv_small(plan, dev(scaled, np.float64, cuda), db, sync=True))
    np.testing.assert_allclose(x3, getattr(oracle, "sptrsv_" + op)(Ap, Ai, scaled, b), rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("op", ["csr_lower", "csr_upper", "csc_lower"])
def test_level_walk_with_a_block_of_right_hand_sides(cuda, oracle, op):
    """The shared walk on k interleaved copies of the pattern: a row-major n x k block of
    right-hand sides (k = 2, 4, 8, 16, also as a view with a larger leading dimension) gives,
    column by column, exactly what the walk gives for that column alone."""
    import torch
    from lcd_b200 import _native as nat, generators as gen, ops
    tri = gen.laplacian3d_tril(15, seed=2)
    if op.endswith("upper"):
        tri = gen.upper_from_lower(tri)
    Ap, Ai, Ax = tri.csc_arrays() if op.startswith("csc") else tri.csr_arrays()
    dAp, dAi, dAx = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda)
    dag = ops.dag_build(op, dAp, dAi)
    plan = ops.SmallPlan(op, dAp, dAi, dag, blocks=7)
    B = np.random.default_rng(8).uniform(-1, 1, (tri.n, 16))
    dB = dev(B, np.float64, cuda)
    alone = np.stack([host(ops.sptrsv_small(plan, dAx, dB[:, q].contiguous(), sync=True)) for q in range(16)], axis=1)
    np.testing.assert_allclose(alone[:, 3], getattr(oracle, "sptrsv_" + op)(Ap, Ai, Ax, B[:, 3].copy()),
                               rtol=1e-10, atol=1e-12)
    for k in (16, 8, 4, 2):
        X = host(ops.sptrsv_small(plan, dAx, dB[:, :k].contiguous(), sync=True, same_values=True))
        np.testing.assert_array_equal(X, alone[:, :k])
    # a view into a wider block: leading dimension 16, four columns
    out = torch.zeros_like(dB)
    ops.sptrsv_small(plan, dAx, dB[:, 4:8], out[:, 4:8], sync=True)
    np.testing.assert_array_equal(host(out)[:, 4:8], alone[:, 4:8])
    assert not host(out)[:, :4].any() and not host(out)[:, 8:].any()
    with pytest.raises(ops.NativeError) as bad:          # three columns: not served
        ops.sptrsv_small(plan, dAx, dB[:, :3].contiguous(), sync=True)
    assert bad.value.code == nat.ERR_INVALID_ARGUMENT
    one_block = ops.SmallPlan(op, dAp, dAi, dag)
    with pytest.raises(ops.NativeError):                 # the one-block form takes one right-hand side
        ops.sptrsv_small(one_block, dAx, dB[:, :2].contiguous(), sync=True)


def test_level_walk_on_factors_random_patterns_and_bad_input(cuda, oracle):
    """Unit-lower / upper solves on ILU0 factors kept in place; a random band matrix whose
    operands reach far back and into other blocks' ranges; an order that is no level order is
    reported by the plan, not walked."""
    import torch
    from lcd_b200 import _native as nat, generators as gen, ops
    mat, b = gen.laplacian3d_ilu0(14, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    fac = oracle.ilu0_csr(Ap, Ai, Ax, fast=True)
    dAp, dAi, dF, db = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(fac, np.float64, cuda), dev(b, np.float64, cuda)
    pos = ops.diag_positions(dAp, dAi)
    lower = ops.dag_build("ilu0_csr", dAp, dAi)
    upper = ops.dag_build("csr_upper_rows", dAp, dAi)
    hp = host(pos)
    y_ref = oracle.sptrsv_unit_lower_of_full(Ap, Ai, fac, hp, b)
    x_ref = oracle.sptrsv_upper_of_full(Ap, Ai, fac, hp, y_ref)
    for blocks in (1, 5, 33):
        pl = ops.SmallPlan("csr_lower", dAp, dAi, lower, diag_pos=pos, unit_diag=True, blocks=blocks)
        pu = ops.SmallPlan("csr_upper", dAp, dAi, upper, diag_pos=pos, blocks=blocks)
        y = ops.sptrsv_small(pl, dF, db, sync=True)
        x = host(ops.sptrsv_small(pu, dF, y, sync=True))
        np.testing.assert_allclose(host(y), y_ref, rtol=1e-10, atol=1e-12)
        np.testing.assert_allclose(x, x_ref, rtol=1e-10, atol=1e-12)
    band = gen.random_band_lower(30_000, seed=12, mean_degree=4.0, band=2000)
    Bp, Bi, Bx = band.csr_arrays()
    dBp, dBi = dev(Bp, np.int32, cuda), dev(Bi, np.int32, cuda)
    bdag = ops.dag_build("csr_lower", dBp, dBi)
    want = oracle.sptrsv_csr_lower(Bp, Bi, Bx, band.b)
    for blocks in (3, 20):
        try:
            plan = ops.SmallPlan("csr_lower", dBp, dBi, bdag, blocks=blocks)
        except nat.NativeError as error:                  # a row with more than eight operands
            assert error.code == nat.ERR_TOO_LARGE
            break
        x = host(ops.sptrsv_small(plan, dev(Bx, np.float64, cuda), dev(band.b, np.float64, cuda), sync=True))
        np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    # levels that do not belong to the matrix: an operand in the same level as its task
    tri = gen.laplacian2d_tril(20, seed=0)
    Tp, Ti, _ = tri.csr_arrays()
    dTp, dTi = dev(Tp, np.int32, cuda), dev(Ti, np.int32, cuda)
    good = ops.dag_build("csr_lower", dTp, dTi)

    class Flat:                                           # every node in one level
        n_levels = 1
        wavefronts = torch.arange(tri.n, dtype=torch.int32, device=cuda)
        level = torch.zeros(tri.n, dtype=torch.int32, device=cuda)
        wavefront_ptr = torch.tensor([0, tri.n], dtype=torch.int32, device=cuda)
        wavefront_ptr_host = np.array([0, tri.n], dtype=np.int32)
    for blocks in (1, 4):
        with pytest.raises(nat.NativeError) as err:
            ops.SmallPlan("csr_lower", dTp, dTi, Flat, blocks=blocks)
        assert err.value.code == nat.ERR_CYCLE
    assert good.n_levels > 1


def test_partition_need_mask_matches_numpy(cuda):
    """need_mask[c] has bit q set exactly when a row owned by rank q stores an off-diagonal entry
    in a column c produced by another rank (lower and upper, node ids reversed for upper)."""
    import ctypes
    import torch
    from lcd_b200 import _native as nat, generators as gen
    from lcd_b200.multigpu import row_partition
    lower = gen.random_band_lower(5000, seed=8, mean_degree=7.0, band=300)
    for tri, upper in ((lower, False), (gen.upper_from_lower(lower), True)):
        Ap, Ai, _ = tri.csr_arrays()
        n = tri.n
        for parts in (2, 3, 8):
            bounds = row_partition(n, parts)
            want = np.zeros(n, dtype=np.uint8)
            owner_of = np.searchsorted(bounds, np.arange(n), side="right") - 1   # by node id
            for r in range(n):
                node = n - 1 - r if upper else r
                lo, hi = (Ap[r] + 1, Ap[r + 1]) if upper else (Ap[r], Ap[r + 1] - 1)
                for c in Ai[lo:hi]:
                    node_c = n - 1 - c if upper else c
                    if node_c < bounds[owner_of[node]]:
                        want[c] |= 1 << owner_of[node]
            need = torch.zeros((n + 3) // 4 * 4, dtype=torch.uint8, device=cuda)
            dAp, dAi, dbounds = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(bounds, np.int32, cuda)
            rc = nat.load().lcd_partition_need_mask(
                n, nat.ptr(dAp), nat.ptr(dAi), nat.SOLVE_UPPER if upper else 0, nat.ptr(dbounds), parts,
                nat.ptr(need), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
            assert rc == 0
            np.testing.assert_array_equal(host(need)[:n], want)


@pytest.mark.parametrize("name", ["lap2d_g8", "band_n300", "band_n600", "lap3d_g5"])
def test_band_chains_on_device_match_reference_fixture(cuda, name):
    """lcd_band_chains against the arrays the reference's preprocess_warp_tasks produced
    (band widths 2, 3, 5), and on a larger grid against the list form."""
    from lcd_b200 import ops
    chains, g = golden("band_chains"), golden("sptrsv_" + name)
    dag = ops.dag_build("csr_lower", dev(g["csr_Ap"], np.int32, cuda), dev(g["csr_Ai"], np.int32, cuda))
    for width in (2, 3, 5):
        nodes, task_ptr, band_ptr = ops.band_chains(dag, width)
        np.testing.assert_array_equal(host(nodes), chains[f"{name}/w{width}/task_nodes"])
        np.testing.assert_array_equal(host(task_ptr), chains[f"{name}/w{width}/task_ptr"])
        np.testing.assert_array_equal(host(band_ptr), chains[f"{name}/w{width}/band_ptr"])


def test_band_chains_on_device_larger(cuda, oracle):
    from lcd_b200 import dag_preprocessing as dp, generators as gen, ops
    for tri in (gen.laplacian2d_tril(70, seed=1), gen.random_band_lower(20_000, seed=5, mean_degree=5.0, band=30)):
        Ap, Ai, _ = tri.csr_arrays()
        dag = ops.dag_build("csr_lower", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
        ref = oracle.dag_build("csr_lower", Ap, Ai)
        for width in (2, 4, 7, 1000):
            want = dp._band_chains(ref.wavefronts, ref.wavefront_ptr, ref.dag_ptr, ref.dag_index, width)
            got = ops.band_chains(dag, width)
            for a, b in zip(got, want):
                np.testing.assert_array_equal(host(a), b)


def test_capped_dag_build_completes_on_demand(cuda, oracle):
    """A level cap stops the propagation on a deep DAG (the other arrays are complete); reading a
    level array finishes the build, element-wise as without a cap.  A shallow DAG is unaffected."""
    from lcd_b200 import generators as gen, ops
    deep = gen.random_band_lower(60_000, seed=1, mean_degree=15.0, band=64)
    Ap, Ai, _ = deep.csr_arrays()
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    ref = oracle.dag_build("csr_lower", Ap, Ai)
    levels = len(ref.wavefront_ptr) - 1
    capped = ops.dag_build("csr_lower", dAp, dAi, level_cap=500)
    assert levels > 501 and capped.capped and capped.levels_at_least == 501
    np.testing.assert_array_equal(host(capped.dep_count), ref.dep_count)
    np.testing.assert_array_equal(host(capped.dag_ptr), ref.dag_ptr)
    np.testing.assert_array_equal(host(capped.dag_index), ref.dag_index)
    assert capped.capped                                  # still: nothing asked for levels yet
    np.testing.assert_array_equal(host(capped.wavefronts), ref.wavefronts)
    assert not capped.capped and capped.n_levels == levels
    np.testing.assert_array_equal(host(capped.level), ref.level)
    np.testing.assert_array_equal(host(capped.wavefront_ptr), ref.wavefront_ptr)
    shallow = gen.laplacian2d_tril(30, seed=0)
    Sp, Si, _ = shallow.csr_arrays()
    d = ops.dag_build("csr_lower", dev(Sp, np.int32, cuda), dev(Si, np.int32, cuda), level_cap=500)
    assert not d.capped and d.n_levels == 59
    # through the decorator: a deep matrix is solved without its level sets ever being built
    import ops_decorated as od
    big = gen.random_band_lower(40_000, seed=3, mean_degree=15.0, band=64)
    Bp, Bi, Bx = big.csr_arrays()
    x = od.csr_warp_syncfree(Bp, Bi, Bx, big.b, big.n)
    assert csr_residual(Bp, Bi, Bx, x, big.b) <= RESIDUAL_TOL
    plan = od.csr_warp_syncfree.schedule_plan(Bp, Bi, Bx, big.b, big.n)
    assert plan.dag.capped and plan.levels == big.n // 64 + 1
    waves = plan.execution_data.task_nodes                # asking for them builds them
    np.testing.assert_array_equal(host(waves.tensor), oracle.dag_build("csr_lower", Bp, Bi).wavefronts)


def test_device_calibration_gives_plausible_constants(cuda):
    """lcd_calibrate: every figure measured (positive), in the range a current GPU can have."""
    from lcd_b200 import scheduler
    raw = scheduler.calibrate(workspace_bytes=128 << 20)
    assert set(raw) == set(scheduler.CALIBRATION_NAMES)
    assert 0.5e-6 < raw["launch_s"] < 50e-6
    assert 0.1e-6 < raw["l2_handoff_s"] < 20e-6
    assert 5e-9 < raw["shared_memory_handoff_s"] < raw["l2_handoff_s"]
    assert 5e-9 < raw["block_barrier_s"] < 5e-6
    assert 1e-11 < raw["contended_atomic_s"] < 1e-6
    assert 0.3e-6 < raw["grid_barrier_s"] < 100e-6
    assert 0.2e12 < raw["copy_bytes_per_s"] < 20e12
    arch = scheduler.measure_arch_constants()
    assert arch.handoff_s == raw["l2_handoff_s"] or arch.handoff_s > 0      # cached per device
    assert arch.memory_bandwidth_bytes_per_s > 0.2e12
