"""Parity of the CUDA kernels (through the C ABI) with the CPU oracle and with the
fixtures produced by the reference.  Integer arrays must match element-wise;
floating-point results are bit-exact where the kernel keeps the sequential order
(exact mode, ILU0) and otherwise within a relative residual of 1e-12."""
import numpy as np
import pytest
import scipy.sparse as sp

from conftest import golden, golden_names

pytestmark = pytest.mark.gpu

RESIDUAL_TOL = 1e-12


def dev(a, dtype, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(device)


def host(t):
    return t.cpu().numpy()


def csr_residual(Ap, Ai, Ax, x, b):
    n = len(Ap) - 1
    A = sp.csr_matrix((Ax, Ai, Ap), shape=(n, n))
    return float(np.linalg.norm(A @ x - b) / np.linalg.norm(b))


def assert_dag_equal(d, ref):
    np.testing.assert_array_equal(host(d.dep_count), ref.dep_count)
    np.testing.assert_array_equal(host(d.edge_count), ref.edge_count)
    np.testing.assert_array_equal(host(d.dag_ptr), ref.dag_ptr)
    np.testing.assert_array_equal(host(d.dag_index), ref.dag_index)
    np.testing.assert_array_equal(host(d.level), ref.level)
    np.testing.assert_array_equal(host(d.wavefronts), ref.wavefronts)
    np.testing.assert_array_equal(host(d.wavefront_ptr), ref.wavefront_ptr)
    assert d.n_levels == len(ref.wavefront_ptr) - 1
    assert d.n_edges == len(ref.dag_index)


# ------------------------------------------------------------------ DAG ----
@pytest.mark.parametrize("name", golden_names("sptrsv_"))
def test_dag_build_matches_reference_fixture(cuda, oracle, name):
    from lcd_b200 import ops
    g = golden(name)
    if "csr_upper_reversed/succ_ptr" in g:
        cases = [("csr_upper", "csr", "csr_upper_reversed/")]
    else:
        cases = [("csr_lower", "csr", "csr_warp_syncfree/"), ("csc_lower", "csc", "csc_warp_push/")]
    for op, fmt, prefix in cases:
        d = ops.dag_build(op, dev(g[fmt + "_Ap"], np.int32, cuda), dev(g[fmt + "_Ai"], np.int32, cuda))
        np.testing.assert_array_equal(host(d.dag_ptr), g[prefix + "succ_ptr"])
        np.testing.assert_array_equal(host(d.dag_index), g[prefix + "succ_idx"])
        assert_dag_equal(d, oracle.dag_build(op, g[fmt + "_Ap"], g[fmt + "_Ai"]))
        if prefix == "csc_warp_push/":
            np.testing.assert_array_equal(host(d.edge_count), g[prefix + "dep_count"])
            np.testing.assert_array_equal(host(d.wavefronts), g[prefix + "task_nodes"])
            np.testing.assert_array_equal(host(d.wavefront_ptr), g[prefix + "band_ptr"])
        elif prefix == "csr_warp_syncfree/":
            np.testing.assert_array_equal(host(d.dep_count), g[prefix + "dep_count"])
            np.testing.assert_array_equal(host(d.wavefronts), g["csr_plain_wavefront/wavefronts"])
            np.testing.assert_array_equal(host(d.wavefront_ptr), g["csr_plain_wavefront/wavefront_ptr"])


@pytest.mark.parametrize("name", golden_names("ilu0_"))
def test_ilu0_dag_and_diag_table_match_reference_fixture(cuda, oracle, name):
    from lcd_b200 import ops
    g = golden(name)
    Ap, Ai = dev(g["indptr"], np.int32, cuda), dev(g["indices"], np.int32, cuda)
    d = ops.dag_build("ilu0_csr", Ap, Ai)
    np.testing.assert_array_equal(host(d.dag_ptr), g["ilu_syncfree/succ_ptr"])
    np.testing.assert_array_equal(host(d.dag_index), g["ilu_syncfree/succ_idx"])
    np.testing.assert_array_equal(host(d.wavefronts), g["ilu_wavefront/task_nodes"])
    np.testing.assert_array_equal(host(d.wavefront_ptr), g["ilu_wavefront/band_ptr"])
    np.testing.assert_array_equal(host(ops.diag_positions(Ap, Ai)), g["diag_pos"])


@pytest.mark.parametrize("op", ["csr_lower", "csc_lower", "ilu0_csr", "csr_upper", "csc_upper"])
def test_dag_build_matches_oracle_medium(cuda, oracle, op):
    from lcd_b200 import generators as gen, ops
    tri = gen.random_band_lower(60_000, seed=11, mean_degree=9.0, band=48)
    if op in ("csr_lower", "ilu0_csr"):
        Ap, Ai, _ = tri.csr_arrays()
    elif op == "csc_lower":
        Ap, Ai, _ = tri.csc_arrays()
    elif op == "csr_upper":
        Ap, Ai, _ = gen.upper_from_lower(tri).csr_arrays()
    else:
        Ap, Ai, _ = gen.upper_from_lower(tri).csc_arrays()
    d = ops.dag_build(op, dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
    assert_dag_equal(d, oracle.dag_build(op, Ap, Ai))


def test_dag_build_grid_and_degenerate_inputs(cuda, oracle):
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian3d_tril(24, seed=0)
    Ap, Ai, _ = tri.csr_arrays()
    assert_dag_equal(ops.dag_build("csr_lower", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)),
                     oracle.dag_build("csr_lower", Ap, Ai))
    # diagonal matrix: no edges, one level
    n = 1000
    Ap = np.arange(n + 1, dtype=np.int32)
    Ai = np.arange(n, dtype=np.int32)
    d = ops.dag_build("csr_lower", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
    assert d.n_edges == 0 and d.n_levels == 1
    assert_dag_equal(d, oracle.dag_build("csr_lower", Ap, Ai))
    # a single chain: n levels of width one
    rows = [[0]] + [[i - 1, i] for i in range(1, 300)]
    Ap = np.cumsum([0] + [len(r) for r in rows]).astype(np.int32)
    Ai = np.concatenate(rows).astype(np.int32)
    d = ops.dag_build("csr_lower", dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda))
    assert d.n_levels == 300
    assert_dag_equal(d, oracle.dag_build("csr_lower", Ap, Ai))
    # dense lower triangle: long successor lists
    n = 200
    L = sp.csr_matrix(np.tril(np.ones((n, n))))
    d = ops.dag_build("csr_lower", dev(L.indptr, np.int32, cuda), dev(L.indices, np.int32, cuda))
    assert_dag_equal(d, oracle.dag_build("csr_lower", L.indptr, L.indices))


def test_reference_unit_test_vectors_on_device(cuda):
    from lcd_b200 import ops
    # compiler/transform_tests/test_dag_codegen.py:113-167
    d = ops.dag_build("csr_lower", dev([0, 1, 3, 6, 9], np.int32, cuda),
                      dev([0, 0, 1, 0, 1, 2, 1, 2, 3], np.int32, cuda))
    np.testing.assert_array_equal(host(d.dep_count), [0, 1, 2, 2])
    np.testing.assert_array_equal(host(d.dag_ptr), [0, 2, 4, 5, 5])
    np.testing.assert_array_equal(host(d.dag_index), [1, 2, 2, 3, 3])
    d = ops.dag_build("csc_lower", dev([0, 4, 7, 9, 10], np.int32, cuda),
                      dev([0, 1, 2, 2, 1, 2, 3, 2, 3, 3], np.int32, cuda))
    np.testing.assert_array_equal(host(d.dep_count), [0, 1, 2, 2])
    np.testing.assert_array_equal(host(d.edge_count), [0, 1, 3, 2])
    np.testing.assert_array_equal(host(d.dag_index), [1, 2, 2, 3, 3])
    np.testing.assert_array_equal(host(d.wavefronts), [0, 1, 2, 3])
    np.testing.assert_array_equal(host(d.wavefront_ptr), [0, 1, 2, 3, 4])
    # compiler/transform_tests/test_structural_lookups.py:64-92
    pos = ops.diag_positions(dev([0, 2, 3, 5], np.int32, cuda), dev([0, 2, 0, 1, 2], np.int32, cuda))
    np.testing.assert_array_equal(host(pos), [0, -1, 4])
    from lcd_b200._native import ERR_UNSORTED, NativeError
    with pytest.raises(NativeError) as err:
        ops.diag_positions(dev([0, 2], np.int32, cuda), dev([1, 0], np.int32, cuda))
    assert err.value.code == ERR_UNSORTED


# ------------------------------------------------------- sync-free CSR ----
@pytest.mark.parametrize("name", ["sptrsv_lap2d_g8", "sptrsv_band_n600", "sptrsv_unsorted_dups"])
def test_csr_syncfree_exact_mode_is_bit_identical_to_reference(cuda, name):
    from lcd_b200 import ops
    g = golden(name)
    Ap, Ai, Ax = dev(g["csr_Ap"], np.int32, cuda), dev(g["csr_Ai"], np.int32, cuda), dev(g["csr_Ax"], np.float64, cuda)
    b = dev(g["b"], np.float64, cuda)
    for threads in (256, 512, 1024):
        x = ops.sptrsv_csr_syncfree(Ap, Ai, Ax, b, exact=True, threads=threads)
        np.testing.assert_array_equal(host(x), g["x_csr"])


@pytest.mark.parametrize("lanes", [1, 2, 4, 8, 16, 32])
@pytest.mark.parametrize("threads", [256, 1024])
def test_csr_syncfree_lane_groups(cuda, oracle, lanes, threads):
    from lcd_b200 import generators as gen, ops
    tri = gen.random_band_lower(30_000, seed=lanes, mean_degree=20.0, band=64)
    Ap, Ai, Ax = tri.csr_arrays()
    x = ops.sptrsv_csr_syncfree(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda),
                                dev(tri.b, np.float64, cuda), lanes=lanes, threads=threads)
    x = host(x)
    assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b), rtol=1e-10, atol=1e-12)


def _chain_solve(ops, cuda, Ap, Ai, Ax, b, **kw):
    dAp, dAi, dAx = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda)
    ws = ops.chain_prepare(dAp, dAi, dAx, ops.chain_workspace(len(Ap) - 1, cuda), **kw)
    return host(ops.sptrsv_csr_chain(dAp, dAi, dAx, dev(b, np.float64, cuda), ws, **kw))


def test_csr_chain_solver(cuda, oracle):
    """The block-inverse chain solver on banded, grid, unsorted, upper-triangular, dense
    and ragged-size inputs."""
    from lcd_b200 import generators as gen, ops
    cases = [gen.random_band_lower(30_011, seed=7, mean_degree=15.0, band=64),
             gen.random_band_lower(5_000, seed=1, mean_degree=40.0, band=200),
             gen.random_band_lower(2_500, seed=2, mean_degree=120.0, band=900),   # compact list overflows
             gen.laplacian2d_tril(96, seed=2), gen.laplacian3d_tril(17, seed=3)]
    for tri in cases:
        Ap, Ai, Ax = tri.csr_arrays()
        x = _chain_solve(ops, cuda, Ap, Ai, Ax, tri.b)
        assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
        np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b), rtol=1e-10, atol=1e-12)
        up = gen.upper_from_lower(tri)
        Up, Ui, Ux = up.csr_arrays()
        x = _chain_solve(ops, cuda, Up, Ui, Ux, up.b, upper=True)
        np.testing.assert_allclose(x, oracle.sptrsv_csr_upper(Up, Ui, Ux, up.b), rtol=1e-10, atol=1e-12)
    for name in ("sptrsv_unsorted_dups", "sptrsv_band_n600", "sptrsv_lap2d_g8"):
        g = golden(name)
        x = _chain_solve(ops, cuda, g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"])
        np.testing.assert_allclose(x, g["x_csr"], rtol=1e-10, atol=1e-12)
    assert _chain_solve(ops, cuda, [0, 1], [0], [4.0], [2.0])[0] == 0.5
    # a dense lower triangle: every row of a block depends on all earlier rows of the block
    n = 150
    L = sp.csr_matrix(np.tril(np.random.default_rng(0).uniform(0.01, 0.02, (n, n))) + 2 * np.eye(n))
    b = np.ones(n)
    x = _chain_solve(ops, cuda, L.indptr, L.indices, L.data, b)
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(L.indptr, L.indices, L.data, b), rtol=1e-10, atol=1e-12)


def test_csr_chain_solver_cluster_sizes(cuda, oracle):
    """Consecutive chunks hand over through distributed shared memory inside a cluster and through
    L2 across clusters (or everywhere, for plain blocks): every cluster size gives the solution."""
    from lcd_b200 import _native as nat, generators as gen, ops
    lib = nat.load()
    tri = gen.random_band_lower(40_000, seed=11, mean_degree=15.0, band=64)     # 40 chunks, the last partial
    Ap, Ai, Ax = tri.csr_arrays()
    want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
    used = []
    try:
        for limit in (1, 2, 4, 8, 0):
            assert lib.lcd_set_tuning(nat.TUNE_CHAIN_CLUSTER, limit) == 0
            x = _chain_solve(ops, cuda, Ap, Ai, Ax, tri.b)
            np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
            used.append(lib.lcd_chain_cluster_size())
            assert used[-1] >= 1 and (limit == 0 or used[-1] <= limit)
        assert lib.lcd_set_tuning(nat.TUNE_CHAIN_CLUSTER, 3) != 0
    finally:
        lib.lcd_set_tuning(nat.TUNE_CHAIN_CLUSTER, 0)
    assert used[0] == 1


@pytest.mark.parametrize("mode", ["sync_free", "wavefront", "ordered"])
@pytest.mark.parametrize("name", golden_names("csc_ilu0_"))
def test_ilu0_on_csc_storage_is_bit_identical(cuda, oracle, name, mode):
    """ILU0 of a matrix stored by columns: gathered into row order, factored by the row kernel,
    scattered back - bit for bit the result of the reference's column loop, stored zeros in pivot
    rows (skipped by that loop), a negative zero and an infinite multiplier included."""
    from lcd_b200 import _native as nat, ops
    g = golden(name)
    Ap, Ai = dev(g["indptr"], np.int32, cuda), dev(g["indices"], np.int32, cuda)
    view = ops.csc_row_view(Ap, Ai)
    kw = {}
    if mode != "sync_free":
        d = ops.dag_build("ilu0_csr", view.Ap, view.Ai)
        kw = dict(wavefronts=d.wavefronts, wavefront_ptr_host=host(d.wavefront_ptr))
    for lookahead in (1, 0):
        nat.load().lcd_set_tuning(nat.TUNE_ILU0_LOOKAHEAD, lookahead)
        out = host(ops.spilu0_csc(Ap, Ai, dev(g["data"], np.float64, cuda), view, mode=mode, **kw))
        nat.load().lcd_set_tuning(nat.TUNE_ILU0_LOOKAHEAD, 1)
        np.testing.assert_array_equal(out, g["factored"])
        np.testing.assert_array_equal(out.view(np.int64), g["factored"].view(np.int64))   # signs of zero too


def test_ilu0_on_csc_storage_larger(cuda, oracle):
    import scipy.sparse as sp
    from lcd_b200 import generators as gen, ops
    mat, _ = gen.laplacian3d_ilu0(14, seed=2)
    rng = np.random.default_rng(4)
    mat = sp.csr_matrix(mat + sp.random(mat.shape[0], mat.shape[0], density=2e-4, random_state=3) * 0.1)
    csc = sp.csc_matrix(mat)
    csc.sort_indices()
    Ap, Ai, Ax = csc.indptr.astype(np.int32), csc.indices.astype(np.int32), csc.data.astype(np.float64)
    out = ops.spilu0_csc(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda))
    np.testing.assert_array_equal(host(out), oracle.ilu0_csc(Ap, Ai, Ax))
    # columns out of order are accepted (the row view sorts)
    perm_cols = Ax.copy()
    idx = Ai.copy()
    for j in range(0, len(Ap) - 1, 7):
        lo, hi = Ap[j], Ap[j + 1]
        order = rng.permutation(hi - lo)
        idx[lo:hi], perm_cols[lo:hi] = Ai[lo:hi][order], Ax[lo:hi][order]
    out = ops.spilu0_csc(dev(Ap, np.int32, cuda), dev(idx, np.int32, cuda), dev(perm_cols, np.float64, cuda))
    np.testing.assert_array_equal(host(out), oracle.ilu0_csc(Ap, idx, perm_cols))


def test_csr_chain_solver_in_row_ranges(cuda, oracle):
    """A solve issued as consecutive row ranges (tiles prepared range by range, from values
    that are only valid for the rows prepared so far) equals the solve in one piece."""
    import torch
    from lcd_b200 import generators as gen, ops
    from lcd_b200._native import ERR_INVALID_ARGUMENT, NativeError
    for upper in (False, True):
        tri = gen.random_band_lower(40_000, seed=13, mean_degree=15.0, band=64)
        if upper:
            tri = gen.upper_from_lower(tri)
        Ap, Ai, Ax = tri.csr_arrays()
        want = (oracle.sptrsv_csr_upper if upper else oracle.sptrsv_csr_lower)(Ap, Ai, Ax, tri.b)
        dAp, dAi, dAx = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda)
        db = dev(tri.b, np.float64, cuda)
        n = tri.n
        ws = ops.chain_workspace(n, cuda)
        x = torch.zeros(n, dtype=torch.float64, device=cuda)
        status = ops.new_status(cuda)
        # values arrive range by range: entries of rows not yet "uploaded" are NaN
        staged = torch.full_like(dAx, float("nan"))
        cuts = [0, 8192, 8192 + 512, 30720, n]
        for begin, end in zip(cuts, cuts[1:]):
            rows = range(begin, end) if not upper else range(n - end, n - begin)
            lo, hi = int(Ap[rows[0]]), int(Ap[rows[-1] + 1])
            staged[lo:hi] = dAx[lo:hi]
            ops.chain_prepare(dAp, dAi, staged, ws, upper=upper, rows=(begin, end))
            ops.sptrsv_csr_chain(dAp, dAi, staged, db, ws, x, upper=upper, status=status,
                                 rows=(begin, end), sync=end == n)
        np.testing.assert_allclose(host(x), want, rtol=1e-10, atol=1e-12)
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csr_chain(dAp, dAi, dAx, db, ws, x, upper=True, rows=(100, n))
    assert err.value.code == ERR_INVALID_ARGUMENT
    with pytest.raises(NativeError) as err:
        ops.chain_prepare(dAp, dAi, dAx, ws, rows=(64, 100))
    assert err.value.code == ERR_INVALID_ARGUMENT


def test_csr_chain_prepare_and_solve_pipelined(cuda, oracle):
    """Preparation on a second stream, range by range, with the solve of a range behind its
    own tiles: same result as the two steps one after the other, for every number of pieces."""
    import torch
    from lcd_b200 import generators as gen, ops
    for upper in (False, True):
        tri = gen.random_band_lower(70_000, seed=21, mean_degree=15.0, band=64)
        if upper:
            tri = gen.upper_from_lower(tri)
        Ap, Ai, Ax = tri.csr_arrays()
        want = (oracle.sptrsv_csr_upper if upper else oracle.sptrsv_csr_lower)(Ap, Ai, Ax, tri.b)
        dAp, dAi, dAx = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda)
        db = dev(tri.b, np.float64, cuda)
        ws = ops.chain_workspace(tri.n, cuda)
        for pieces in (1, 2, 5, 8, 1000):
            ws.zero_()
            x = ops.chain_prepare_and_solve(dAp, dAi, dAx, db, ws, upper=upper, pieces=pieces)
            np.testing.assert_allclose(host(x), want, rtol=1e-10, atol=1e-12)
            assert ops.chain_growth(ws, tri.n) <= ops.CHAIN_MAX_GROWTH


def test_csr_chain_solver_on_ilu_factors_and_errors(cuda, oracle):
    from lcd_b200 import generators as gen, ops
    from lcd_b200._native import ERR_INDEX_RANGE, ERR_WORKSPACE, NativeError
    mat, b = gen.laplacian3d_ilu0(12, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    pos = ops.diag_positions(dAp, dAi)
    fac = ops.spilu0_csr(dAp, dAi, dev(Ax, np.float64, cuda), pos)
    ws = ops.chain_workspace(len(Ap) - 1, cuda)
    ops.chain_prepare(dAp, dAi, fac, ws, diag_pos=pos, unit_diag=True)
    y = ops.sptrsv_csr_chain(dAp, dAi, fac, dev(b, np.float64, cuda), ws, diag_pos=pos, unit_diag=True)
    ops.chain_prepare(dAp, dAi, fac, ws, diag_pos=pos, upper=True)
    x = ops.sptrsv_csr_chain(dAp, dAi, fac, y, ws, diag_pos=pos, upper=True)
    want = oracle.ilu0_csr(Ap, Ai, Ax, fast=True)
    hp = host(pos)
    x_ref = oracle.sptrsv_upper_of_full(Ap, Ai, want, hp, oracle.sptrsv_unit_lower_of_full(Ap, Ai, want, hp, b))
    np.testing.assert_allclose(host(x), x_ref, rtol=1e-10, atol=1e-12)
    tri = gen.random_band_lower(5000, seed=9, mean_degree=8.0, band=32)
    Ap, Ai, Ax = tri.csr_arrays()
    bad = Ai.copy()
    row = next(r for r in range(10, 100) if Ap[r + 1] - Ap[r] >= 2)
    bad[Ap[row]] = row + 10
    dAp, dbad, dAx = dev(Ap, np.int32, cuda), dev(bad, np.int32, cuda), dev(Ax, np.float64, cuda)
    ws = ops.chain_prepare(dAp, dbad, dAx, ops.chain_workspace(tri.n, cuda))
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csr_chain(dAp, dbad, dAx, dev(tri.b, np.float64, cuda), ws, timeout_ms=300)
    assert err.value.code == ERR_INDEX_RANGE
    import torch
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csr_chain(dAp, dev(Ai, np.int32, cuda), dAx, dev(tri.b, np.float64, cuda),
                             torch.empty(16, dtype=torch.float64, device=cuda))
    assert err.value.code == ERR_WORKSPACE


def test_csr_syncfree_upper_and_golden(cuda, oracle):
    from lcd_b200 import generators as gen, ops
    g = golden("sptrsv_upper_n48")
    x = ops.sptrsv_csr_syncfree(dev(g["csr_Ap"], np.int32, cuda), dev(g["csr_Ai"], np.int32, cuda),
                                dev(g["csr_Ax"], np.float64, cuda), dev(g["b"], np.float64, cuda),
                                upper=True, exact=True)
    np.testing.assert_array_equal(host(x), g["x_csr"])
    tri = gen.upper_from_lower(gen.random_band_lower(50_000, seed=5, mean_degree=12.0, band=32))
    Ap, Ai, Ax = tri.csr_arrays()
    for lanes in (1, 4):
        x = host(ops.sptrsv_csr_syncfree(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda),
                                         dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda),
                                         upper=True, lanes=lanes))
        assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
        np.testing.assert_allclose(x, oracle.sptrsv_csr_upper(Ap, Ai, Ax, tri.b), rtol=1e-10, atol=1e-12)


def test_csr_syncfree_grid_matrix_and_edge_cases(cuda, oracle):
    import torch
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian2d_tril(256, seed=0)   # the 65,536-row configuration
    Ap, Ai, Ax = tri.csr_arrays()
    dAp, dAi, dAx, db = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda)
    x = host(ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db))
    assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
    xe = host(ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db, exact=True))
    np.testing.assert_array_equal(xe, oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b))
    # empty system and 1x1 system
    e = ops.sptrsv_csr_syncfree(dev([0], np.int32, cuda), dev([], np.int32, cuda), dev([], np.float64, cuda),
                                dev([], np.float64, cuda))
    assert e.numel() == 0
    one = ops.sptrsv_csr_syncfree(dev([0, 1], np.int32, cuda), dev([0], np.int32, cuda),
                                  dev([4.0], np.float64, cuda), dev([2.0], np.float64, cuda))
    assert host(one)[0] == 0.5
    # two solves in a row reuse nothing from the first
    x2 = host(ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db, exact=True))
    np.testing.assert_array_equal(x2, xe)
    assert torch.isfinite(torch.from_numpy(x2)).all()


@pytest.mark.parametrize("nrhs", [1, 3, 8, 17, 32, 64])
def test_csr_syncfree_multi_rhs(cuda, oracle, nrhs):
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian3d_tril(20, seed=1, nrhs=nrhs)
    Ap, Ai, Ax = tri.csr_arrays()
    B = np.ascontiguousarray(tri.b)          # row-major n x nrhs
    X = host(ops.sptrsv_csr_syncfree_multi(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda),
                                           dev(Ax, np.float64, cuda), dev(B, np.float64, cuda)))
    for q in range(nrhs):
        want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, B[:, q])
        np.testing.assert_allclose(X[:, q], want, rtol=1e-10, atol=1e-12)
        assert csr_residual(Ap, Ai, Ax, X[:, q], B[:, q]) <= RESIDUAL_TOL


@pytest.mark.parametrize("nrhs", [1, 5, 32, 33, 64])
def test_wavefront_multi_rhs(cuda, oracle, nrhs):
    from lcd_b200 import generators as gen, ops
    for tri, upper in ((gen.laplacian3d_tril(18, seed=1, nrhs=nrhs), False),
                       (gen.random_band_lower(4000, seed=2, mean_degree=9.0, band=40), True)):
        if upper:
            tri = gen.upper_from_lower(tri)
            B = np.random.default_rng(nrhs).uniform(-1, 1, (tri.n, nrhs))
        else:
            B = np.ascontiguousarray(tri.b)
        Ap, Ai, Ax = tri.csr_arrays()
        dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
        dag = ops.dag_build("csr_upper" if upper else "csr_lower", dAp, dAi)
        X = host(ops.sptrsv_wavefront_multi(dAp, dAi, dev(Ax, np.float64, cuda), dev(B, np.float64, cuda),
                                            dag.wavefronts, dag.wavefront_ptr, upper=upper))
        solve = oracle.sptrsv_csr_upper if upper else oracle.sptrsv_csr_lower
        for q in range(0, nrhs, max(1, nrhs // 4)):
            np.testing.assert_allclose(X[:, q], solve(Ap, Ai, Ax, np.ascontiguousarray(B[:, q])),
                                       rtol=1e-10, atol=1e-12)


def test_sharded_multi_rhs_single_rank(cuda, oracle):
    """The multi-GPU front end with one rank: 70 columns go through two launches."""
    from lcd_b200 import generators as gen
    from lcd_b200.multigpu import ShardedMultiRHS
    tri = gen.laplacian3d_tril(14, seed=2, nrhs=70)
    Ap, Ai, Ax = tri.csr_arrays()
    solver = ShardedMultiRHS(Ap, Ai, Ax)
    X = host(solver.solve(np.asarray(tri.b), gather=True))
    assert X.shape == (70, tri.n)
    for q in (0, 33, 63, 64, 69):
        want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, np.ascontiguousarray(tri.b[:, q]))
        np.testing.assert_allclose(X[q], want, rtol=1e-10, atol=1e-12)


def test_transpose_roundtrip(cuda):
    import torch
    from lcd_b200 import ops
    a = torch.rand(1000, 37, dtype=torch.float64, device=cuda)
    t = ops.transpose(a, 1000, 37)
    assert torch.equal(t, a.t().contiguous())
    assert torch.equal(ops.transpose(t, 37, 1000), a)


# ------------------------------------------------------- sync-free CSC ----
@pytest.mark.parametrize("lanes", [1, 4, 32])
def test_csc_syncfree_push(cuda, oracle, lanes):
    from lcd_b200 import generators as gen, ops
    for name in ("sptrsv_band_n600", "sptrsv_unsorted_dups"):
        g = golden(name)
        Ap, Ai = dev(g["csc_Ap"], np.int32, cuda), dev(g["csc_Ai"], np.int32, cuda)
        dep = ops.csc_edge_count(Ap, Ai)
        np.testing.assert_array_equal(host(dep), g["csc_warp_push/dep_count"])
        x = ops.sptrsv_csc_syncfree(Ap, Ai, dev(g["csc_Ax"], np.float64, cuda), dev(g["b"], np.float64, cuda),
                                    dep, lanes=lanes)
        np.testing.assert_allclose(host(x), g["x_csc"], rtol=1e-10, atol=1e-12)
    tri = gen.random_band_lower(40_000, seed=21, mean_degree=14.0, band=64)
    Ap, Ai, Ax = tri.csc_arrays()
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    x = host(ops.sptrsv_csc_syncfree(dAp, dAi, dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda),
                                     ops.csc_edge_count(dAp, dAi), lanes=lanes))
    rAp, rAi, rAx = tri.csr_arrays()
    assert csr_residual(rAp, rAi, rAx, x, tri.b) <= RESIDUAL_TOL
    up = gen.upper_from_lower(tri)
    Ap, Ai, Ax = up.csc_arrays()
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    x = host(ops.sptrsv_csc_syncfree(dAp, dAi, dev(Ax, np.float64, cuda), dev(up.b, np.float64, cuda),
                                     ops.csc_edge_count(dAp, dAi, upper=True), upper=True, lanes=lanes))
    np.testing.assert_allclose(x, oracle.sptrsv_csc_upper(Ap, Ai, Ax, up.b), rtol=1e-10, atol=1e-12)


# ---------------------------------------------------------- wavefront ----
@pytest.mark.parametrize("mode", ["per_level", "cooperative"])
@pytest.mark.parametrize("lanes", [1, 8])
def test_wavefront_csr_and_csc(cuda, oracle, mode, lanes):
    from lcd_b200 import generators as gen, ops
    for tri in (gen.laplacian2d_tril(96, seed=2), gen.random_band_lower(3000, seed=3, mean_degree=10.0, band=32)):
        Ap, Ai, Ax = tri.csr_arrays()
        dAp, dAi, dAx, db = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda), dev(tri.b, np.float64, cuda)
        d = ops.dag_build("csr_lower", dAp, dAi)
        x = host(ops.sptrsv_wavefront("csr_lower", dAp, dAi, dAx, db, d.wavefronts, d.wavefront_ptr,
                                      d.wavefront_ptr_host, mode=mode, lanes=lanes, exact=(lanes == 1)))
        want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
        if lanes == 1:
            np.testing.assert_array_equal(x, want)
        np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
        Cp, Ci, Cx = tri.csc_arrays()
        dCp, dCi = dev(Cp, np.int32, cuda), dev(Ci, np.int32, cuda)
        d = ops.dag_build("csc_lower", dCp, dCi)
        x = host(ops.sptrsv_wavefront("csc_lower", dCp, dCi, dev(Cx, np.float64, cuda), db, d.wavefronts,
                                      d.wavefront_ptr, d.wavefront_ptr_host, mode=mode, lanes=lanes))
        assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
        up = gen.upper_from_lower(tri)
        Up, Ui, Ux = up.csr_arrays()
        dUp, dUi = dev(Up, np.int32, cuda), dev(Ui, np.int32, cuda)
        d = ops.dag_build("csr_upper", dUp, dUi)
        x = host(ops.sptrsv_wavefront("csr_upper", dUp, dUi, dev(Ux, np.float64, cuda), db, d.wavefronts,
                                      d.wavefront_ptr, d.wavefront_ptr_host, mode=mode, lanes=lanes))
        np.testing.assert_allclose(x, oracle.sptrsv_csr_upper(Up, Ui, Ux, up.b), rtol=1e-10, atol=1e-12)


# -------------------------------------------------------------- ILU0 ----
@pytest.mark.parametrize("name", golden_names("ilu0_"))
def test_ilu0_is_bit_identical_to_reference(cuda, name):
    from lcd_b200 import ops
    g = golden(name)
    Ap, Ai = dev(g["indptr"], np.int32, cuda), dev(g["indices"], np.int32, cuda)
    pos = ops.diag_positions(Ap, Ai)
    d = ops.dag_build("ilu0_csr", Ap, Ai)
    for lanes in (1, 2, 4, 8, 16, 32):
        out = ops.spilu0_csr(Ap, Ai, dev(g["data"], np.float64, cuda), pos, mode="sync_free", lanes=lanes)
        np.testing.assert_array_equal(host(out), g["factored"])
        out = ops.spilu0_csr(Ap, Ai, dev(g["data"], np.float64, cuda), pos, mode="wavefront",
                             wavefronts=d.wavefronts, wavefront_ptr_host=d.wavefront_ptr_host, lanes=lanes)
        np.testing.assert_array_equal(host(out), g["factored"])


def test_ilu0_then_forward_backward_solves(cuda, oracle):
    from lcd_b200 import generators as gen, ops
    mat, b = gen.laplacian3d_ilu0(24, seed=0)
    Ap, Ai, Ax = mat.indptr.astype(np.int32), mat.indices.astype(np.int32), mat.data
    dAp, dAi = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda)
    pos = ops.diag_positions(dAp, dAi)
    fac = ops.spilu0_csr(dAp, dAi, dev(Ax, np.float64, cuda), pos)
    want = oracle.ilu0_csr(Ap, Ai, Ax, fast=True)
    np.testing.assert_array_equal(host(fac), want)
    db = dev(b, np.float64, cuda)
    y = ops.sptrsv_csr_syncfree(dAp, dAi, fac, db, diag_pos=pos, unit_diag=True, exact=True)
    x = ops.sptrsv_csr_syncfree(dAp, dAi, fac, y, diag_pos=pos, upper=True, exact=True)
    hp = host(pos)
    y_ref = oracle.sptrsv_unit_lower_of_full(Ap, Ai, want, hp, b)
    x_ref = oracle.sptrsv_upper_of_full(Ap, Ai, want, hp, y_ref)
    np.testing.assert_array_equal(host(y), y_ref)
    np.testing.assert_array_equal(host(x), x_ref)
    # SciPy cross-check of the split factors (L unit lower, U upper with diagonal)
    from scipy.sparse.linalg import spsolve_triangular
    n = len(Ap) - 1
    F = sp.csr_matrix((want, Ai, Ap), shape=(n, n))
    L = sp.tril(F, -1, format="csr") + sp.identity(n, format="csr")
    U = sp.triu(F, 0, format="csr")
    xs = spsolve_triangular(U, spsolve_triangular(L, b, lower=True, unit_diagonal=True), lower=False)
    np.testing.assert_allclose(host(x), xs, rtol=1e-10, atol=1e-12)
    # fast (fused, reciprocal) variants stay within the residual tolerance
    y2 = ops.sptrsv_csr_syncfree(dAp, dAi, fac, db, diag_pos=pos, unit_diag=True)
    x2 = ops.sptrsv_csr_syncfree(dAp, dAi, fac, y2, diag_pos=pos, upper=True)
    np.testing.assert_allclose(host(x2), x_ref, rtol=1e-10, atol=1e-12)


# --------------------------------------------------------- supernodal ----
@pytest.mark.parametrize("name", golden_names("supernodal_"))
def test_supernodal_matches_reference_fixture(cuda, name):
    import torch
    from lcd_b200 import supernodal
    g = golden(name)
    plan = supernodal.analyse(g["sn"], g["Lip"], g["Li"], g["Lp"], g["Lx"], g["col_to_super"])
    for _ in range(2):  # the plan is reusable
        x = supernodal.solve(plan, dev(g["b"], np.float64, cuda))
        np.testing.assert_allclose(host(x), g["x"], rtol=1e-10, atol=1e-12)
    x = g["b"].copy()
    supernodal.sptrsv_csc_supernodal(g["sn"], g["col_to_super"], g["Lip"], g["Li"], g["Lp"], g["Lx"], x)
    np.testing.assert_allclose(x, g["x"], rtol=1e-10, atol=1e-12)
    assert torch.cuda.is_available()


def test_supernodal_medium(cuda, oracle):
    from lcd_b200 import generators as gen, supernodal
    s = gen.supernodal_random(n=20_000, seed=3, widths=(16, 32, 64, 128), min_targets=4, max_targets=12)
    want = oracle.sptrsv_supernodal(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.b)
    L = s.to_csc().tocsr()
    for invert in (True, False):      # with the inverted diagonal blocks, and step by step
        plan = supernodal.analyse(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.col_to_super, invert_triangles=invert)
        assert (plan.block_inverses is not None) == invert
        x = host(supernodal.solve(plan, dev(s.b, np.float64, cuda)))
        np.testing.assert_allclose(x, want, rtol=1e-9, atol=1e-12)
        assert np.linalg.norm(L @ x - s.b) / np.linalg.norm(s.b) <= RESIDUAL_TOL
    # widths that are no powers of two, and some wider than a thread block
    s = gen.supernodal_random(n=6_000, seed=5, widths=(5, 17, 40, 70, 300), min_targets=2, max_targets=6)
    plan = supernodal.analyse(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.col_to_super)
    x = host(supernodal.solve(plan, dev(s.b, np.float64, cuda)))
    np.testing.assert_allclose(x, oracle.sptrsv_supernodal(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.b), rtol=1e-9, atol=1e-12)


@pytest.mark.parametrize("relaxation", [0, 1, 3])
def test_csc_to_supernodal_matches_reference_converter(cuda, relaxation):
    """The device converter against what the reference's convert_csc_to_supernodal returned
    (utils/symbolic_cholesky_csc.py:950-1021): every array element-wise, values bit-exact."""
    import os
    from lcd_b200 import supernodal
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "csc_to_supernodal.npz"))
    for name in sorted({k.split("/")[0] for k in g.files}):
        got = supernodal.from_csc(g[f"{name}/indptr"], g[f"{name}/indices"], g[f"{name}/data"],
                                  relaxation=relaxation, device=cuda)
        ref = {f: g[f"{name}/r{relaxation}/{f}"] for f in ("x", "i", "ip", "p", "supernodes", "col_to_super")}
        np.testing.assert_array_equal(host(got.sn), ref["supernodes"], err_msg=name)
        np.testing.assert_array_equal(host(got.col_to_super), ref["col_to_super"], err_msg=name)
        np.testing.assert_array_equal(host(got.Lip), ref["ip"], err_msg=name)
        np.testing.assert_array_equal(host(got.Li), ref["i"], err_msg=name)
        np.testing.assert_array_equal(host(got.Lp), ref["p"], err_msg=name)
        np.testing.assert_array_equal(host(got.Lx), ref["x"], err_msg=name)
        assert got.n_super == int(g[f"{name}/r{relaxation}/nSuper"])
        assert got.max_width == int(g[f"{name}/r{relaxation}/max_width"])


def test_csc_to_supernodal_medium_then_solve(cuda, oracle):
    """A 20,000-column matrix: layout equal to the CPU restatement, then analysed and solved
    from the converted arrays; new values into the same panels; malformed input is reported."""
    import torch
    from lcd_b200 import _native as nat, generators as gen, supernodal
    s = gen.supernodal_random(n=20_000, seed=11, widths=(8, 16, 32, 64), min_targets=3, max_targets=9)
    L = s.to_csc()
    L.sort_indices()
    Cp, Ci, Cx = L.indptr.astype(np.int32), L.indices.astype(np.int32), L.data
    for relaxation in (0, 2):
        got = supernodal.from_csc(Cp, Ci, Cx, relaxation=relaxation, device=cuda)
        ref = oracle.csc_to_supernodal(Cp, Ci, Cx, relaxation)
        for mine, field in ((got.sn, "supernodes"), (got.col_to_super, "col_to_super"), (got.Lip, "ip"),
                            (got.Li, "i"), (got.Lp, "p"), (got.Lx, "x")):
            np.testing.assert_array_equal(host(mine), ref[field], err_msg=field)
        plan = supernodal.analyse(got.sn, got.Lip, got.Li, got.Lp, got.Lx, got.col_to_super)
        x = host(supernodal.solve(plan, dev(s.b, np.float64, cuda)))
        np.testing.assert_allclose(x, oracle.sptrsv_csc_lower(Cp, Ci, Cx, s.b), rtol=1e-9, atol=1e-12)
    got.fill(dev(Cp, np.int32, cuda), dev(Ci, np.int32, cuda), dev(2.0 * Cx, np.float64, cuda))
    np.testing.assert_array_equal(host(got.Lx), 2.0 * ref["x"])
    empty = supernodal.from_csc(np.zeros(1, np.int32), np.zeros(0, np.int32), np.zeros(0), device=cuda)
    assert empty.n_super == 0 and empty.Lx.numel() == 0
    shuffled = Ci.copy()
    col = int(np.argmax(np.diff(Cp) >= 3))
    shuffled[Cp[col]:Cp[col] + 2] = shuffled[Cp[col]:Cp[col] + 2][::-1]
    with pytest.raises(nat.NativeError) as err:
        supernodal.from_csc(Cp, shuffled, Cx, device=cuda)
    assert err.value.code == nat.ERR_UNSORTED


# ------------------------------------------------- failure detection ----
def test_waits_are_bounded_and_errors_reported(cuda):
    """Faults are made on the host (bad counters / bad indices); the kernels give
    up after a short wall-clock budget and report a status, the context stays usable."""
    from lcd_b200 import generators as gen, ops
    from lcd_b200._native import (ERR_INDEX_RANGE, ERR_MISSING_DIAGONAL, ERR_TIMEOUT, NativeError)
    tri = gen.random_band_lower(5000, seed=9, mean_degree=8.0, band=32)
    Cp, Ci, Cx = tri.csc_arrays()
    dCp, dCi, dCx, db = dev(Cp, np.int32, cuda), dev(Ci, np.int32, cuda), dev(Cx, np.float64, cuda), dev(tri.b, np.float64, cuda)
    dep = ops.csc_edge_count(dCp, dCi)
    dep[100] += 1   # a contribution that never arrives
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csc_syncfree(dCp, dCi, dCx, db, dep, timeout_ms=300)
    assert err.value.code == ERR_TIMEOUT
    # an entry on the wrong side of the diagonal (row 10 refers to row 20)
    Ap, Ai, Ax = tri.csr_arrays()
    bad = Ai.copy()
    row = next(r for r in range(10, 100) if Ap[r + 1] - Ap[r] >= 2)
    bad[Ap[row]] = row + 10   # first off-diagonal entry now points below the diagonal
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csr_syncfree(dev(Ap, np.int32, cuda), dev(bad, np.int32, cuda), dev(Ax, np.float64, cuda),
                                db, timeout_ms=300)
    assert err.value.code == ERR_INDEX_RANGE
    # factor solve without a stored diagonal
    g = golden("ilu0_missing_diag_n90")
    Fp, Fi = dev(g["indptr"], np.int32, cuda), dev(g["indices"], np.int32, cuda)
    pos = ops.diag_positions(Fp, Fi)
    with pytest.raises(NativeError) as err:
        ops.sptrsv_csr_syncfree(Fp, Fi, dev(g["factored"], np.float64, cuda),
                                dev(np.ones(90), np.float64, cuda), diag_pos=pos, upper=True, timeout_ms=300)
    assert err.value.code == ERR_MISSING_DIAGONAL
    # the device is still healthy: a normal solve succeeds afterwards
    x = host(ops.sptrsv_csr_syncfree(dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda),
                                     dev(Ax, np.float64, cuda), db))
    assert csr_residual(Ap, Ai, Ax, x, tri.b) <= RESIDUAL_TOL
