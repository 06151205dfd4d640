"""The decorator path end to end on the GPU: host NumPy in, host NumPy out, checked
against the reference fixtures, SciPy and the CPU oracle (modelled on the reference's
compiler/e2e_tests/test_sptrsv_e2e.py and test_spilu0_e2e.py)."""
import numpy as np
import pytest
import scipy.sparse as sp
from scipy.sparse.linalg import spsolve_triangular

from conftest import golden, golden_names

pytestmark = pytest.mark.gpu


def _lists(ptr, idx):
    return [idx[ptr[k]:ptr[k + 1]].tolist() for k in range(len(ptr) - 1)]


@pytest.mark.parametrize("name", ["sptrsv_lap2d_g8", "sptrsv_band_n300", "sptrsv_unsorted_dups"])
def test_inspector_outputs_equal_the_reference(cuda, name):
    import ops_decorated as od
    g = golden(name)
    csr = (g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"], len(g["b"]))
    csc = (g["csc_Ap"], g["csc_Ai"], g["csc_Ax"], g["b"], len(g["b"]))
    succ, dep = od.csr_warp_syncfree.build_dag(*csr)
    assert succ == _lists(g["csr_warp_syncfree/succ_ptr"], g["csr_warp_syncfree/succ_idx"])
    assert dep == np.bincount(g["csr_warp_syncfree/succ_idx"], minlength=len(dep)).tolist()
    succ, waves = od.simple_sptrsv_csr.build_dag(*csr)
    wp = g["csr_plain_wavefront/wavefront_ptr"]
    assert waves == _lists(wp, g["csr_plain_wavefront/wavefronts"])
    cases = [(od.csr_warp_syncfree, csr, "csr_warp_syncfree/"), (od.csr_plain_syncfree, csr, "csr_plain_syncfree/"),
             (od.simple_sptrsv_csr, csr, "csr_plain_wavefront/"), (od.csc_warp_push, csc, "csc_warp_push/"),
             (od.simple_sptrsv_csc, csc, "csc_plain_wavefront/")]
    for op, args, prefix in cases:
        if prefix + "schedule" not in g:
            continue
        plan = op.schedule_plan(*args)
        assert list(map(str, plan.schedule.lowering_key)) == g[prefix + "schedule"].tolist()
        data = plan.execution_data
        for field in ("dep_count", "initial_dep_count", "dag_ptr", "dag_index", "wavefronts", "wavefront_ptr",
                      "task_nodes", "task_ptr", "band_ptr"):
            if prefix + field in g:
                value = getattr(data, field)
                value = value.cpu().numpy() if hasattr(value, "cpu") else np.asarray(value)
                np.testing.assert_array_equal(value, g[prefix + field], err_msg=prefix + field)
                assert value.dtype == np.int32
        assert op.schedule_plan(*args) is plan            # cached by structure fingerprint
        prepared = op.prepare_cuda_arguments(*args)
        assert prepared.launcher_argument_names == tuple(op.cuda_lowering.launcher_arguments)
        assert isinstance(prepared.values["n"], (int, np.integer))


@pytest.mark.parametrize("name", golden_names("sptrsv_"))
def test_decorated_sptrsv_matches_scipy_and_reference(cuda, name):
    import ops_decorated as od
    g = golden(name)
    n = len(g["b"])
    if "csr_upper_reversed/succ_ptr" in g:
        x = od.csr_upper_reversed(g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"], n)
        np.testing.assert_allclose(x, g["x_csr"], rtol=1e-10, atol=1e-12)
        return
    L = sp.csr_matrix((g["csr_Ax"], g["csr_Ai"], g["csr_Ap"]), shape=(n, n))
    L.sum_duplicates()
    want = spsolve_triangular(L, g["b"], lower=True)
    for op in (od.simple_sptrsv_csr, od.csr_warp_syncfree, od.csr_plain_syncfree, od.csr_auto):
        b_before = g["b"].copy()
        x = op(g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"], n)
        assert isinstance(x, np.ndarray) and x.shape == (n,)
        np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)     # the reference's E2E tolerance
        np.testing.assert_allclose(x, g["x_csr"], rtol=1e-10, atol=1e-12)
        np.testing.assert_array_equal(g["b"], b_before)                   # inputs are never mutated
    for op in (od.simple_sptrsv_csc, od.csc_warp_push):
        x = op(g["csc_Ap"], g["csc_Ai"], g["csc_Ax"], g["b"], n)
        np.testing.assert_allclose(x, g["x_csc"], rtol=1e-10, atol=1e-12)
        if name != "sptrsv_unsorted_dups":      # that fixture's CSC matrix has its own values
            np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    assert od.csr_auto.current_schedule is not None and od.csr_auto.cuda_source is not None


def test_decorated_first_configuration(cuda, oracle):
    """L = tril of the 2-D 5-point Laplacian on a 256 x 256 grid through the decorated CSC demo."""
    import ops_decorated as od
    from lcd_b200 import generators as gen
    tri = gen.laplacian2d_tril(256, seed=0)
    Cp, Ci, Cx = tri.csc_arrays()
    x = od.csc_warp_push(Cp, Ci, Cx, tri.b, tri.n)
    want = spsolve_triangular(tri.csr, tri.b, lower=True)
    np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    Ap, Ai, Ax = tri.csr_arrays()
    assert oracle.relative_residual_csr(Ap, Ai, Ax, x, tri.b) <= 1e-12
    host = od.csc_warp_push.original_function(Cp, Ci, Cx, tri.b, tri.n)
    np.testing.assert_allclose(x, host, rtol=1e-10, atol=1e-12)
    plan = od.csc_warp_push.schedule_plan(Cp, Ci, Cx, tri.b, tri.n)
    assert len(plan.execution_data.band_ptr) - 1 == 511           # levels of the 256 x 256 grid


@pytest.mark.parametrize("name", ["sptrsv_lap2d_g8", "sptrsv_band_n600", "sptrsv_lap3d_g5", "sptrsv_unsorted_dups"])
def test_decorated_band_chains(cuda, name):
    """band_width > 1 (compiler/dag_preprocessing.py:207-298): tasks are chains of nodes connected
    inside a band of consecutive levels; a lane group solves a chain node after node, bands are
    separated like levels.  Same results as every other schedule."""
    import ops_decorated as od
    from lcd_b200.dag_preprocessing import preprocess_warp_tasks
    g = golden(name)
    n = len(g["b"])
    csr = (g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"], n)
    csc = (g["csc_Ap"], g["csc_Ai"], g["csc_Ax"], g["b"], n)
    data = od.csr_warp_wavefront_band2.schedule_plan(*csr).execution_data
    succ, waves = od.simple_sptrsv_csr.build_dag(*csr)
    want = preprocess_warp_tasks(succ, waves, band_width=2)               # list form (host logic tests pin it)
    to_host = lambda a: a.cpu().numpy() if hasattr(a, "cpu") else np.asarray(a)   # built on the device
    np.testing.assert_array_equal(to_host(data.task_nodes), want.task_nodes)
    np.testing.assert_array_equal(to_host(data.task_ptr), want.task_ptr)
    np.testing.assert_array_equal(to_host(data.band_ptr), want.band_ptr)
    assert len(data.task_ptr) - 1 < n or len(waves) == n                  # chains do form
    x = od.csr_warp_wavefront_band2(*csr)
    np.testing.assert_allclose(x, g["x_csr"], rtol=1e-10, atol=1e-12)
    x = od.csc_warp_wavefront_band3(*csc)
    np.testing.assert_allclose(x, g["x_csc"], rtol=1e-10, atol=1e-12)


@pytest.mark.parametrize("name", golden_names("gauss_seidel_"))
def test_decorated_gauss_seidel_matches_the_reference(cuda, oracle, name):
    """The reference's Gauss-Seidel demo operators (compiler/demo/gauss_seidel.py:18-41), inputs
    built as compiler/e2e_tests/test_gauss_seidel_e2e.py:57-84 does; inspector arrays against
    the reference's, results against its undecorated loops (rtol 1e-10 / atol 1e-12)."""
    import ops_decorated as od
    g = golden(name)
    n, sweeps = len(g["b"]), int(g["max_iter"])
    simple = (g["simple_Ap"], g["simple_Ai"], g["simple_Ax"], g["D"], g["b"], g["x0"].copy(), n, sweeps)
    full = (g["full_Ap"], g["full_Ai"], g["full_Ax"], g["b"], g["x0"].copy(), n, sweeps)
    for op, args, prefix in ((od.simple_gauss_seidel_csr, simple, "simple/"), (od.full_gauss_seidel_csr, full, "full/")):
        succ, waves = op.build_dag(*args)
        assert succ == _lists(g[prefix + "succ_ptr"], g[prefix + "succ_idx"])
        assert waves == _lists(g[prefix + "wavefront_ptr"], g[prefix + "wavefronts"])
        plan = op.schedule_plan(*args)
        assert list(map(str, plan.schedule.lowering_key)) == g[prefix + "schedule"].tolist()
        np.testing.assert_array_equal(plan.execution_data.wavefronts.cpu().numpy(), g[prefix + "wavefronts"])
    x0 = simple[5].copy()
    x = od.simple_gauss_seidel_csr(*simple)
    np.testing.assert_allclose(x, g["x_simple"], rtol=1e-10, atol=1e-12)
    np.testing.assert_array_equal(simple[5], x0)                       # arguments are never mutated
    x = od.full_gauss_seidel_csr(*full)
    np.testing.assert_allclose(x, g["x_full"], rtol=1e-10, atol=1e-12)
    x = od.full_gauss_seidel_csr_syncfree(*full)
    np.testing.assert_allclose(x, g["x_full"], rtol=1e-10, atol=1e-12)
    # zero sweeps return the start vector, one sweep already is the triangular solve
    start = np.linspace(-1.0, 1.0, n)
    np.testing.assert_array_equal(od.full_gauss_seidel_csr(*full[:4], start, n, 0), start)
    np.testing.assert_allclose(od.full_gauss_seidel_csr(*full[:4], start, n, 1), g["x_full"], rtol=1e-10, atol=1e-12)
    # new values on the same structure (plan and layout are reused, values converted again)
    D2 = g["D"] * 2.0
    want = oracle.gauss_seidel_simple_csr(g["simple_Ap"], g["simple_Ai"], g["simple_Ax"], D2, g["b"], g["x0"], sweeps)
    got = od.simple_gauss_seidel_csr(g["simple_Ap"], g["simple_Ai"], g["simple_Ax"], D2, g["b"], g["x0"].copy(), n, sweeps)
    np.testing.assert_allclose(got, want, rtol=1e-10, atol=1e-12)


def test_gauss_seidel_layout_edge_cases(cuda, oracle):
    """Unsorted rows, repeated and missing diagonal entries, and entries right of the diagonal."""
    from lcd_b200 import ops
    from lcd_b200._native import ERR_INDEX_RANGE, NativeError
    import torch
    rows = [[0], [1, 0], [0], [3, 1, 3, 0], [2, 4, 2], [], [5, 6, 0, 3]]      # row 2 and 5: no diagonal
    Ap = np.cumsum([0] + [len(r) for r in rows]).astype(np.int32)
    Ai = np.asarray([c for r in rows for c in r], dtype=np.int32)
    rng = np.random.default_rng(0)
    Ax = rng.uniform(1.0, 2.0, len(Ai))
    b = rng.uniform(-1, 1, len(rows))
    dev = lambda a, t: torch.from_numpy(np.ascontiguousarray(a, dtype=t)).to(cuda)
    layout = ops.gs_layout(dev(Ap, np.int32), dev(Ai, np.int32), separate_diagonal=False)
    values = ops.gs_values(layout, dev(Ax, np.float64))
    x = ops.sptrsv_csr_syncfree(layout.Ap, layout.Ai, values, dev(b, np.float64), exact=True).cpu().numpy()
    want = oracle.gauss_seidel_full_csr(Ap, Ai, Ax, b, np.zeros(len(rows)), 1)
    np.testing.assert_allclose(x, want, rtol=1e-13, atol=1e-15)
    hAp, hAi = layout.Ap.cpu().numpy(), layout.Ai.cpu().numpy()
    assert hAp.tolist() == [0, 1, 3, 5, 8, 11, 12, 16] and layout.nnz == 16
    assert all(hAi[hAp[i + 1] - 1] == i for i in range(len(rows)))            # diagonal last
    assert layout.perm.cpu().numpy()[:len(Ai)].tolist()[4:8] == [-1, 5, 7, 6]   # the later diagonal entry wins
    bad = Ai.copy()
    bad[1] = 4                                                                 # right of the diagonal
    with pytest.raises(NativeError) as err:
        ops.gs_layout(dev(Ap, np.int32), dev(bad, np.int32), separate_diagonal=False)
    assert err.value.code == ERR_INDEX_RANGE
    with pytest.raises(NativeError) as err:                                    # a diagonal entry in "separate" form
        ops.gs_layout(dev(Ap, np.int32), dev(Ai, np.int32), separate_diagonal=True)
    assert err.value.code == ERR_INDEX_RANGE
    empty = ops.gs_layout(dev([0], np.int32), dev([], np.int32), separate_diagonal=True)
    assert empty.nnz == 0


def test_demos_on_a_matrix_market_file(cuda, tmp_path, capsys):
    """The three demos end to end on a file (the reference's E2E tests load theirs the same way,
    compiler/e2e_tests/gpu_test_utils.py:24-33): CSR and CSC solves against SciPy, ILU0 and the
    Gauss-Seidel sweeps against the sequential loops, and the command line."""
    import scipy.sparse as sp
    from lcd_b200 import demos
    from lcd_b200.matrix_market import write_matrix_market
    rng = np.random.default_rng(5)
    pattern = sp.random(300, 300, density=0.03, random_state=6, format="csr")
    pattern = pattern + pattern.T + sp.identity(300)
    pattern.data = rng.uniform(-5.0, 5.0, pattern.nnz)
    path = tmp_path / "synthetic.mtx"
    write_matrix_market(path, pattern)
    solves = demos.run_sptrsv(path, 0, "both")
    np.testing.assert_allclose(solves["csr"], np.linspace(1.0, 2.0, 300), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(solves["csc"], solves["csr"], rtol=1e-10, atol=1e-12)
    assert demos.run_sptrsv(path, 128, "csr")["csr"].shape == (128,)          # leading principal sample
    for mode in ("wavefront", "sync_free"):
        factors = demos.run_spilu0(path, 0, mode, storage="both")
        # the same matrix factored by rows and by columns: the same values, entry by entry
        n = 300
        by_rows = sp.csr_matrix((factors["csr"], *_pattern(path, "csr")), shape=(n, n))
        by_cols = sp.csc_matrix((factors["csc"], *_pattern(path, "csc")), shape=(n, n))
        assert (by_rows != sp.csr_matrix(by_cols)).nnz == 0
    sweeps = demos.run_gauss_seidel(path, 0, "both", 2)
    np.testing.assert_allclose(sweeps["simple"], np.linspace(1.0, 2.0, 300), rtol=1e-10, atol=1e-12)
    np.testing.assert_allclose(sweeps["full"], sweeps["simple"], rtol=1e-10, atol=1e-12)
    demos.main(["gauss-seidel", str(path), "--max-n", "64", "--variant", "full", "--iterations", "3"])
    printed = capsys.readouterr().out
    errors = [float(line.rsplit("=", 1)[1]) for line in printed.splitlines() if "max_abs_error" in line]
    assert len(errors) == 10 and max(errors) <= 1e-12
    with pytest.raises(SystemExit):
        demos.main(["sptrsv", str(path), "--max-n", "-1"])


def test_decorated_narrow_levels_take_the_chain_solver(cuda, oracle, monkeypatch):
    """A long dependence chain (5-6 rows per level) through the decorator: the inspector's level
    count sends the sync-free launcher to the block-recurrence chain solver; the block tiles are
    rebuilt when the values change and only then."""
    import ops_decorated as od
    from lcd_b200 import generators as gen, ops
    tri = gen.random_band_lower(65_536, seed=3)
    Ap, Ai, Ax = tri.csr_arrays()
    # "prepare": preparation + solve pipelined over row ranges (new values); "solve": a solve in
    # one piece on tiles that are kept
    calls = {"prepare": 0, "solve": 0}
    real_pipeline, real_solve = ops.chain_prepare_and_solve, ops.sptrsv_csr_chain

    def counted_pipeline(*a, **k):          # (65,536 rows are one piece: it solves in one call)
        calls["prepare"] += 1
        return real_pipeline(*a, **k)

    def counted_solve(*a, **k):
        if k.get("rows") is None:
            calls["solve"] += 1
        return real_solve(*a, **k)
    monkeypatch.setattr(ops, "chain_prepare_and_solve", counted_pipeline)
    monkeypatch.setattr(ops, "sptrsv_csr_chain", counted_solve)
    plan = od.csr_warp_syncfree.schedule_plan(Ap, Ai, Ax, tri.b, tri.n)
    assert plan.rows == tri.n and plan.rows / plan.levels < 64
    want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
    x = od.csr_warp_syncfree(Ap, Ai, Ax, tri.b, tri.n)
    np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)         # the reference's E2E tolerance
    assert oracle.relative_residual_csr(Ap, Ai, Ax, x, tri.b) <= 1e-12
    assert calls == {"prepare": 1, "solve": 1}
    x2 = od.csr_warp_syncfree(Ap, Ai, Ax, tri.b, tri.n)                 # same values: tiles are kept
    # (operands from earlier chunks are subtracted in the order they arrive, so two runs may
    # differ in the last bits; LCD_SOLVE_EXACT is the bit-reproducible path)
    np.testing.assert_allclose(x2, x, rtol=1e-13, atol=1e-15)
    assert calls == {"prepare": 1, "solve": 2}
    Ax2 = Ax.copy()
    Ax2[Ap[1:] - 1] *= 2.0                                               # new diagonal: tiles rebuilt
    x3 = od.csr_warp_syncfree(Ap, Ai, Ax2, tri.b, tri.n)
    np.testing.assert_allclose(x3, oracle.sptrsv_csr_lower(Ap, Ai, Ax2, tri.b), rtol=1e-10, atol=1e-12)
    assert calls == {"prepare": 2, "solve": 3}
    # small systems and wide levels stay on the polling kernel
    grid = gen.laplacian2d_tril(64, seed=0)
    od.csr_warp_syncfree(*grid.csr_arrays(), grid.b, grid.n)
    assert calls["solve"] == 3


def test_decorated_wide_levels_take_the_shared_level_walk(cuda, oracle, monkeypatch):
    """A 3-D grid with hundreds of rows per level through the decorator: the sync-free launcher
    walks the levels with one thread block per node range; the coefficients are gathered into
    slot order on the first call and again only when the values change."""
    import ops_decorated as od
    from lcd_b200 import generators as gen, ops
    tri = gen.laplacian3d_tril(48, seed=2)
    Ap, Ai, Ax = tri.csr_arrays()
    seen = []
    real = ops.sptrsv_small

    def counted(plan, *a, **k):
        seen.append((plan.blocks, bool(k.get("same_values"))))
        return real(plan, *a, **k)
    monkeypatch.setattr(ops, "sptrsv_small", counted)
    for op in (od.csr_warp_syncfree, od.csr_plain_syncfree):
        seen.clear()
        x = op(Ap, Ai, Ax, tri.b, tri.n)
        np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b), rtol=1e-10, atol=1e-12)
        assert oracle.relative_residual_csr(Ap, Ai, Ax, x, tri.b) <= 1e-12
        b2 = tri.b[::-1].copy()
        x2 = op(Ap, Ai, Ax, b2, tri.n)                                     # same matrix, new right-hand side
        np.testing.assert_allclose(x2, oracle.sptrsv_csr_lower(Ap, Ai, Ax, b2), rtol=1e-10, atol=1e-12)
        Ax3 = Ax * 1.5
        x3 = op(Ap, Ai, Ax3, tri.b, tri.n)                                 # new values: gathered again
        np.testing.assert_allclose(x3, oracle.sptrsv_csr_lower(Ap, Ai, Ax3, tri.b), rtol=1e-10, atol=1e-12)
        assert [same for _, same in seen] == [False, True, False]
        assert all(blocks >= 8 for blocks, _ in seen)


def _pattern(path, storage):
    from lcd_b200.matrix_market import load_matrix_market
    matrix = load_matrix_market(path, 0)
    matrix = sp.csr_matrix(matrix) if storage == "csr" else sp.csc_matrix(matrix)
    matrix.sort_indices()
    return matrix.indices, matrix.indptr


@pytest.mark.parametrize("mode", ["wavefront", "sync_free"])
@pytest.mark.parametrize("name", golden_names("csc_ilu0_"))
def test_decorated_ilu0_on_csc_storage_is_bit_identical(cuda, name, mode):
    """The column loop of compiler/demo/spilu0.py:50-82 through the decorator."""
    import ops_decorated as od
    g = golden(name)
    op = od.compile_ilu0_csc(mode, 128)
    out = op(g["data"].copy(), g["indices"], g["indptr"])
    np.testing.assert_array_equal(out, g["factored"])
    np.testing.assert_array_equal(out, od.ilu0_csc(g["data"].copy(), g["indices"], g["indptr"]))
    again = op(g["data"].copy(), g["indices"], g["indptr"])     # cached plan and row view
    np.testing.assert_array_equal(again, g["factored"])


def test_decorated_chain_solve_follows_a_streamed_upload(cuda, oracle, monkeypatch):
    """Page-locked value arrays above the streaming threshold are uploaded in pieces; the chain
    solver's launcher prepares and solves the rows of each piece as it arrives.  Other launchers
    (and smaller arrays) see the whole array as before."""
    import torch
    import ops_decorated as od
    import lcd_b200.cuda_runtime as rt
    from lcd_b200 import generators as gen, ops
    monkeypatch.setattr(rt, "STREAMED_UPLOAD_BYTES", 1 << 20)
    tri = gen.random_band_lower(65_536, seed=5)
    Ap, Ai, Ax = tri.csr_arrays()
    pinned = torch.from_numpy(Ax).pin_memory().numpy()         # 8 MB: eight pieces
    ranges = []
    real_solve = ops.sptrsv_csr_chain
    monkeypatch.setattr(ops, "sptrsv_csr_chain",
                        lambda *a, **k: (ranges.append(k.get("rows")), real_solve(*a, **k))[1])
    want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
    x = od.csr_warp_syncfree(Ap, Ai, pinned, tri.b, tri.n)
    np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    assert len(ranges) >= 4 and ranges[0][0] == 0 and ranges[-1][1] == tri.n
    assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
    ranges.clear()
    x = od.csr_warp_syncfree(Ap, Ai, Ax, tri.b, tri.n)          # pageable values: one piece
    np.testing.assert_allclose(x, want, rtol=1e-10, atol=1e-12)
    assert ranges == [None]
    # a launcher that does not follow the pieces waits for the whole array
    grid = gen.laplacian2d_tril(300, seed=1)
    gp, gi, gx = grid.csr_arrays()
    monkeypatch.setattr(rt, "STREAMED_UPLOAD_BYTES", 1 << 18)
    x = od.csr_warp_syncfree(gp, gi, torch.from_numpy(gx).pin_memory().numpy(), grid.b, grid.n)
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(gp, gi, gx, grid.b), rtol=1e-10, atol=1e-12)


def test_decorated_chain_solve_starts_under_the_previous_plan(cuda, oracle, monkeypatch):
    """A call whose page-locked arrays have the lengths of the previous call's starts under that
    call's plan, with the column indices uploaded side by side with the values; the structure
    fingerprint is compared after the launch, and a call with another structure is run again
    under its own plan."""
    import torch
    import ops_decorated as od
    import lcd_b200.cuda_runtime as rt
    from lcd_b200 import generators as gen, ops
    monkeypatch.setattr(rt, "STREAMED_UPLOAD_BYTES", 1 << 19)
    pin = lambda a: torch.from_numpy(np.ascontiguousarray(a)).pin_memory().numpy()
    tri = gen.random_band_lower(262_144, seed=5)      # (a right-hand side of 2 MB)
    Ap, Ai, Ax = (pin(a) for a in tri.csr_arrays())
    op = od.csr_warp_syncfree
    want = oracle.sptrsv_csr_lower(Ap, Ai, Ax, tri.b)
    np.testing.assert_allclose(op(Ap, Ai, Ax, tri.b, tri.n), want, rtol=1e-10, atol=1e-12)
    together, plans = [], []
    real_together = rt.TorchCUDA.to_device_together
    monkeypatch.setattr(rt.TorchCUDA, "to_device_together",
                        staticmethod(lambda arrays, **kw: (together.append(len(arrays)), real_together(arrays, **kw))[1]))
    real_dag = ops.dag_build
    monkeypatch.setattr(ops, "dag_build", lambda *a, **k: (plans.append(1), real_dag(*a, **k))[1])
    # same structure, new values: one side-by-side upload of indices and values, no new plan
    Ax2 = pin(Ax * 1.25)
    x = op(Ap, Ai, Ax2, tri.b, tri.n)
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax2, tri.b), rtol=1e-10, atol=1e-12)
    assert 2 in together and not plans
    # the right-hand side went in two parts around the first pieces of the matrix, and the result
    # came back range by range
    sent = []
    real_split = rt.TorchCUDA.to_device_split
    monkeypatch.setattr(rt.TorchCUDA, "to_device_split",
                        staticmethod(lambda array, head: (sent.append(head), real_split(array, head))[1]))
    early = []
    real_rows = rt.DeviceArray.download_rows
    monkeypatch.setattr(rt.DeviceArray, "download_rows",
                        lambda self, lo, hi: (early.append((lo, hi)), real_rows(self, lo, hi))[1])
    b2 = pin(tri.b * 0.5)
    x = op(Ap, Ai, Ax2, b2, tri.n)
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai, Ax2, b2), rtol=1e-10, atol=1e-12)
    assert sent == [tri.n // 16] and early and early[0][0] == 0 and early[-1][1] == tri.n
    # another structure of the same lengths
    Ai3 = Ai.copy()
    for r in range(40_000, 40_100):
        lo = Ap[r]                                # (the row's first column moves one to the left)
        if Ap[r + 1] - 1 - lo >= 1 and Ai3[lo] > 0:
            Ai3[lo] -= 1
    assert not np.array_equal(Ai3, Ai)
    Ai3 = pin(Ai3)
    together.clear()
    x = op(Ap, Ai3, Ax, tri.b, tri.n)
    np.testing.assert_allclose(x, oracle.sptrsv_csr_lower(Ap, Ai3, Ax, tri.b), rtol=1e-10, atol=1e-12)
    assert 2 in together and plans                # predicted, found different, planned afresh
    # and back: the first structure's plan is still cached, the prediction (now the third
    # structure's plan) is wrong again
    plans.clear()
    np.testing.assert_allclose(op(Ap, Ai, Ax, tri.b, tri.n), want, rtol=1e-10, atol=1e-12)
    assert not plans


@pytest.mark.parametrize("mode", ["wavefront", "sync_free"])
@pytest.mark.parametrize("name", golden_names("ilu0_"))
def test_decorated_ilu0_is_bit_identical(cuda, name, mode):
    import ops_decorated as od
    g = golden(name)
    op = od.compile_ilu0_csr(mode, 128, 1)
    data = g["data"].copy()
    out = op(data, g["indices"], g["indptr"])
    np.testing.assert_array_equal(out, g["factored"])
    np.testing.assert_array_equal(data, g["data"])                 # the caller's array is not modified
    np.testing.assert_array_equal(out, od.ilu0_csr(g["data"].copy(), g["indices"], g["indptr"]))
    assert op.current_schedule.execution_mode == mode
    data_obj = op.build_execution_data(g["data"].copy(), g["indices"], g["indptr"])
    table = data_obj.auxiliary_values["_lcd_lookup_position_0"]
    np.testing.assert_array_equal(table.cpu().numpy(), g["diag_pos"])


def test_structural_lookup_errors_surface_as_in_the_reference(cuda):
    import ops_decorated as od
    from lcd_b200.structural_lookups import StructuralLookupError
    op = od.compile_ilu0_csr("sync_free", 128, 1)
    indptr = np.array([0, 2, 4], np.int32)
    indices = np.array([1, 0, 0, 1], np.int32)        # first row unsorted
    with pytest.raises(StructuralLookupError):
        op(np.ones(4), indices, indptr)
