"""The solvers that multiply by explicit inverses of diagonal blocks (block-recurrence chain
solver, supernodal solve with inverted triangles) must notice blocks whose inverse grows and
hand the solve to substitution: same residual bound (1e-12) either way."""
import numpy as np
import pytest
import scipy.sparse as sp

pytestmark = pytest.mark.gpu

RESIDUAL_TOL = 1e-12


def dev(a, dtype, device):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=dtype)).to(device)


def graded_chain(n, stretch=41, ratio=1.3, seed=0):
    """One dependence chain (n levels) whose 64-row diagonal blocks have inverses with entries
    up to ratio ** stretch: sub-diagonal -ratio inside stretches of rows, -1e-6 between them (so
    that errors do not grow from stretch to stretch), weak long-range entries, diagonal 1.  b = L x_true with x_true ~ U[-1, 1]."""
    rng = np.random.default_rng(seed)
    i = np.arange(1, n)
    sub = np.where(i % stretch == 0, -1e-6, -ratio)
    far = np.arange(200, n)
    rows = np.concatenate([i, far, np.arange(n)])
    cols = np.concatenate([i - 1, far - 200, np.arange(n)])
    vals = np.concatenate([sub, rng.uniform(-1e-7, 1e-7, len(far)), np.ones(n)])
    L = sp.csr_matrix((vals, (rows, cols)), shape=(n, n))
    L.sort_indices()
    x_true = rng.uniform(-1.0, 1.0, n)
    return L, L @ x_true, x_true


def test_chain_solver_growth_guard(cuda, oracle):
    import torch
    from lcd_b200 import generators as gen, ops
    n = 40_960
    L, b, _ = graded_chain(n)
    Ap, Ai, Ax = L.indptr.astype(np.int32), L.indices.astype(np.int32), L.data
    dAp, dAi, dAx, db = dev(Ap, np.int32, cuda), dev(Ai, np.int32, cuda), dev(Ax, np.float64, cuda), dev(b, np.float64, cuda)
    workspace = ops.chain_prepare(dAp, dAi, dAx, ops.chain_workspace(n, cuda))
    growth = ops.chain_growth(workspace, n)
    assert growth > 1e3 > ops.CHAIN_MAX_GROWTH          # inverse entries reach 1.3 ** 40 = 3.6e4
    # substitution keeps the residual bound on this matrix
    x = ops.sptrsv_csr_syncfree(dAp, dAi, dAx, db).cpu().numpy()
    assert np.linalg.norm(L @ x - b) / np.linalg.norm(b) <= RESIDUAL_TOL
    # a diagonally dominant matrix of the benchmark's kind stays far below the bound
    tri = gen.random_band_lower(40_000, seed=0, mean_degree=15.0, band=64)
    Bp, Bi, Bx = tri.csr_arrays()
    ws = ops.chain_prepare(dev(Bp, np.int32, cuda), dev(Bi, np.int32, cuda), dev(Bx, np.float64, cuda),
                           ops.chain_workspace(tri.n, cuda))
    assert 0.0 < ops.chain_growth(ws, tri.n) <= 10.0
    # non-finite tiles count as unbounded growth
    bad = Bx.copy()
    bad[Bp[1000 + 1] - 1] = 0.0                         # a zero on the diagonal
    ws = ops.chain_prepare(dev(Bp, np.int32, cuda), dev(Bi, np.int32, cuda), dev(bad, np.float64, cuda), ws)
    assert ops.chain_growth(ws, tri.n) == float("inf")
    torch.cuda.synchronize()


def test_decorated_solve_falls_back_to_substitution_on_graded_blocks(cuda):
    """Through parallel(...): a matrix with narrow levels goes to the chain solver, whose growth
    figure sends this one to the substitution kernel; the residual bound holds either way."""
    import sys, os
    sys.path.insert(0, os.path.dirname(__file__))
    from ops_decorated import csr_warp_syncfree
    from lcd_b200 import generators as gen
    n = 40_960
    L, b, _ = graded_chain(n, seed=1)
    Ap, Ai, Ax = L.indptr.astype(np.int32), L.indices.astype(np.int32), L.data
    for _ in range(2):                                    # second call: cached plan and growth figure
        x = csr_warp_syncfree(Ap, Ai, Ax, b, n)
        assert np.linalg.norm(L @ x - b) / np.linalg.norm(b) <= RESIDUAL_TOL
    tri = gen.random_band_lower(40_000, seed=2, mean_degree=15.0, band=64)   # well conditioned: chain solver
    Bp, Bi, Bx = tri.csr_arrays()
    x = csr_warp_syncfree(Bp, Bi, Bx, tri.b, tri.n)
    assert np.linalg.norm(tri.csr @ x - tri.b) / np.linalg.norm(tri.b) <= RESIDUAL_TOL


def test_supernodal_inverse_growth_guard(cuda, oracle):
    from lcd_b200 import generators as gen, supernodal
    s = gen.supernodal_random(n=4_000, seed=7, widths=(32, 64), min_targets=2, max_targets=5)
    Lx = s.Lx.copy()
    # make every diagonal block a graded bidiagonal-dominated triangle: sub-diagonal -1.4
    for k in range(len(s.sn) - 1):
        c0, w = int(s.sn[k]), int(s.sn[k + 1] - s.sn[k])
        ln = int(s.Lip[k + 1] - s.Lip[k])
        base = int(s.Lp[c0])
        for c in range(w):
            Lx[base + c * ln + c] = 1.0
            if c + 1 < w:
                Lx[base + c * ln + c + 1] = -1.4
    want = oracle.sptrsv_supernodal(s.sn, s.Lip, s.Li, s.Lp, Lx, s.b)
    plan = supernodal.analyse(s.sn, s.Lip, s.Li, s.Lp, Lx, s.col_to_super)
    assert plan.inverse_growth > 1e3 and plan.block_inverses is None      # 1.4 ** 31 and more
    x = supernodal.solve(plan, dev(s.b, np.float64, cuda)).cpu().numpy()
    np.testing.assert_allclose(x, want, rtol=1e-9, atol=1e-9 * np.max(np.abs(want)))
    good = supernodal.analyse(s.sn, s.Lip, s.Li, s.Lp, s.Lx, s.col_to_super)
    assert 0.0 < good.inverse_growth <= 10.0 and good.block_inverses is not None
