"""The CPU oracle against fixtures produced by the reference's own pipeline."""
import os
import numpy as np
import pytest

from conftest import golden, golden_names

SPTRSV = golden_names("sptrsv_")
ILU = golden_names("ilu0_")
SUPER = golden_names("supernodal_")


def _check_dag(d, g, prefix, edge_multiplicity=False):
    np.testing.assert_array_equal(d.dag_ptr, g[prefix + "succ_ptr"])
    np.testing.assert_array_equal(d.dag_index, g[prefix + "succ_idx"])
    if prefix + "dag_ptr" in g:
        np.testing.assert_array_equal(d.dag_ptr, g[prefix + "dag_ptr"])
        np.testing.assert_array_equal(d.dag_index, g[prefix + "dag_index"])
    if prefix + "dep_count" in g:
        want = d.edge_count if edge_multiplicity else d.dep_count
        np.testing.assert_array_equal(want, g[prefix + "dep_count"])
        np.testing.assert_array_equal(want, g[prefix + "initial_dep_count"])
    if prefix + "wavefronts" in g:
        np.testing.assert_array_equal(d.wavefronts, g[prefix + "wavefronts"])
        np.testing.assert_array_equal(d.wavefront_ptr, g[prefix + "wavefront_ptr"])
    if prefix + "task_nodes" in g:
        np.testing.assert_array_equal(d.wavefronts, g[prefix + "task_nodes"])
        np.testing.assert_array_equal(d.wavefront_ptr, g[prefix + "band_ptr"])
        np.testing.assert_array_equal(np.arange(len(d.dep_count) + 1), g[prefix + "task_ptr"])
    assert not d.cyclic


@pytest.mark.parametrize("name", SPTRSV)
def test_dag_arrays_match_reference(oracle, name):
    g = golden(name)
    if "csr_upper_reversed/succ_ptr" in g:
        d = oracle.dag_build("csr_upper", g["csr_Ap"], g["csr_Ai"])
        _check_dag(d, g, "csr_upper_reversed/")
        return
    d = oracle.dag_build("csr_lower", g["csr_Ap"], g["csr_Ai"])
    for variant in ("csr_warp_syncfree/", "csr_plain_wavefront/", "csr_plain_syncfree/"):
        if variant + "succ_ptr" in g:
            _check_dag(d, g, variant)
    d = oracle.dag_build("csc_lower", g["csc_Ap"], g["csc_Ai"])
    _check_dag(d, g, "csc_warp_push/", edge_multiplicity=True)
    _check_dag(d, g, "csc_plain_wavefront/")
    if "levels_ptr" in g:
        np.testing.assert_array_equal(d.wavefronts, g["levels_idx"])
        np.testing.assert_array_equal(d.wavefront_ptr, g["levels_ptr"])


@pytest.mark.parametrize("name", SPTRSV)
def test_sptrsv_matches_undecorated_reference(oracle, name):
    g = golden(name)
    if "csr_upper_reversed/succ_ptr" in g:
        x = oracle.sptrsv_csr_upper(g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"])
        np.testing.assert_array_equal(x, g["x_csr"])  # same arithmetic, same order: bit-exact
        return
    x = oracle.sptrsv_csr_lower(g["csr_Ap"], g["csr_Ai"], g["csr_Ax"], g["b"])
    np.testing.assert_array_equal(x, g["x_csr"])
    x = oracle.sptrsv_csc_lower(g["csc_Ap"], g["csc_Ai"], g["csc_Ax"], g["b"])
    np.testing.assert_array_equal(x, g["x_csc"])


@pytest.mark.parametrize("name", golden_names("gauss_seidel_"))
def test_gauss_seidel_matches_reference(oracle, name):
    """Inspector arrays and sweep results of the reference's Gauss-Seidel demo operators."""
    g = golden(name)
    for variant in ("simple", "full"):
        d = oracle.dag_build("csr_lower_rows", g[variant + "_Ap"], g[variant + "_Ai"])
        _check_dag(d, g, variant + "/")
    sweeps = int(g["max_iter"])
    x = oracle.gauss_seidel_simple_csr(g["simple_Ap"], g["simple_Ai"], g["simple_Ax"], g["D"], g["b"],
                                       g["x0"], sweeps)
    np.testing.assert_array_equal(x, g["x_simple"])     # same arithmetic, same order: bit-exact
    x = oracle.gauss_seidel_full_csr(g["full_Ap"], g["full_Ai"], g["full_Ax"], g["b"], g["x0"], sweeps)
    np.testing.assert_array_equal(x, g["x_full"])
    # no sweep leaves the start vector alone; sweeps of a triangular system repeat themselves
    start = np.linspace(-1.0, 1.0, len(g["b"]))
    np.testing.assert_array_equal(
        oracle.gauss_seidel_full_csr(g["full_Ap"], g["full_Ai"], g["full_Ax"], g["b"], start, 0), start)
    np.testing.assert_array_equal(
        oracle.gauss_seidel_full_csr(g["full_Ap"], g["full_Ai"], g["full_Ax"], g["b"], start, 1), g["x_full"])


@pytest.mark.parametrize("name", golden_names("csc_ilu0_"))
def test_ilu0_on_csc_storage_matches_reference(oracle, name):
    """The column loop of compiler/demo/spilu0.py:50-82; it gives, entry by entry, the values of
    the row loop on the same matrix (which is how the native path serves it) - except where a
    pivot row stores an explicit zero."""
    import scipy.sparse as sp
    g = golden(name)
    out = oracle.ilu0_csc(g["indptr"], g["indices"], g["data"])
    np.testing.assert_array_equal(out, g["factored"])
    n = len(g["indptr"]) - 1
    csc = sp.csc_matrix((np.arange(1, len(g["data"]) + 1.0), g["indices"], g["indptr"]), shape=(n, n))
    csr = sp.csr_matrix(csc)
    csr.sort_indices()
    position = csr.data.astype(np.int64) - 1                   # row order -> column order
    by_rows = oracle.ilu0_csr(csr.indptr, csr.indices, g["data"][position])
    back = np.empty_like(by_rows)
    back[position] = by_rows
    if name.endswith("stored_zeros_n60"):
        # the one place where the two loops differ: the column loop skips an explicitly stored
        # zero of the pivot row, the row loop multiplies by it (inf * 0 = NaN in this matrix);
        # the native path serves the column form with that rule switched on
        assert np.isnan(back).any() and not np.isnan(g["factored"]).any()
    else:
        np.testing.assert_array_equal(back, g["factored"])


@pytest.mark.parametrize("name", ILU)
def test_ilu0_matches_reference(oracle, name):
    g = golden(name)
    pos, rc = oracle.diag_positions(g["indptr"], g["indices"])
    assert rc == 0
    np.testing.assert_array_equal(pos, g["diag_pos"])
    np.testing.assert_array_equal(pos, g["ilu_syncfree/aux__lcd_lookup_position_0"])
    out = oracle.ilu0_csr(g["indptr"], g["indices"], g["data"])
    np.testing.assert_array_equal(out, g["factored"])
    fast = oracle.ilu0_csr(g["indptr"], g["indices"], g["data"], fast=True)
    np.testing.assert_array_equal(fast, g["factored"])
    d = oracle.dag_build("ilu0_csr", g["indptr"], g["indices"])
    _check_dag(d, g, "ilu_syncfree/")
    _check_dag(d, g, "ilu_wavefront/")


@pytest.mark.parametrize("name", SUPER)
def test_supernodal_matches_reference(oracle, name):
    g = golden(name)
    x = oracle.sptrsv_supernodal(g["sn"], g["Lip"], g["Li"], g["Lp"], g["Lx"], g["b"])
    np.testing.assert_allclose(x, g["x"], rtol=1e-14, atol=1e-15)


def test_reference_unit_test_vectors(oracle):
    # compiler/transform_tests/test_dag_codegen.py:113-167 (CSR and CSC, one repeated entry)
    d = oracle.dag_build("csr_lower", [0, 1, 3, 6, 9], [0, 0, 1, 0, 1, 2, 1, 2, 3])
    np.testing.assert_array_equal(d.dep_count, [0, 1, 2, 2])
    np.testing.assert_array_equal(d.dag_ptr, [0, 2, 4, 5, 5])
    np.testing.assert_array_equal(d.dag_index, [1, 2, 2, 3, 3])
    d = oracle.dag_build("csc_lower", [0, 4, 7, 9, 10], [0, 1, 2, 2, 1, 2, 3, 2, 3, 3])
    np.testing.assert_array_equal(d.dep_count, [0, 1, 2, 2])
    np.testing.assert_array_equal(d.dag_index, [1, 2, 2, 3, 3])
    # :204-226 wavefronts of the CSC chain
    d = oracle.dag_build("csc_lower", [0, 3, 6, 8, 9], [0, 1, 2, 1, 2, 3, 2, 3, 3])
    np.testing.assert_array_equal(d.wavefronts, [0, 1, 2, 3])
    np.testing.assert_array_equal(d.wavefront_ptr, [0, 1, 2, 3, 4])
    # compiler/transform_tests/test_spilu0_codegen.py:159-167 dense 3x3
    d = oracle.dag_build("ilu0_csr", [0, 3, 6, 9], [0, 1, 2, 0, 1, 2, 0, 1, 2])
    np.testing.assert_array_equal(d.dep_count, [0, 1, 2])
    np.testing.assert_array_equal(d.dag_index, [1, 2, 2])
    # compiler/transform_tests/test_structural_lookups.py:64-92
    pos, rc = oracle.diag_positions([0, 2, 3, 5], [0, 2, 0, 1, 2])
    assert rc == 0
    np.testing.assert_array_equal(pos, [0, -1, 4])
    _, rc = oracle.diag_positions([0, 2], [1, 0])
    assert rc == 2  # unsorted segment -> StructuralLookupError in the reference


def _conversion_cases():
    g = np.load(os.path.join(os.path.dirname(__file__), "golden", "csc_to_supernodal.npz"))
    names = sorted({k.split("/")[0] for k in g.files})
    return g, names


@pytest.mark.parametrize("relaxation", [0, 1, 3])
def test_csc_to_supernodal_matches_reference_converter(oracle, relaxation):
    """The restated converter against what utils/symbolic_cholesky_csc.py:950-1021 returned."""
    g, names = _conversion_cases()
    for name in names:
        got = oracle.csc_to_supernodal(g[f"{name}/indptr"], g[f"{name}/indices"], g[f"{name}/data"],
                                       relaxation)
        for field in ("i", "ip", "p", "supernodes", "col_to_super"):
            np.testing.assert_array_equal(got[field], g[f"{name}/r{relaxation}/{field}"], err_msg=f"{name} {field}")
        np.testing.assert_array_equal(got["x"], g[f"{name}/r{relaxation}/x"])
        assert got["nSuper"] == int(g[f"{name}/r{relaxation}/nSuper"])
        assert got["max_width"] == int(g[f"{name}/r{relaxation}/max_width"])
