"""The allocation-free ILU(0) entry point.

``lcd_spilu0_csr_static`` serves callers that must not allocate device memory when
they factorise (a fixed memory pool, a callback running while the allocator is held,
a loop that cannot afford a synchronising cudaMalloc): its flags and status block sit
in a fixed array inside the library.  The test drives it through the C ABI and checks
that it returns exactly what the ordinary entry point returns, twice in a row, because
the second call finds the array filled by the first.  It runs last so that a failure
here cannot hide the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _factor_static(lib, nat, Ap, Ai, Ax, pos, lanes=0, stream=None):
    import torch
    host = ctypes.c_int(-1)
    stream = ctypes.c_void_p((stream or torch.cuda.current_stream()).cuda_stream)
    rc = lib.lcd_spilu0_csr_static(Ap.numel() - 1, Ai.numel(), nat.ptr(Ap), nat.ptr(Ai),
                                   nat.ptr(Ax), nat.ptr(pos), lanes, 0, stream,
                                   ctypes.byref(host))
    return rc, host.value


def test_static_scratch_ilu0_matches_the_allocating_entry_point(cuda):
    import torch
    from lcd_b200 import _native as nat, generators as gen, ops
    lib = nat.load()
    mat, _ = gen.laplacian3d_ilu0(20, seed=4)           # 8000 rows, 7-point stencil
    rnd = gen.random_band_lower(3000, seed=5, mean_degree=10.0, band=48)
    full = (rnd.csr + rnd.csr.T).tocsr()                 # a second, irregular pattern
    full.sort_indices()
    for matrix in (mat, full):
        Ap = torch.from_numpy(matrix.indptr.astype(np.int32)).to(cuda)
        Ai = torch.from_numpy(matrix.indices.astype(np.int32)).to(cuda)
        values = torch.from_numpy(matrix.data.astype(np.float64)).to(cuda)
        pos = ops.diag_positions(Ap, Ai)
        want = ops.spilu0_csr(Ap, Ai, values.clone(), pos, mode="sync_free").cpu().numpy()
        for call in range(2):                            # the array keeps the last call's contents
            work = values.clone()
            torch.cuda.synchronize()
            # torch's counter only sees torch's own allocator; the driver's free-memory figure
            # also sees a cudaMalloc inside the library (from the second call on: the first one
            # on a device may load the module and look up the array's address)
            before = torch.cuda.memory_allocated(cuda)
            free_before = torch.cuda.mem_get_info(cuda)[0]
            rc, status = _factor_static(lib, nat, Ap, Ai, work, pos)
            assert (rc, status) == (0, 0), (call, rc, status)
            assert torch.cuda.memory_allocated(cuda) == before
            if call:
                assert torch.cuda.mem_get_info(cuda)[0] == free_before
            np.testing.assert_array_equal(work.cpu().numpy(), want)   # ILU0 parity is bit-exact
        work = values.clone()
        rc, status = _factor_static(lib, nat, Ap, Ai, work, pos, lanes=1)
        assert (rc, status) == (0, 0)
        np.testing.assert_array_equal(work.cpu().numpy(), want)
        # on a stream of the caller's own (one call at a time: the calls share the array)
        side = torch.cuda.Stream(device=cuda)
        work = values.clone()
        torch.cuda.synchronize()
        with torch.cuda.stream(side):
            rc, status = _factor_static(lib, nat, Ap, Ai, work, pos, stream=side)
        assert (rc, status) == (0, 0)
        np.testing.assert_array_equal(work.cpu().numpy(), want)


def test_static_scratch_ilu0_rejects_what_does_not_fit(cuda):
    from lcd_b200 import _native as nat
    lib = nat.load()
    host = ctypes.c_int(0)
    too_many = (1 << 20) + 1
    assert lib.lcd_spilu0_csr_static(too_many, 0, None, None, None, None, 0, 0, None,
                                     ctypes.byref(host)) == nat.ERR_TOO_LARGE
    assert lib.lcd_spilu0_csr_static(10, 10, None, None, None, None, 0, 0, None,
                                     None) == nat.ERR_INVALID_ARGUMENT
    assert lib.lcd_spilu0_csr_static(0, 0, None, None, None, None, 0, 0, None,
                                     ctypes.byref(host)) == 0 and host.value == 0
