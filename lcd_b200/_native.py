"""ctypes binding of ``liblcd_b200.so`` (the C ABI declared in ``include/lcd_b200.h``).

There is no CPU fallback: if the CUDA library has not been built, or a call
returns a non-zero code, this module raises.
"""

from __future__ import annotations

import ctypes
import os
from ctypes import c_double, c_int, c_int32, c_int64, c_uint64, c_void_p

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liblcd_b200.so")

# LCD_* codes of include/lcd_b200.h
OK, ERR_INVALID_ARGUMENT, ERR_CUDA, ERR_WORKSPACE, ERR_TIMEOUT, ERR_UNSORTED, \
    ERR_BAD_POINTERS, ERR_INDEX_RANGE, ERR_CYCLE, ERR_MISSING_DIAGONAL, ERR_TOO_LARGE, \
    ERR_LEVEL_CAP = range(12)
(OP_CSR_LOWER, OP_CSC_LOWER, OP_ILU0_CSR, OP_CSR_UPPER, OP_CSC_UPPER, OP_CSR_LOWER_ROWS,
 OP_CSR_UPPER_ROWS) = range(7)
SOLVE_UPPER, SOLVE_UNIT_DIAG, SOLVE_OF_FULL, SOLVE_EXACT = 1, 2, 4, 8
WAVEFRONT_PER_LEVEL, WAVEFRONT_COOPERATIVE = 0, 1
STATUS_WORDS = 8
ILU0_SKIP_STORED_ZEROS = 8      # LCD_ILU0_SKIP_STORED_ZEROS
CHAIN_MAX_GROWTH = 100.0        # LCD_CHAIN_MAX_GROWTH
(TUNE_SLEEP_LOCAL_NS, TUNE_SLEEP_GLOBAL_NS, TUNE_GAP_NS, TUNE_ROW_VARIANT, TUNE_STAGE_PERCENT,
 TUNE_CHAIN_CLUSTER, TUNE_ORDERED_PAUSE_NS, TUNE_SMALL_THREADS, TUNE_ILU0_LOOKAHEAD,
 TUNE_ORDERED_MIN_LANES) = range(10)


class NativeLibraryMissing(RuntimeError):
    """The CUDA library is not built; there is no other implementation."""


class NativeError(RuntimeError):
    """A C-ABI call returned a non-zero LCD_* code."""

    def __init__(self, code, where, detail=""):
        self.code = int(code)
        self.where = where
        super().__init__(f"{where}: LCD error {code} ({detail})")


_P = c_void_p
_SIGNATURES = {
    # name: (restype, argtypes)
    "lcd_error_string": (ctypes.c_char_p, [c_int]),
    "lcd_last_cuda_error": (ctypes.c_char_p, []),
    "lcd_version": (c_int, []),
    "lcd_read_status": (c_int, [_P, _P, ctypes.POINTER(c_int32)]),
    "lcd_dag_workspace_bytes": (c_int, [c_int, c_int32, c_int64, ctypes.POINTER(c_int64)]),
    "lcd_dag_build": (c_int, [c_int, c_int32, _P, _P, c_int64, _P, _P, _P, _P,
                              ctypes.POINTER(c_int64), _P, _P, _P, ctypes.POINTER(c_int32),
                              _P, c_int64, c_int32, _P]),
    "lcd_band_chains_workspace_bytes": (c_int, [c_int32, ctypes.POINTER(c_int64)]),
    "lcd_band_chains": (c_int, [c_int32, _P, _P, _P, _P, _P, c_int32, c_int32, _P, _P, _P,
                                ctypes.POINTER(c_int32), _P, c_int64, _P]),
    "lcd_dag_build_capped": (c_int, [c_int, c_int32, _P, _P, c_int64, _P, _P, _P, _P,
                                     ctypes.POINTER(c_int64), _P, _P, _P, ctypes.POINTER(c_int32),
                                     c_int32, _P, c_int64, c_int32, _P]),
    "lcd_diag_positions": (c_int, [c_int32, _P, _P, c_int64, _P, _P, _P, ctypes.POINTER(c_int)]),
    "lcd_sptrsv_csr_syncfree": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, c_int,
                                        c_int, _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_gs_layout_workspace_bytes": (c_int, [c_int32, ctypes.POINTER(c_int64)]),
    "lcd_gs_layout": (c_int, [c_int32, c_int64, _P, _P, c_int, _P, _P, _P, ctypes.POINTER(c_int64),
                              _P, c_int64, _P, _P, ctypes.POINTER(c_int)]),
    "lcd_gs_values": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P]),
    "lcd_chain_workspace_bytes": (c_int, [c_int32, ctypes.POINTER(c_int64)]),
    "lcd_chain_growth": (c_int, [c_int32, _P, c_int64, _P, ctypes.POINTER(c_double)]),
    "lcd_chain_cluster_size": (c_int, []),
    "lcd_chain_prepare": (c_int, [c_int32, c_int64, _P, _P, _P, _P, c_int, _P, c_int64, _P]),
    "lcd_sptrsv_csr_chain": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, _P, c_int64,
                                     _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_permute_f64": (c_int, [c_int64, _P, _P, _P, c_int, _P]),
    "lcd_chain_prepare_rows": (c_int, [c_int32, c_int64, _P, _P, _P, _P, c_int, _P, c_int64, c_int32,
                                       c_int32, _P]),
    "lcd_sptrsv_csr_chain_rows": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, _P, c_int64,
                                          c_int32, c_int32, _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_sptrsv_csr_syncfree_multi": (c_int, [c_int32, c_int64, c_int32, _P, _P, _P, _P, _P, _P,
                                              c_int64, c_int, _P, c_int32, _P,
                                              ctypes.POINTER(c_int)]),
    "lcd_transpose_f64": (c_int, [c_int64, c_int64, _P, c_int64, _P, c_int64, _P]),
    "lcd_sptrsv_csc_syncfree": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, c_int,
                                        _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_csc_edge_count": (c_int, [c_int32, _P, _P, c_int, _P, _P]),
    "lcd_sptrsv_wavefront": (c_int, [c_int, c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, _P,
                                     _P, _P, c_int32, c_int, c_int, _P, c_int32, _P,
                                     ctypes.POINTER(c_int)]),
    "lcd_sptrsv_wavefront_tasks": (c_int, [c_int, c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int,
                                           _P, _P, _P, _P, c_int32, c_int, c_int, _P, c_int32, _P,
                                           ctypes.POINTER(c_int)]),
    "lcd_sptrsv_wavefront_multi": (c_int, [c_int32, c_int64, c_int32, _P, _P, _P, _P, _P, _P, c_int64,
                                           c_int, _P, _P, c_int32, _P, c_int32, _P,
                                           ctypes.POINTER(c_int)]),
    "lcd_sptrsv_csr_ordered": (c_int, [c_int32, c_int64, c_int32, _P, _P, _P, _P, _P, _P, c_int64,
                                       c_int, _P, _P, c_int, _P, c_int64, _P, c_int32, _P,
                                       ctypes.POINTER(c_int)]),
    "lcd_small_max_entries": (c_int, []),
    "lcd_small_level_cuts": (c_int, [c_int32, c_int32, c_int32, _P, _P, _P, _P]),
    "lcd_small_plan_measure": (c_int, [c_int, c_int, c_int32, c_int64, _P, _P, _P, _P, _P, _P, _P, _P,
                                       c_int32, c_int32, c_int32, _P, _P, _P, _P, _P,
                                       ctypes.POINTER(c_int32 * 4)]),
    "lcd_small_plan_fill": (c_int, [c_int, c_int, c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int32, c_int32,
                                    _P, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P, _P,
                                    ctypes.POINTER(c_int32)]),
    "lcd_small_scratch_bytes": (c_int, [c_int32, c_int32, ctypes.POINTER(c_int64)]),
    "lcd_sptrsv_small": (c_int, [c_int32, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P, _P, c_int32,
                                 c_int32, c_int32, c_int32, _P, c_int64, _P, c_int32, _P, _P]),
    "lcd_small_scratch_bytes_multi": (c_int, [c_int32, c_int32, c_int32, ctypes.POINTER(c_int64)]),
    "lcd_sptrsv_small_multi": (c_int, [c_int32, c_int32, c_int32, _P, _P, _P, c_int32, c_int64, _P, _P, _P, _P,
                                       _P, c_int32, c_int32, c_int32, c_int32, _P, c_int64, _P, c_int32,
                                       _P, _P]),
    "lcd_spilu0_csr": (c_int, [c_int32, c_int64, _P, _P, _P, _P, c_int, _P, _P, _P, c_int32,
                               c_int, _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_supernodal_layout_workspace_bytes": (c_int, [c_int32, c_int64, _P]),
    "lcd_supernodal_layout": (c_int, [c_int32, c_int64, _P, _P, c_int32, _P, _P, _P, _P, _P, _P, _P,
                                      c_int64, _P]),
    "lcd_supernodal_fill": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, _P, _P, c_int64, _P, _P,
                                    _P]),
    "lcd_spilu0_csr_ordered": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, _P, c_int, c_int, _P,
                                       c_int32, _P, _P]),
    "lcd_spilu0_csr_static": (c_int, [c_int32, c_int64, _P, _P, _P, _P, c_int, c_int32, _P,
                                      ctypes.POINTER(c_int)]),
    "lcd_supernodal_pending": (c_int, [c_int32, _P, _P, _P, _P, _P, _P]),
    "lcd_supernodal_strip_rows": (c_int, []),
    "lcd_sptrsv_supernodal": (c_int, [c_int32, c_int32, c_int32, _P, _P, _P, _P, _P, _P, _P, _P,
                                      _P, _P, _P, _P, _P, _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_supernodal_prepare": (c_int, [c_int32, _P, _P, _P, _P, _P, _P, _P, _P]),
    "lcd_peer_alloc": (c_int, [c_int64, ctypes.POINTER(c_void_p), ctypes.c_char_p]),
    "lcd_peer_open": (c_int, [ctypes.c_char_p, ctypes.POINTER(c_void_p)]),
    "lcd_peer_close": (c_int, [_P]),
    "lcd_peer_free": (c_int, [_P]),
    "lcd_partition_need_mask": (c_int, [c_int32, _P, _P, c_int, _P, c_int32, _P, _P]),
    "lcd_sptrsv_csr_syncfree_part": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, c_int, c_int32,
                                             c_int32, _P, ctypes.POINTER(c_void_p), c_int32, c_int,
                                             _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_sptrsv_csr_ordered_part": (c_int, [c_int32, c_int64, _P, _P, _P, _P, _P, c_int, _P, c_int32,
                                            _P, c_int, _P, ctypes.POINTER(c_void_p), c_int32, c_int64,
                                            _P, c_int32, _P, ctypes.POINTER(c_int)]),
    "lcd_calibrate": (c_int, [_P, c_int64, _P, ctypes.POINTER(c_double * 16)]),
    "lcd_set_tuning": (c_int, [c_int, c_int]),
    "lcd_debug_set_trace": (c_int, [_P]),
    "lcd_checksum_i32": (c_int, [_P, c_int64, _P, ctypes.POINTER(c_uint64 * 2), _P]),
    "lcd_fill_u64": (c_int, [_P, c_int64, c_uint64, _P]),
    "lcd_device_sm_count": (c_int, [ctypes.POINTER(c_int)]),
}
EXPORTED_SYMBOLS = tuple(_SIGNATURES)

_lib = None


def load():
    """Load the shared library (once) and attach the prototypes."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise NativeLibraryMissing(
            f"{LIB_PATH} is missing. Build it with `python -m lcd_b200.build` "
            "(needs nvcc); lcd_b200 has no CPU or interpreter fallback.")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _lib = lib
    return lib


def error_string(code):
    return load().lcd_error_string(int(code)).decode()


def check(code, where):
    """Raise NativeError for a non-zero return code."""
    if code != OK:
        detail = error_string(code)
        if code == ERR_CUDA:
            detail += ": " + load().lcd_last_cuda_error().decode()
        raise NativeError(code, where, detail)


def ptr(tensor):
    """Device address of a torch tensor (or None)."""
    if tensor is None:
        return None
    return c_void_p(tensor.data_ptr())
