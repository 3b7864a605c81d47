"""ctypes binding of libkmc.so (include/kmc.h).

The library is loaded from this package's directory (built in-tree by mlx_kmeans_b200/build.py). There is
no fallback: if the library is missing or cannot be loaded the import of the compute path raises, and every
non-zero status from a call is raised as the Python exception the reference raises for the same condition
(ValueError for bad input, RuntimeError for a device failure, core.py:581-593 and 2022-2035).
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libkmc.so")

KMC_OK, KMC_ERR_INVALID, KMC_ERR_CUDA, KMC_ERR_UNSUPPORTED = 0, 1, 2, 3
KMC_PASS_ACCUMULATE = 1
KMC_PASS_GENERIC = 2
KMC_PASS_LABEL32 = 4
KMC_PASS_APPROX = 8
KMC_PASS_ELKAN_BUILD = 16
KMC_MAX_DIMS = 4096
STATS_BYTES = 64

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
_u = ctypes.c_uint
_u64 = ctypes.c_uint64
_sz = ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/kmc.h
SIGNATURES = {
    "kmc_version": (_int, []),
    "kmc_last_error": (ctypes.c_char_p, []),
    "kmc_num_sms": (_int, []),
    "kmc_row_block": (_i64, [_i64]),
    "kmc_workspace_bytes": (_sz, [_int, _int]),
    "kmc_far_workspace_bytes": (_sz, [_i64]),
    "kmc_colmax": (_int, [_vp, _i64, _int, _vp, _u, _vp]),
    "kmc_pass": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _vp, _vp, _u, _vp, _sz, _vp]),
    "kmc_pass_static": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _vp, _vp, _u, _vp]),
    "kmc_bounds_bytes": (_sz, [_i64, _int, _int]),
    "kmc_bounds_reset": (_int, [_vp, _vp]),
    "kmc_pass_bounded": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _u, _vp, _sz, _vp, _sz, _vp]),
    "kmc_exchange_bytes": (_sz, [_int, _int]),
    "kmc_exchange_alloc": (_int, [_sz, _vp, _vp]),
    "kmc_exchange_open": (_int, [_vp, _vp]),
    "kmc_exchange_close": (_int, [_vp, _int]),
    "kmc_exchange_sum": (_int, [_vp, _int, _int, _vp, _int, _int, _u64, _vp, _sz, _vp]),
    "kmc_exchange_finish": (_int, [_vp, _int, _int, _vp, _int, _int, _u64, _vp, _vp, _vp, _sz, _vp]),
    "kmc_split_bytes": (_sz, [_i64, _int]),
    "kmc_split_rows": (_int, [_vp, _i64, _int, _vp, _sz, _vp]),
    "kmc_csplit_bytes": (_sz, [_int, _int]),
    "kmc_pass_split": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _vp, _vp, _u, _vp, _sz, _vp, _sz, _vp, _sz,
                              _vp]),
    "kmc_elkan_bytes": (_sz, [_i64, _int, _int]),
    "kmc_pass_elkan": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _vp, _vp, _u, _vp, _sz, _vp, _sz, _vp, _sz,
                              _vp, _sz, _vp]),
    "kmc_cascade_bytes": (_sz, [_i64, _int]),
    "kmc_pass_cascade": (_int, [_vp, _i64, _int, _vp, _int, _vp, _i64, _vp, _vp, _vp, _u, _vp, _sz, _vp, _sz, _vp,
                                _int, _vp, _sz, _vp, _sz, _vp, _sz, _vp, _sz, _vp]),
    "kmc_tc_dot": (_int, [_vp, _i64, _int, _int, _vp, _sz, _vp, _sz, _vp, _vp, _vp]),
    "kmc_loop_init": (_int, [_vp, ctypes.c_double, _i64, _i64, ctypes.c_double, _int, _vp]),
    "kmc_lloyd": (_int, [_vp, _i64, _int, _vp, _vp, _int, _vp, _i64, _vp, _u, _vp, _sz, _vp, _vp, _int, _vp, _sz,
                         _vp]),
    "kmc_far_rows": (_int, [_vp, _i64, _int, _vp, _vp, _i64, _i64, _vp, _vp, _sz, _vp]),
    "kmc_finish": (_int, [_vp, _int, _int, _vp, _i64, _int, _vp, _vp, _vp, _sz, _vp]),
    "kmc_stats_read": (_int, [_vp, _vp, _vp]),
    "kmc_totals_unpack": (_int, [_vp, _int, _int, _vp, _vp, _vp, _vp, _sz, _vp]),
    "kmc_d64": (_int, [_vp, _vp, _int, _i64, _vp, _vp]),
    "kmc_pp_workspace_bytes": (_sz, [_i64, _int, _int]),
    "kmc_pp_init": (_int, [_vp, _i64, _int, _int, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "kmc_gen": (_int, [_int, _vp, _i64, _int, _i64, ctypes.c_uint64, _vp, _vp, _int, ctypes.c_float,
                       ctypes.c_float, _vp]),
    "kmc_colsums": (_int, [_vp, _i64, _int, _vp, _i64, _vp, _vp]),
    "kmc_standardize": (_int, [_vp, _i64, _int, _vp, _vp, _i64, _vp, _vp]),
}

_lib = None


def load():
    """Load libkmc.so and bind every entry point of include/kmc.h. Raises if it is absent."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m mlx_kmeans_b200.build` "
                           f"(the CUDA path has no CPU fallback)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class KmcError(RuntimeError):
    pass


def check(status, what=""):
    """Raise the reference's exception type for a non-zero status."""
    if status == KMC_OK:
        return
    msg = load().kmc_last_error().decode(errors="replace")
    text = f"{what}: {msg}" if what else msg
    if status in (KMC_ERR_INVALID, KMC_ERR_UNSUPPORTED):
        raise ValueError(text)
    raise RuntimeError(text)


def call(name, *args):
    """Call kmc_<name>(*args) and raise on a non-zero status."""
    check(getattr(load(), name)(*args), name)
