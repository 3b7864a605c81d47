"""NumPy-facing wrapper around the C oracle (kmc_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg,
as the checker. The product (mlx_kmeans_b200) never imports this module.

Each function states the reference code it restates (kakollu/mlx-kmeans, path:line).
"""
import ctypes
import os
import subprocess

import numpy as np

_DIR = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_DIR, "libkmc_oracle.so")
_lib = None

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i64p = np.ctypeslib.ndpointer(np.int64, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(np.uint64, flags="C_CONTIGUOUS")


def build():
    """Compile kmc_oracle.c with its Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _DIR], check=True)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(os.path.join(_DIR, "kmc_oracle.c")):
            build()
        L = ctypes.CDLL(_SO)
        L.kmo_d64.restype = ctypes.c_double
        L.kmo_d64.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.kmo_best32.restype = ctypes.c_float
        L.kmo_best32.argtypes = [_f32p, _f32p, ctypes.c_int]
        L.kmo_assign.restype = None
        L.kmo_assign.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int, _i64p, _f64p, _f32p,
                                 ctypes.c_int]
        L.kmo_assign_rule.restype = None
        L.kmo_assign_rule.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int, _i64p, _f64p,
                                      _f32p, ctypes.c_int, ctypes.c_int]
        L.kmo_finish.restype = ctypes.c_int
        L.kmo_finish.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, _f32p, ctypes.c_int, _i64p, _f32p, _f32p,
                                 ctypes.POINTER(ctypes.c_double), _i64p]
        L.kmo_log.restype = ctypes.c_double
        L.kmo_log.argtypes = [ctypes.c_double]
        L.kmo_philox.restype = None
        L.kmo_philox.argtypes = [np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")] * 3
        L.kmo_pp_init.restype = None
        L.kmo_pp_init.argtypes = [_f32p, ctypes.c_int64, ctypes.c_int, ctypes.c_int, ctypes.c_int64, _u64p, _i64p,
                                  _f32p]
        _lib = L
    return _lib


def _threads():
    return max(1, min(64, os.cpu_count() or 1))


RULES = {"float64": 0, "float32": 1}


def assign(X, C, threads=None, rule="float64"):
    """Exact labels and each row's float64 distance and float32 `best` distance (core.py:248-257, square and add
    rounded separately) to its label.  rule "float64": argmin of the float64 distance, lowest index on ties
    (tests/accuracy.py:31-51); rule "float32": the reference's rows kernel (core.py:263-274), argmin of the float32
    direct sum with strict < in index order.  -> (labels int64, d64 float64, best32 float32)."""
    X = np.ascontiguousarray(X, np.float32)
    C = np.ascontiguousarray(C, np.float32)
    n, d = X.shape
    k = C.shape[0]
    labels = np.empty(n, np.int64)
    d64 = np.empty(n, np.float64)
    best = np.empty(n, np.float32)
    lib().kmo_assign_rule(X, n, d, C, k, labels, d64, best, threads or _threads(), RULES[rule])
    return labels, d64, best


def lloyd_step(X, C, labels=None, best=None, rule="float64"):
    """core.py:2209-2242 on the oracle's exact labels (of the given label rule).
    -> (C_new float32, inertia float, n_empty int, relocations [(cluster, row)], labels, best32)."""
    X = np.ascontiguousarray(X, np.float32)
    C = np.ascontiguousarray(C, np.float32)
    if labels is None or best is None:
        labels, _, best = assign(X, C, rule=rule)
    labels = np.ascontiguousarray(labels, np.int64)
    best = np.ascontiguousarray(best, np.float32)
    n, d = X.shape
    k = C.shape[0]
    C_new = np.empty_like(C)
    inertia = ctypes.c_double()
    reloc = np.full(2 * k, -1, np.int64)
    n_empty = lib().kmo_finish(X, n, d, C, k, labels, best, C_new, ctypes.byref(inertia), reloc)
    pairs = [(int(reloc[2 * i]), int(reloc[2 * i + 1])) for i in range(k) if reloc[2 * i] >= 0]
    return C_new, inertia.value, int(n_empty), pairs, labels, best


def accumulate(X, labels, k):
    """Float64 per-cluster sums and counts of X over given labels (core.py:2223, np.add.at order)."""
    X64 = np.asarray(X, np.float64)
    sums = np.zeros((k, X.shape[1]))
    np.add.at(sums, labels, X64)
    return sums, np.bincount(labels, minlength=k).astype(np.int64)


def d64(x, c):
    x = np.ascontiguousarray(x, np.float32)
    c = np.ascontiguousarray(c, np.float32)
    return lib().kmo_d64(x, c, x.shape[0])


def pp_init(S, k, first, seeds):
    """Greedy k-means++ on the sample S (core.py:153-192) with Philox keys seeds[r] per round.
    -> (picks int64 k, C float32 k x d)."""
    S = np.ascontiguousarray(S, np.float32)
    m, d = S.shape
    seeds = np.ascontiguousarray(seeds, np.uint64)
    picks = np.empty(k, np.int64)
    C = np.empty((k, d), np.float32)
    lib().kmo_pp_init(S, m, d, k, int(first), seeds, picks, C)
    return picks, C


def philox(ctr, key):
    ctr = np.ascontiguousarray(ctr, np.uint32)
    key = np.ascontiguousarray(key, np.uint32)
    out = np.empty(4, np.uint32)
    lib().kmo_philox(ctr, key, out)
    return out


def log(v):
    return lib().kmo_log(float(v))
