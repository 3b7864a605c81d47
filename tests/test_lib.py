"""libkmc.so: it builds for sm_100a, loads, and exports every entry point include/kmc.h declares (CPU tier:
no compute call is made without a GPU)."""
import os
import re
import subprocess

import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "kmc.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(kmc_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_boundary():
    names = declared()
    for n in ["kmc_pass", "kmc_finish", "kmc_far_rows", "kmc_colmax", "kmc_pp_init", "kmc_gen", "kmc_stats_read",
              "kmc_totals_unpack", "kmc_workspace_bytes"]:
        assert n in names


def test_library_builds_and_exports_every_declared_symbol():
    from mlx_kmeans_b200 import build
    lib = build.build()
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    exported = set(re.findall(r" T (kmc_\w+)", out))
    missing = [n for n in declared() if n not in exported]
    assert not missing, f"declared in kmc.h but not exported: {missing}"


def test_ctypes_binding_covers_the_header():
    from mlx_kmeans_b200 import _lib
    assert sorted(_lib.SIGNATURES) == declared()
    L = _lib.load()
    assert L.kmc_version() >= 1
    # size queries need no device
    assert L.kmc_workspace_bytes(4, 16) > 0
    assert L.kmc_far_workspace_bytes(8) > 0
    assert L.kmc_pp_workspace_bytes(1000, 4, 16) > 0


def test_invalid_arguments_are_reported_not_thrown():
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    # null pointers / bad shapes fail in the argument checks, before any CUDA call
    assert L.kmc_pass(None, 10, 0, None, 4, None, 10, None, None, None, 0, None, 0, None) == _lib.KMC_ERR_INVALID
    assert b"dims" in L.kmc_last_error()
    assert L.kmc_pass(None, 10, 5000, None, 4, None, 10, None, None, None, 0, None, 0, None) == _lib.KMC_ERR_UNSUPPORTED
    assert L.kmc_finish(None, 4, 4, None, 0, 1, None, None, None, 0, None) == _lib.KMC_ERR_INVALID
    with pytest.raises(ValueError):
        _lib.call("kmc_pass", None, 10, 0, None, 4, None, 10, None, None, None, 0, None, 0, None)


def test_exchange_buffers_shared_per_group(monkeypatch):
    """Datasets of one process group share one set of peer-memory exchange buffers per (k, d) and never free
    them mid-run (a peer may still read a buffer when a Dataset goes away): a second Dataset reuses the first
    one's buffers and step count instead of opening new ones.  Host logic only (the opening is stubbed)."""
    from mlx_kmeans_b200 import core
    opened = []

    def fake_open(self, k):
        opened.append((k, self.d))
        return dict(dev=None, step=0)

    monkeypatch.setattr(core.Dataset, "_open_exchange", fake_open)
    monkeypatch.setattr(core, "_exchanges", {})
    group = object()

    def ds(d):
        x = object.__new__(core.Dataset)
        x.group, x.d, x._xch = group, d, {}
        return x

    a, b, c = ds(4), ds(4), ds(8)
    xa = a._exchange(16)
    xa["step"] += 3
    assert b._exchange(16) is xa and b._exchange(16)["step"] == 3
    assert c._exchange(16) is not xa
    assert opened == [(16, 4), (16, 8)]


def test_cascade_shape_rule_and_prefix_width():
    """The cascade's prefix width (core.py:1198-1200: half the dims in multiples of 8, from 8 up to 96) and where it
    applies (core.py:486-491, 1203-1204: 128 to 256 dims, k >= 256; here also k % 8 == 0 for the survivor words),
    checked on the Dataset's own methods without a GPU."""
    import types
    from mlx_kmeans_b200.core import Dataset

    def ds(d, n=1000):
        o = types.SimpleNamespace(d=d, tensor_cores=True, n_local=n, cascade=True, _cascade={})
        for name in ("CASCADE_MIN_DIMS", "CASCADE_MAX_DIMS", "CASCADE_MIN_K", "CASCADE_MAX_BYTES"):
            setattr(o, name, getattr(Dataset, name))
        return o

    assert [Dataset.cascade_m(ds(d)) for d in (8, 17, 64, 128, 192, 256, 960)] == [8, 8, 32, 64, 96, 96, 96]
    assert Dataset.cascade_ok(ds(128), 256) and Dataset.cascade_ok(ds(256), 4096, forced=True)
    assert not Dataset.cascade_ok(ds(127), 256, forced=True) and not Dataset.cascade_ok(ds(257), 256, forced=True)
    assert not Dataset.cascade_ok(ds(128), 248, forced=True) and not Dataset.cascade_ok(ds(128), 260, forced=True)
    off = ds(128)
    off.cascade = False
    assert not Dataset.cascade_ok(off, 256) and Dataset.cascade_ok(off, 256, forced=True)
    dropped = ds(128)
    dropped._cascade = {256: {"ok": False}}
    assert not Dataset.cascade_ok(dropped, 256) and Dataset.cascade_ok(dropped, 256, forced=True)


def test_cascade_arguments_checked_before_any_launch():
    """kmc_pass_cascade refuses what it cannot run -- a missing pointer, a prefix wider than the row, k not a
    multiple of 8, the approximate or bounds-building flags, a state buffer too small -- with a status and a
    message, before any CUDA call (the pointers below are never dereferenced)."""
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    p = 256                               # a nonzero stand-in; every call below fails in its argument checks

    def call(n=10, d=128, k=256, flags=0, Cm=p, m=64, cascade=p, cbytes=1 << 40, msb=1 << 40, mcb=1 << 40):
        return L.kmc_pass_cascade(p, n, d, p, k, p, n, p, None, None, flags, p, 1 << 40, p, 1 << 40, Cm, m, p, msb,
                                  p, mcb, cascade, cbytes, p, 1 << 40, None)

    assert call(Cm=None) == _lib.KMC_ERR_INVALID and b"null" in L.kmc_last_error()
    assert call(cascade=None) == _lib.KMC_ERR_INVALID
    assert call(m=0) == _lib.KMC_ERR_INVALID and call(m=129) == _lib.KMC_ERR_INVALID
    assert call(k=260) == _lib.KMC_ERR_UNSUPPORTED
    assert call(flags=_lib.KMC_PASS_APPROX) == _lib.KMC_ERR_INVALID
    assert call(flags=_lib.KMC_PASS_ELKAN_BUILD) == _lib.KMC_ERR_INVALID
    assert call(cbytes=16) == _lib.KMC_ERR_INVALID and b"cascade state" in L.kmc_last_error()
    assert call(msb=16) == _lib.KMC_ERR_INVALID and b"prefix split" in L.kmc_last_error()
    assert call(mcb=16) == _lib.KMC_ERR_INVALID
    assert L.kmc_cascade_bytes(1000, 4096) >= 1000 * 4096 // 8
