"""kmc_pass_static: the assignment pass for callers that cannot allocate device memory.

Such callers -- a host runtime that owns every device allocation through its own pool, or code running where
calling an allocator is not allowed -- cannot hand kmc_pass the workspace it asks for. kmc_pass_static keeps that
scratch in a fixed device array inside the library instead. This file checks, through the C ABI, that two calls
in a row give the same totals as kmc_pass with a caller workspace (the parity tests' bar for totals of one
kernel: identical), on a shape of the fused low-dimensional kernel and one of the any-shape kernel, and that a
shape needing more scratch than the array holds is refused. It is collected last so that a failure here stops
a -x run only after every other test has run; it also passes alone in a fresh process.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(n, d, k, seed, device):
    import torch
    rng = np.random.default_rng(seed)
    X = (rng.uniform(-5, 5, (k, d))[rng.integers(0, k, n)] + rng.standard_normal((n, d))).astype(np.float32)
    C = X[rng.choice(n, k, replace=False)].copy()
    Xd = torch.from_numpy(X).to(device)
    Cd = torch.from_numpy(C).to(device)
    return Xd, Cd


@pytest.mark.parametrize("n,d,k", [(300_000, 4, 16), (20_000, 33, 40)])
def test_static_scratch_pass_matches_workspace_pass(n, d, k, cuda_device):
    import torch
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    Xd, Cd = _setup(n, d, k, 5, cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    cm = torch.zeros(d, dtype=torch.int32, device=cuda_device)
    _lib.check(L.kmc_colmax(Xd.data_ptr(), n, d, cm.data_ptr(), 0, st), "kmc_colmax")
    # the existing entry point, with a caller workspace
    wsb = int(L.kmc_workspace_bytes(d, k))
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda_device)
    ref = torch.empty((k, d + 2), dtype=torch.int64, device=cuda_device)
    _lib.check(L.kmc_pass(Xd.data_ptr(), n, d, Cd.data_ptr(), k, cm.data_ptr(), n, ref.data_ptr(), None, None, 0,
                          ws.data_ptr(), wsb, st), "kmc_pass")
    torch.cuda.synchronize()
    want = ref.cpu().numpy()
    assert want[:, 0].sum() == n
    # the static-scratch entry point, twice in a row (the array keeps the previous call's contents)
    for _ in range(2):
        out = torch.full((k, d + 2), -1, dtype=torch.int64, device=cuda_device)
        _lib.check(L.kmc_pass_static(Xd.data_ptr(), n, d, Cd.data_ptr(), k, cm.data_ptr(), n, out.data_ptr(), None,
                                     None, 0, st), "kmc_pass_static")
        torch.cuda.synchronize()
        assert np.array_equal(out.cpu().numpy(), want)


def test_static_scratch_refuses_shapes_beyond_its_size(cuda_device):
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    k, d = 60_000, 64
    assert L.kmc_workspace_bytes(d, k) > 64 * 1024
    # rejected in the argument checks, before any pointer is used
    rc = L.kmc_pass_static(ctypes.c_void_p(16), 10, d, ctypes.c_void_p(16), k, ctypes.c_void_p(16), 10,
                           ctypes.c_void_p(16), None, None, 0, None)
    assert rc == _lib.KMC_ERR_UNSUPPORTED
    assert b"scratch" in L.kmc_last_error()
