"""kmc_pass_static: the assignment pass for callers that cannot allocate device memory.

Such callers -- a host runtime that owns every device allocation through its own pool, or code running where
calling an allocator is not allowed -- cannot hand kmc_pass the workspace it asks for. kmc_pass_static keeps that
scratch in a fixed device array inside the library instead, and kmc_finish / kmc_totals_unpack given no
workspace read the fixed-point grid of the totals from the same array. This file checks, through the C ABI, that
two steps in a row give the same totals, new centers, statistics and unpacked sums as kmc_pass + kmc_finish with a
caller workspace (the parity tests' bar for one kernel against itself: identical), on a shape of the fused
low-dimensional kernel and one of the any-shape kernel, and that a shape needing more scratch than the array
holds is refused. It is collected last so that a failure here stops a -x run only after every other test has run;
it also passes alone in a fresh process.
"""
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


def _step(L, lib, Xd, Cd, cm, n, d, k, ws, wsb, static, device):
    """One Lloyd step through the C ABI -> (totals, C_new, stats, sums, counts, inertia) on the host."""
    import torch
    st = torch.cuda.current_stream().cuda_stream
    tot = torch.full((k, d + 2), -1, dtype=torch.int64, device=device)
    C_new = torch.full((k, d), float("nan"), dtype=torch.float32, device=device)
    stats = torch.zeros(lib.STATS_BYTES, dtype=torch.uint8, device=device)
    sums = torch.empty((k, d), dtype=torch.float64, device=device)
    counts = torch.empty(k, dtype=torch.int64, device=device)
    inertia = torch.empty(1, dtype=torch.float64, device=device)
    if static:
        lib.check(L.kmc_pass_static(Xd.data_ptr(), n, d, Cd.data_ptr(), k, cm.data_ptr(), n, tot.data_ptr(), None,
                                    None, 0, st), "kmc_pass_static")
        w, wb = None, 0
    else:
        lib.check(L.kmc_pass(Xd.data_ptr(), n, d, Cd.data_ptr(), k, cm.data_ptr(), n, tot.data_ptr(), None, None, 0,
                             ws.data_ptr(), wsb, st), "kmc_pass")
        w, wb = ws.data_ptr(), wsb
    lib.check(L.kmc_totals_unpack(tot.data_ptr(), k, d, sums.data_ptr(), counts.data_ptr(), inertia.data_ptr(), w, wb,
                                  st), "kmc_totals_unpack")
    lib.check(L.kmc_finish(tot.data_ptr(), k, d, None, 0, 1, C_new.data_ptr(), stats.data_ptr(), w, wb, st),
              "kmc_finish")
    torch.cuda.synchronize()
    return (tot.cpu().numpy(), C_new.cpu().numpy(), stats.cpu().numpy(), sums.cpu().numpy(), counts.cpu().numpy(),
            inertia.cpu().numpy())


@pytest.mark.parametrize("n,d,k", [(300_000, 4, 16), (20_000, 33, 40)])
def test_static_scratch_step_matches_workspace_step(n, d, k, cuda_device):
    import torch
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    Xd, Cd = _setup(n, d, k, 5, cuda_device)
    st = torch.cuda.current_stream().cuda_stream
    cm = torch.zeros(d, dtype=torch.int32, device=cuda_device)
    _lib.check(L.kmc_colmax(Xd.data_ptr(), n, d, cm.data_ptr(), 0, st), "kmc_colmax")
    # the existing entry points, with a caller workspace
    wsb = int(L.kmc_workspace_bytes(d, k))
    ws = torch.empty(wsb, dtype=torch.uint8, device=cuda_device)
    want = _step(L, _lib, Xd, Cd, cm, n, d, k, ws, wsb, False, cuda_device)
    assert want[0][:, 0].sum() == n
    assert np.isfinite(want[1]).all()
    # the static-scratch entry point, two steps in a row (the array keeps the previous call's contents)
    for _ in range(2):
        got = _step(L, _lib, Xd, Cd, cm, n, d, k, None, 0, True, cuda_device)
        for a, b in zip(got, want):
            assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_static_scratch_refuses_shapes_beyond_its_size(cuda_device):
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    k, d = 60_000, 64
    assert L.kmc_workspace_bytes(d, k) > 64 * 1024
    # rejected in the argument checks, before any pointer is used
    rc = L.kmc_pass_static(None, 10, d, None, k, None, 10, None, None, None, 0, None)
    assert rc == _lib.KMC_ERR_UNSUPPORTED
    assert b"scratch" in L.kmc_last_error()
