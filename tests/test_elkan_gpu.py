"""Per-center bounds between passes on the tensor-core shapes (kmc_pass_elkan, -m gpu).

The reference keeps one lower bound per (row, center) between Lloyd passes at high d and visits only the centers
whose bound fell below the row's own distance (core.py:1690-2015; tests/accuracy.py:173-246 check its labels).
Here the bounded pass must give the full tensor-core pass's results bit for bit: Lloyd steps with the bounds
against steps without, from the same start -- new centers, every totals column (counts, float64-distance inertia,
sums) and the empties identical at every step, under both label rules -- while visiting a small share of the
(row, center) pairs once the centers settle. Rows at exact float64 ties and centers that jump (every bound fails)
get the oracle's labels.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _embeddings(n, d, k_true, seed):
    rng = np.random.default_rng(seed)
    dirs = rng.standard_normal((k_true, d))
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    X = dirs[rng.integers(0, k_true, n)] + 0.15 * rng.standard_normal((n, d))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


@pytest.mark.parametrize("n,d,k,rule", [(20_000, 768, 256, "float64"), (50_000, 32, 64, "float64"),
                                        (30_000, 100, 96, "float32"), (20_000, 128, 512, "float64")])
def test_bounded_steps_equal_full_steps(n, d, k, rule, cuda_device):
    import mlx_kmeans_b200 as km
    X = _embeddings(n, d, max(k // 2, 2), n + d)
    C0 = torch.from_numpy(X[np.random.default_rng(k).choice(n, k, replace=False)].copy()).to(cuda_device)
    Xt = torch.from_numpy(X).to(cuda_device)
    a, b = km.Dataset([Xt]), km.Dataset([Xt])
    a.elkan = True
    assert a.elkan_ok(k) and not b.elkan_ok(k)
    Ca, Cb = C0.clone(), C0.clone()
    visited = []
    for step in range(8):
        if step == 4:
            # a labels pass in between (the dense pass: for small totals it reduces the rows in order and leaves
            # them ungrouped), after which the bounded pass visits the rows in row order
            a.assign(Ca, return_labels=True, rule=rule)
        Na, sa = a.step(Ca, rule=rule)
        ta = a.buffers(k)["totals"].clone()
        Nb, sb = b.step(Cb, rule=rule)
        tb = b.buffers(k)["totals"].clone()
        assert torch.equal(ta, tb), f"step {step}: totals differ"
        assert torch.equal(Na, Nb), f"step {step}: centers differ"
        assert sa["n_empty"] == sb["n_empty"] and sa["inertia"] == sb["inertia"]
        visited.append(sa["screened"] / (n * k))
        Ca, Cb = Na.clone(), Nb.clone()
    assert visited[0] == 0.0                      # the first pass builds the bounds
    assert min(visited[3:]) < 0.25, visited      # later passes visit a small share of the pairs


def _elkan_labels(X, C_build, C, device, rule=0):
    """Labels of a bounded pass with centers C on bounds built with C_build, through the C ABI."""
    from mlx_kmeans_b200 import _lib
    import mlx_kmeans_b200 as km
    L = _lib.load()
    n, d = X.shape
    k = C.shape[0]
    ds = km.Dataset([torch.from_numpy(X).to(device)])
    p = ds.parts[0]
    (sp, sb), (cs, cb) = ds.split()[0], ds.csplit(k)
    eb = int(L.kmc_elkan_bytes(n, d, k))
    e = torch.empty(eb, dtype=torch.uint8, device=device)
    buf = ds.buffers(k)
    lab = torch.empty(n, dtype=torch.int32, device=device)
    st = torch.cuda.current_stream().cuda_stream
    flags = _lib.KMC_PASS_LABEL32 if rule else 0
    for Cx, f in ((C_build, flags | _lib.KMC_PASS_ELKAN_BUILD), (C, flags)):
        Ct = torch.from_numpy(np.ascontiguousarray(Cx)).to(device)
        _lib.call("kmc_pass_elkan", p.data_ptr(), n, d, Ct.data_ptr(), k, ds.colmax.data_ptr(), n,
                  buf["totals"].data_ptr(), lab.data_ptr(), None, f, sp.data_ptr(), sb, cs.data_ptr(), cb,
                  e.data_ptr(), eb, buf["ws"].data_ptr(), buf["wsb"], st)
    torch.cuda.synchronize()
    return lab.cpu().numpy().astype(np.int64)


def test_exact_ties_and_jumps(cuda_device):
    rng = np.random.default_rng(23)
    d, pairs = 128, 64
    M = (np.rint(rng.standard_normal((pairs, d)) * 1024) / 1024).clip(-7.9, 7.9).astype(np.float32)
    U = np.where(rng.random((pairs, d)) < 0.5, -1.0, 1.0).astype(np.float32) * np.float32(2.0 ** -6)
    C = np.concatenate([M + U, M - U, rng.standard_normal((128, d)).astype(np.float32) * 4]).astype(np.float32)
    X = np.concatenate([M, M + np.float32(1e-3) * rng.standard_normal(M.shape).astype(np.float32),
                        rng.standard_normal((3000, d)).astype(np.float32)]).astype(np.float32)
    ref, _, _ = O.assign(X, C)
    assert np.array_equal(ref[:pairs], np.arange(pairs))            # exact ties go to the lower index
    # bounds built on the same centers (zero drift) and on centers far off (every bound useless)
    assert np.array_equal(_elkan_labels(X, C, C, cuda_device), ref)
    far = (C * np.float32(0.25) + np.float32(3.0)).astype(np.float32)
    assert np.array_equal(_elkan_labels(X, far, C, cuda_device), ref)
    ref32, _, _ = O.assign(X, C, rule="float32")
    assert np.array_equal(_elkan_labels(X, far, C, cuda_device, rule=1), ref32)


def test_bounds_dropped_when_they_do_not_pay(cuda_device):
    """Isotropic data (uniform noise, no structure): the bounds visit most pairs, the policy drops them and
    waits before building again; the results stay those of the full pass."""
    import mlx_kmeans_b200 as km
    rng = np.random.default_rng(3)
    X = rng.standard_normal((20_000, 256)).astype(np.float32)
    C = torch.from_numpy(X[:64].copy()).to(cuda_device)
    a, b = km.Dataset([X]), km.Dataset([X])
    a.elkan = True
    for _ in range(4):
        Na, _ = a.step(C)
        Nb, _ = b.step(C)
        assert torch.equal(Na, Nb)
        C = Na.clone() + 0.05 * torch.randn_like(Na)                 # centers keep moving a lot
    e = a._elkan[64]
    assert e["cool"] >= 1 or not e["valid"]
