"""The prefix-pruning cascade (kmc_pass_cascade, -m gpu).

The reference scores a row's distance over the highest-variance half of the columns first and finishes only the
centers whose prefix distance does not exceed the row's distance to its previous label (core.py:1091-1260, forced
by method="cascade" in tests/accuracy.py:81-83 and on anisotropic data at 128 dims, tests/accuracy.py:275-280).
Nothing approximate may reach the answer: a cascade pass must give the dense tensor-core pass's labels, counts,
sums and inertia bit for bit, under both label rules, whatever its starting labels are -- and prune most pairs on
data with variance structure.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _anisotropic(n, d, k_true, seed):
    """Blobs whose column spread falls off geometrically (SIFT-like variance structure), columns shuffled so
    that the high-variance ones are not the leading ones."""
    rng = np.random.default_rng(seed)
    scale = 4.0 * 0.97 ** np.arange(d)
    means = rng.standard_normal((k_true, d)) * scale
    X = means[rng.integers(0, k_true, n)] + rng.standard_normal((n, d)) * (0.25 * scale + 0.02)
    return X[:, rng.permutation(d)].astype(np.float32)


@pytest.mark.parametrize("n,d,k,rule,slices", [(30_000, 128, 256, "float64", 1), (24_000, 192, 256, "float32", 1),
                                               (30_000, 128, 512, "float64", 3)])
def test_cascade_steps_equal_dense_steps(n, d, k, rule, slices, cuda_device):
    import mlx_kmeans_b200 as km
    X = _anisotropic(n, d, 64, n + d + k)
    C0 = torch.from_numpy(X[np.random.default_rng(k).choice(n, k, replace=False)].copy()).to(cuda_device)
    Xt = torch.from_numpy(X).to(cuda_device)
    parts = list(torch.tensor_split(Xt, slices)) if slices > 1 else [Xt]
    a, b = km.Dataset(parts), km.Dataset(parts)
    assert a.cascade_ok(k, forced=True) and not b.cascade_ok(k)
    Ca, Cb = C0.clone(), C0.clone()
    survived = []
    for step in range(6):
        Na, sa = a.step(Ca, rule=rule, cascade=True)
        ta = a.buffers(k)["totals"].clone()
        Nb, sb = b.step(Cb, rule=rule)
        tb = b.buffers(k)["totals"].clone()
        assert torch.equal(ta, tb), f"step {step}: totals differ"
        assert torch.equal(Na, Nb), f"step {step}: centers differ"
        assert sa["n_empty"] == sb["n_empty"] and sa["inertia"] == sb["inertia"]
        survived.append(sa["screened"] / (n * k))
        Ca, Cb = Na.clone(), Nb.clone()
    assert a._cascade[k]["m"] == a.cascade_m() == min(96, d // 2)
    assert max(survived[2:]) < 0.15, survived        # the prefix prunes most pairs on this data
    # labels of a final cascade pass against the float64 oracle (or the float32 rule's)
    _, _, _, lab = a.assign(Ca, return_labels=True, rule=rule, cascade=True)
    ref, _, _ = O.assign(X, Ca.cpu().numpy(), rule=rule)
    assert np.array_equal(lab, ref)


def _cascade_labels(X, C_prev, C, device, rule=0):
    """Labels of a cascade pass with centers C after a plain pass with C_prev (its labels are the starting
    guesses), through the C ABI."""
    from mlx_kmeans_b200 import _lib
    import mlx_kmeans_b200 as km
    L = _lib.load()
    n, d = X.shape
    k = C.shape[0]
    ds = km.Dataset([torch.from_numpy(X).to(device)])
    p = ds.parts[0]
    (sp, sb), (cs, cb) = ds.split()[0], ds.csplit(k)
    m = ds.cascade_m()
    cols = torch.arange(m, device=device)                    # any prefix is correct; only the work depends on it
    xm = p[:, :m].contiguous()
    mb = int(L.kmc_split_bytes(n, m))
    ms = torch.empty(mb, dtype=torch.uint8, device=device)
    mcb = int(L.kmc_csplit_bytes(m, k))
    mcs = torch.empty(mcb, dtype=torch.uint8, device=device)
    eb = int(L.kmc_cascade_bytes(n, k))
    e = torch.empty(eb, dtype=torch.uint8, device=device)
    buf = ds.buffers(k)
    lab = torch.empty(n, dtype=torch.int32, device=device)
    st = torch.cuda.current_stream().cuda_stream
    flags = _lib.KMC_PASS_LABEL32 if rule else 0
    _lib.call("kmc_split_rows", xm.data_ptr(), n, m, ms.data_ptr(), mb, st)
    Cp = torch.from_numpy(np.ascontiguousarray(C_prev)).to(device)
    _lib.call("kmc_pass_split", p.data_ptr(), n, d, Cp.data_ptr(), k, ds.colmax.data_ptr(), n,
              buf["totals"].data_ptr(), None, None, flags, sp.data_ptr(), sb, cs.data_ptr(), cb,
              buf["ws"].data_ptr(), buf["wsb"], st)
    Ct = torch.from_numpy(np.ascontiguousarray(C)).to(device)
    Cm = Ct.index_select(1, cols).contiguous()
    _lib.call("kmc_pass_cascade", p.data_ptr(), n, d, Ct.data_ptr(), k, ds.colmax.data_ptr(), n,
              buf["totals"].data_ptr(), lab.data_ptr(), None, flags, sp.data_ptr(), sb, cs.data_ptr(), cb,
              Cm.data_ptr(), m, ms.data_ptr(), mb, mcs.data_ptr(), mcb, e.data_ptr(), eb, buf["ws"].data_ptr(),
              buf["wsb"], st)
    torch.cuda.synchronize()
    return lab.cpu().numpy().astype(np.int64)


def test_cascade_exact_ties_and_stale_labels(cuda_device):
    """Rows at exact float64 ties between two centers (the lower index wins), and starting labels from centers
    far off (the previous label is a poor bound, so most centers survive): the oracle's labels either way."""
    rng = np.random.default_rng(29)
    d, pairs = 128, 64
    M = (np.rint(rng.standard_normal((pairs, d)) * 1024) / 1024).clip(-7.9, 7.9).astype(np.float32)
    U = np.where(rng.random((pairs, d)) < 0.5, -1.0, 1.0).astype(np.float32) * np.float32(2.0 ** -6)
    C = np.concatenate([M + U, M - U, rng.standard_normal((128, d)).astype(np.float32) * 4]).astype(np.float32)
    X = np.concatenate([M, M + np.float32(1e-3) * rng.standard_normal(M.shape).astype(np.float32),
                        rng.standard_normal((3000, d)).astype(np.float32)]).astype(np.float32)
    ref, _, _ = O.assign(X, C)
    assert np.array_equal(ref[:pairs], np.arange(pairs))            # exact ties go to the lower index
    assert np.array_equal(_cascade_labels(X, C, C, cuda_device), ref)
    far = (C * np.float32(0.25) + np.float32(3.0)).astype(np.float32)
    assert np.array_equal(_cascade_labels(X, far, C, cuda_device), ref)
    ref32, _, _ = O.assign(X, C, rule="float32")
    assert np.array_equal(_cascade_labels(X, far, C, cuda_device, rule=1), ref32)


def test_cascade_dropped_without_variance_structure(cuda_device):
    """Isotropic data: a half prefix is half of every distance and prunes little (core.py:1100-1102); a Dataset
    offered the cascade stops using it after a pass over the survivor limit, and its steps stay the dense ones."""
    import mlx_kmeans_b200 as km
    rng = np.random.default_rng(5)
    X = rng.standard_normal((20_000, 128)).astype(np.float32)
    C = torch.from_numpy(X[:256].copy()).to(cuda_device)
    a, b = km.Dataset([X]), km.Dataset([X])
    a.cascade = True
    assert a.cascade_ok(256)
    for _ in range(3):
        Na, _ = a.step(C)
        Nb, _ = b.step(C)
        assert torch.equal(Na, Nb)
        C = Na.clone()
    assert not a._cascade[256]["ok"] and not a.cascade_ok(256)
    assert not a.cascade_ok(64) and not a.cascade_ok(256 + 4)       # the reference's shape rule: k >= 256, k % 8


def test_cascade_after_a_pass_with_more_centers(cuda_device):
    """The previous labels come from a pass with more centers (labels past this k): those rows are scored in
    full, and every label is the oracle's."""
    import mlx_kmeans_b200 as km
    X = _anisotropic(20_000, 128, 64, 41)
    rng = np.random.default_rng(41)
    C512 = X[rng.choice(len(X), 512, replace=False)].copy()
    C256 = C512[256:].copy()                      # the rows labelled 256.. before have no center of that index now
    ds = km.Dataset([X])
    ds.assign(torch.from_numpy(C512).to(cuda_device), return_labels=True)
    _, _, _, lab = ds.assign(torch.from_numpy(C256).to(cuda_device), return_labels=True, cascade=True)
    assert ds._cascade[256]["used"]
    ref, _, _ = O.assign(X, C256)
    assert np.array_equal(lab, ref)
