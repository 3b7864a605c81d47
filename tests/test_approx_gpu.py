"""exact=False: the approximate tensor-core assignment (-m gpu).

The reference's exact=False labels come from an fp16 matrix product with no error bound (core.py:859-1088); its
own tests pin them loosely (tests/reuse.py:61: at most 10% of rows wrong after a stale copy, ~0.1% for fp16
itself), so their parity is unpinned. Here the approximate pass (one bf16 product per score, no window) is pinned
by what it can guarantee:
  - every row's label is within the bf16 product's error of the optimum: D(x, c_approx) - D(x, c_best) <=
    4 (2^-7 + dp 2^-24) |x| max|c| (twice the per-score bound of x.c from bf16 operands, on two scores);
  - on configuration-4-shaped data at most 1% of the labels differ from the exact pass and the inertia is within
    1e-4 of the exact inertia (it is never below it);
  - counts, sums and inertia are exact for the labels it gives (the float32 rows are summed, not the bf16 copy);
  - a fit with exact=False ends within 1e-3 of the exact fit's inertia, and below 64 dims it is the exact path.
"""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _embeddings(n, d, k_true, seed):
    rng = np.random.default_rng(seed)
    dirs = rng.standard_normal((k_true, d))
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    X = dirs[rng.integers(0, k_true, n)] + 0.15 * rng.standard_normal((n, d))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


@pytest.mark.parametrize("n,d,k", [(20_000, 768, 1024), (30_000, 128, 512), (20_000, 64, 96)])
def test_approx_labels_within_the_bf16_bound(n, d, k, cuda_device):
    import torch
    import mlx_kmeans_b200 as km
    X = _embeddings(n, d, max(k // 2, 2), n + d)
    rng = np.random.default_rng(k)
    C = X[rng.choice(n, k, replace=False)] + np.float32(0.02) * rng.standard_normal((k, d)).astype(np.float32)
    C = C.astype(np.float32)
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    assert ds.uses_approx(True)
    Ct = torch.from_numpy(C).to(cuda_device)
    sums, counts, inertia, lab = ds.assign(Ct, return_labels=True, approx=True)
    ref, d64_best, _ = O.assign(X, C)
    X64, C64 = X.astype(np.float64), C.astype(np.float64)
    d_apx = ((X64 - C64[lab]) ** 2).sum(1)
    dp = (d + 63) // 64 * 64
    bound = 4.0 * (2.0 ** -7 + dp * 2.0 ** -24) * np.linalg.norm(X64, axis=1) * np.linalg.norm(C64, axis=1).max()
    assert np.all(d_apx - d64_best <= bound * (1 + 1e-6) + 1e-12)
    assert (lab != ref).mean() <= 0.01
    # exact totals of the labels it gave
    assert np.array_equal(counts, np.bincount(lab, minlength=k))
    ref_sums = np.zeros((k, d))
    np.add.at(ref_sums, lab, X64)
    rms = float(np.sqrt((X64 ** 2).mean()))
    assert (np.abs(sums - ref_sums) / (rms * np.maximum(counts, 1)[:, None])).max() <= 1e-7
    assert abs(inertia - d_apx.sum()) <= 1e-6 * d_apx.sum()
    exact_inertia = float(d64_best.sum())
    assert exact_inertia <= inertia * (1 + 1e-12) and inertia <= exact_inertia * (1 + 1e-4)


def test_approx_fit_and_predict(cuda_device):
    import mlx_kmeans_b200 as km
    X = _embeddings(40_000, 256, 300, 1)
    a = km.KMeans(n_clusters=256, max_iter=10, tol=0.0, random_state=0, exact=False).fit(X)
    e = km.KMeans(n_clusters=256, max_iter=10, tol=0.0, random_state=0, exact=True).fit(X)
    assert abs(a.inertia_ - e.inertia_) <= 1e-3 * e.inertia_
    # predict on a second array: the reference allows 10% wrong (tests/reuse.py:61); the bf16 product gets far fewer
    B = _embeddings(20_000, 256, 300, 2)
    ref, _, _ = O.assign(B, a.cluster_centers_)
    assert (a.predict(B) != ref).mean() <= 0.01


def test_approx_below_its_crossover_is_exact(cuda_device):
    import torch
    import mlx_kmeans_b200 as km
    X = _embeddings(20_000, 32, 64, 5)
    C = X[:64].copy()
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    assert not ds.uses_approx(True)
    lab = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True, approx=True)[3]
    assert np.array_equal(lab, O.assign(X, C)[0])
