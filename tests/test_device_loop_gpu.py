"""The Lloyd loop on the device (kmc_lloyd + kmc_loop_init, -m gpu).

The loop's stopping rule runs in the finish kernel (estimator.py:132-150: stop once |prev - inertia| <=
tol * prev) and the steps queued after it stopped do nothing, so a fit reads the host once at the end. Bar: the
same bits as the step-by-step loop (Dataset.step per step, the tol test on the host) -- centers, inertia, the
number of steps, labels -- with bounded and plain passes, both label rules, and a run where relocation interrupts
the device loop and it resumes.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _stepwise(ds, C, max_iter, tol, generic=False, bounded=True, rule=None):
    """The reference's loop (estimator.py:132-150) one Dataset.step at a time."""
    prev, inertia, it = None, float("nan"), 0
    for it in range(max_iter):
        C_new, s = ds.step(C, generic=generic, bounded=bounded, rule=rule)
        C = C_new.clone()
        inertia = s["inertia"]
        if prev is not None and abs(prev - inertia) <= tol * prev:
            break
        prev = inertia
    return C, inertia, it + 1


@pytest.mark.parametrize("d,k,tol,generic,bounded,rule", [
    (4, 16, 1e-4, False, True, "float64"), (4, 16, 0.0, False, False, "float64"), (8, 8, 1e-6, False, True, "float32"),
    (12, 24, 1e-4, True, False, "float64"), (2, 32, 1e-5, False, True, "float64")])
def test_device_loop_matches_stepwise(d, k, tol, generic, bounded, rule, cuda_device):
    import mlx_kmeans_b200 as km
    X = km.make_data_numpy(200_000, d, k, d + k)[0]
    C0 = X[np.random.default_rng(k).choice(len(X), k, replace=False)].copy()
    C0t = torch.from_numpy(C0).to(cuda_device)
    a = km.Dataset([X])
    assert a.device_loop_ok(generic)
    Ca, ia, na, fa = a.lloyd_loop(C0t, 25, tol, generic=generic, bounded=bounded, rule=rule)
    b = km.Dataset([X])
    Cb, ib, nb = _stepwise(b, C0t, 25, tol, generic=generic, bounded=bounded, rule=rule)
    assert na == nb and ia == ib and fa == 0
    assert torch.equal(Ca, Cb)


def test_device_loop_resumes_after_relocation(cuda_device):
    """Centers parked far away: the first step empties clusters, the device loop stops for the host's
    relocation of that step and resumes; the result is the step-by-step loop's."""
    import mlx_kmeans_b200 as km
    from conftest import load_golden
    g = load_golden("relocation_4empty_d4_k16")
    X, C0 = g["X"], g["C"]
    C0t = torch.from_numpy(C0).to(cuda_device)
    a, b = km.Dataset([X]), km.Dataset([X])
    Ca, ia, na, _ = a.lloyd_loop(C0t, 12, 0.0)
    Cb, ib, nb = _stepwise(b, C0t, 12, 0.0)
    assert na == nb and ia == ib
    assert torch.equal(Ca, Cb)


def test_kmeans_fit_uses_the_device_loop(cuda_device, monkeypatch):
    """KMeans.fit through the device loop gives the bits of the step-by-step fit (the same estimator with the
    device loop switched off)."""
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200 import core
    X = km.make_data_numpy(100_000, 8, 8, 0)[0]
    calls = []
    orig = core.Dataset.lloyd_loop

    def spy(self, *args, **kw):
        calls.append(1)
        return orig(self, *args, **kw)
    monkeypatch.setattr(core.Dataset, "lloyd_loop", spy)
    m1 = km.KMeans(n_clusters=8, max_iter=30, random_state=0).fit(X)
    assert calls
    monkeypatch.setattr(core.Dataset, "device_loop_ok", lambda self, generic=False: False)
    m2 = km.KMeans(n_clusters=8, max_iter=30, random_state=0).fit(X)
    assert m1.n_iter_ == m2.n_iter_ and m1.inertia_ == m2.inertia_
    assert np.array_equal(m1.cluster_centers_, m2.cluster_centers_)
    assert np.array_equal(m1.labels_, m2.labels_)
