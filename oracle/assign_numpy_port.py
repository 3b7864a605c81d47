"""The reference's CPU Lloyd pass, restated in NumPy for the CPU-baseline timing.

TEST/BASELINE INFRASTRUCTURE ONLY: bench.py times it as `cpu_baseline` and as the `--impl reference`
arm; the product never imports it.

assign_numpy follows kakollu/mlx-kmeans mlx_kmeans/core.py:197-215 (chunked expanded-form float32
distances through a BLAS matmul, argmin, float64 bincount sums); cpu_lloyd_pass adds the center update
of the NumPy backend in core.py:2255-2262 (sums / counts; empty clusters keep their center here, the
reference re-seeds them from random rows).
"""
import numpy as np


def assign_numpy(parts, C, chunk=2_000_000):
    """One pass: nearest-center labels -> per-cluster sums (float64), counts, inertia (core.py:197-215)."""
    k, d = C.shape
    sums = np.zeros((k, d), dtype=np.float64)
    counts = np.zeros(k, dtype=np.int64)
    inertia = 0.0
    c_sq = (C * C).sum(1)
    for X in parts:
        for s in range(0, len(X), chunk):
            x = X[s:s + chunk]
            dist = c_sq[None, :] - 2.0 * (x @ C.T)
            lab = dist.argmin(1)
            x_sq = np.einsum("ij,ij->i", x, x)
            inertia += float((x_sq + dist[np.arange(len(x)), lab]).sum())
            counts += np.bincount(lab, minlength=k)
            for j in range(d):
                sums[:, j] += np.bincount(lab, weights=x[:, j], minlength=k)
    return sums, counts, inertia


def cpu_lloyd_pass(parts, C, chunk=2_000_000):
    """assign_numpy followed by the center divide (core.py:2255-2259)."""
    sums, counts, inertia = assign_numpy(parts, C, chunk)
    newC = C.copy()
    has = counts > 0
    newC[has] = (sums[has] / counts[has, None]).astype(np.float32)
    return newC, inertia, int((~has).sum())
