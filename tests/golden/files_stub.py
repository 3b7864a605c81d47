"""A deterministic stand-in for KMeans in the file-workflow fixtures (test infrastructure only).

The reference's cluster_file (mlx_kmeans/files.py) cannot fit here (its estimator needs MLX), so its fixtures are
made with this stub in place of the estimator, and the tests run this build's cluster_file with the same stub: the
file handling, feature preparation, labels export, summary and metadata are then compared as written files.
Centers: the first k rows; labels: the float64-nearest of them, lowest index on ties.
"""
import numpy as np


class StubKMeans:
    def __init__(self, n_clusters=8, n_init=1, max_iter=300, tol=1e-4, random_state=None, **_):
        self.n_clusters = n_clusters

    def fit(self, X):
        X = np.asarray(X, np.float32)
        C = X[:self.n_clusters].copy()
        d = ((X.astype(np.float64)[:, None, :] - C.astype(np.float64)[None]) ** 2).sum(2)
        self.labels_ = d.argmin(1)
        self.cluster_centers_ = C
        self.inertia_ = float(d.min(1).sum())
        self.n_iter_ = 1
        return self
