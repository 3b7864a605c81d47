"""Exact k-means (Lloyd) on NVIDIA B200 GPUs: the hot path of kakollu/mlx-kmeans, rebuilt on hand-written
sm_100a CUDA kernels behind a C ABI (include/kmc.h, libkmc.so).

    from mlx_kmeans_b200 import KMeans
    km = KMeans(n_clusters=64).fit(X)        # X: (rows, dims) float32
    km.cluster_centers_, km.labels_, km.inertia_

Every label is the center with the smallest float64 distance, lowest index on exact ties; per-cluster totals
are exact integers, so results are bit-reproducible and independent of how rows are split over GPUs.
"""
from .core import (  # noqa: F401
    Dataset, assign, assign_mlx, kmeans, kmeans_pp_init, lloyd_step, make_data_numpy, pp_init_device,
    slice_rows, take_rows,
)
from .estimator import KMeans  # noqa: F401

__version__ = "0.1.0"
__all__ = ["KMeans", "Dataset", "kmeans", "lloyd_step", "assign_mlx", "assign", "kmeans_pp_init",
           "make_data_numpy", "take_rows", "slice_rows"]
