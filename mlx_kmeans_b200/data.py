"""The five benchmark configurations as seeded synthetic data, generated on the device shard by shard.

Every row is a function of (seed, global row index) (libkmc kmc_gen, Philox4x32-10), so the rows a GPU holds
are the same whether one GPU or eight generate them. Mixture parameters come from NumPy's default_rng(seed).

    1  100k x 8,  k=8:    8 blob centers uniform in [-10,10]^8, sd 1 (the reference's make_data_numpy recipe)
    2  10M x 32,  k=64:   uniform [0,1)
    3  96M x 4,   k=16:   16 anisotropic Gaussians, means U[0.05,0.6]^4, per-dim sd U[0.01,0.08], equal
                          weights, clipped to [0,1], standardised per column (float64 mean / std)
    4  1M x 768,  k=1024: 1024 unit directions + N(0, 0.15^2) noise, rows renormalised
    5  50M x 128, k=4096: 4096 component means N(0, 4I), within-component sd 1
"""
import numpy as np
import torch

from . import _lib

CONFIGS = {
    1: dict(rows=100_000, dims=8, k=8, seed=0, iters=20, pp_sample=16_000),
    2: dict(rows=10_000_000, dims=32, k=64, seed=1, iters=25, pp_sample=256_000),
    3: dict(rows=96_000_000, dims=4, k=16, seed=2, iters=30, pp_sample=None),
    4: dict(rows=1_000_000, dims=768, k=1024, seed=3, iters=15, pp_sample=None),
    5: dict(rows=50_000_000, dims=128, k=4096, seed=5, iters=10, pp_sample=None),
}

DESCRIPTION = {
    1: "config1: 100k x 8 f32 Gaussian blobs, k=8",
    2: "config2: 10M x 32 f32 uniform [0,1), k=64",
    3: "config3: 96M x 4 f32, 16 anisotropic Gaussians clipped to [0,1] and standardised, k=16",
    4: "config4: 1M x 768 f32 unit-norm embeddings (1024 directions + N(0,0.15^2)), k=1024",
    5: "config5: 50M x 128 f32, 4096-component Gaussian mixture (means N(0,4I), sd 1), k=4096",
}


def mixture_params(cfg):
    """(kind, means (ncomp, d), sds (ncomp, d), lo, hi) of a configuration, from default_rng(seed)."""
    c = CONFIGS[cfg]
    rng = np.random.default_rng(c["seed"])
    d = c["dims"]
    if cfg == 1:
        means = rng.uniform(-10, 10, size=(8, d)).astype(np.float32)
        return 1, means, np.ones_like(means), 0.0, 0.0
    if cfg == 2:
        return 0, None, None, 0.0, 0.0
    if cfg == 3:
        means = rng.uniform(0.05, 0.6, size=(16, d)).astype(np.float32)
        sds = rng.uniform(0.01, 0.08, size=(16, d)).astype(np.float32)
        return 1, means, sds, 0.0, 1.0
    if cfg == 4:
        dirs = rng.standard_normal((1024, d))
        dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
        return 2, dirs.astype(np.float32), np.full((1024, d), 0.15, np.float32), 0.0, 0.0
    if cfg == 5:
        means = (2.0 * rng.standard_normal((4096, d))).astype(np.float32)
        return 1, means, np.ones_like(means), 0.0, 0.0
    raise ValueError(f"unknown configuration {cfg}")


def column_scales(d, r, seed):
    """Per-column factors r^p(j), p a permutation from default_rng(seed): applied to a configuration's rows they
    give data whose column spread falls off geometrically in an unordered way (the variance structure of SIFT-like
    descriptors), the case the prefix-pruning cascade is for."""
    p = np.random.default_rng(seed + 0x5C).permutation(d)
    return (float(r) ** p).astype(np.float32)


def shard_range(n_total, rank, world, align=None):
    """Contiguous rows [lo, hi) of rank `rank` of `world`; every boundary a multiple of `align` (default: the
    library's row block, so the totals are bit-identical for any number of GPUs)."""
    if align is None:
        align = int(_lib.load().kmc_row_block(n_total))
    blocks = (n_total + align - 1) // align
    lo = min(n_total, (blocks * rank // world) * align)
    hi = min(n_total, (blocks * (rank + 1) // world) * align)
    return lo, hi


def generate(cfg, row0, n, device, rows_total=None, group=None):
    """Rows [row0, row0 + n) of configuration cfg as a (n, d) float32 CUDA tensor. Config 3 is standardised
    with the mean and std of ALL rows_total rows (summed over `group` when sharded)."""
    c = CONFIGS[cfg]
    d = c["dims"]
    seed = 0x6B6D63 * 1000 + c["seed"]
    kind, means, sds, lo, hi = mixture_params(cfg)
    X = torch.empty((n, d), dtype=torch.float32, device=device)
    st = torch.cuda.current_stream().cuda_stream
    md = torch.from_numpy(means).to(device) if means is not None else None
    sd = torch.from_numpy(sds).to(device) if sds is not None else None
    _lib.call("kmc_gen", kind, X.data_ptr(), n, d, row0, seed, md.data_ptr() if md is not None else None,
              sd.data_ptr() if sd is not None else None, 0 if means is None else len(means), lo, hi, st)
    if cfg == 3:
        standardise(X, rows_total or n, group)
    return X


def standardise(X, n_total, group=None):
    """In place (x - mean) / std per column, mean/std over all n_total rows (all ranks), exact sums."""
    n, d = X.shape
    st = torch.cuda.current_stream().cuda_stream
    cm = torch.zeros(d, dtype=torch.int32, device=X.device)
    _lib.call("kmc_colmax", X.data_ptr(), n, d, cm.data_ptr(), 0, st)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(cm, op=dist.ReduceOp.MAX, group=group)
    sums = torch.zeros(2 * d, dtype=torch.int64, device=X.device)
    _lib.call("kmc_colsums", X.data_ptr(), n, d, cm.data_ptr(), n_total, sums.data_ptr(), st)
    if group is not None:
        import torch.distributed as dist
        dist.all_reduce(sums, op=dist.ReduceOp.SUM, group=group)
    ms = torch.empty(2 * d, dtype=torch.float64, device=X.device)
    _lib.call("kmc_standardize", X.data_ptr(), n, d, sums.data_ptr(), cm.data_ptr(), n_total, ms.data_ptr(), st)
    return ms


def host_sample(cfg, n, seed_offset=0):
    """A host NumPy sample of configuration cfg's distribution (for the CPU baseline, which runs without a
    GPU): the same mixture parameters, NumPy's own normal draws, config 3 standardised over the sample."""
    c = CONFIGS[cfg]
    d = c["dims"]
    rng = np.random.default_rng(1000 + c["seed"] + seed_offset)
    kind, means, sds, lo, hi = mixture_params(cfg)
    if kind == 0:
        return rng.random((n, d), dtype=np.float32)
    comp = rng.integers(0, len(means), n)
    X = means[comp] + sds[comp] * rng.standard_normal((n, d), dtype=np.float32)
    if lo < hi:
        np.clip(X, lo, hi, out=X)
    if kind == 2:
        X /= np.linalg.norm(X.astype(np.float64), axis=1, keepdims=True).astype(np.float32)
    if cfg == 3:
        X64 = X.astype(np.float64)
        X = ((X64 - X64.mean(0)) / X64.std(0)).astype(np.float32)
    return np.ascontiguousarray(X, dtype=np.float32)
