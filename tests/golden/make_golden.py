#!/usr/bin/env python3
"""Generate the golden fixtures in tests/golden/ from the reference's own Python oracle.

Run where the reference checkout is mounted, with its directory in REFERENCE_ROOT:

    REFERENCE_ROOT=<reference checkout> python tests/golden/make_golden.py

It imports the reference's float64 test oracle (tests/accuracy.py: `reference`, lines 31-51, and
`reference_lloyd_step`, lines 108-129) and its CPU path (mlx_kmeans/core.py:197-215 `assign_numpy`),
none of which needs MLX, and records their outputs on seeded cases shaped after the reference's own
case list (tests/accuracy.py:254-318), scaled down so every fixture stays small. The GPU box has no
reference checkout; the tests there read only the .npz files written here.
"""
import importlib.util
import os
import sys

import numpy as np

REF = os.environ.get("REFERENCE_ROOT")
if not REF:
    sys.exit("set REFERENCE_ROOT to the reference checkout (kakollu/mlx-kmeans)")
OUT = os.path.dirname(os.path.abspath(__file__))


def _load_reference():
    sys.path.insert(0, REF)
    spec = importlib.util.spec_from_file_location("ref_accuracy", os.path.join(REF, "tests", "accuracy.py"))
    acc = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(acc)
    import mlx_kmeans.core as core
    return acc, core


def rows_kernel_labels(X, C):
    """NumPy restatement of the reference's exact-mode label rule, its rows kernel (mlx_kmeans/core.py:263-274,
    a Metal kernel that cannot run here): for each center in index order s = s + t * t with t = x_j - c_j over
    the columns in order, every operation a float32 operation rounded on its own (NumPy does not fuse the
    multiply and add), and the center is taken when s < best. -> (labels int64, best float32)."""
    n, d = X.shape
    best = np.full(n, np.inf, np.float32)
    lab = np.zeros(n, np.int64)
    for c in range(len(C)):
        s = np.zeros(n, np.float32)
        for j in range(d):
            t = X[:, j] - C[c, j]
            s = s + t * t
        lt = s < best
        best = np.where(lt, s, best)
        lab = np.where(lt, c, lab)
    return lab, best


def blobs(rng, n, d, true_k, spread, noise):
    centers = rng.uniform(-spread, spread, size=(true_k, d))
    return (centers[rng.integers(0, true_k, n)] + rng.normal(0, noise, (n, d))).astype(np.float32)


def cases(rng):
    """(name, X, C, relocation?) -- the reference's case list at fixture size."""
    out = []
    X = blobs(rng, 3000, 8, 16, 10, 1)
    out.append(("separated_d8_k16", X, X[rng.choice(len(X), 16, replace=False)], False))
    X = blobs(rng, 2000, 32, 32, 1, 1)
    out.append(("overlapping_d32_k256", X, X[rng.choice(len(X), 256, replace=False)], False))
    X = blobs(rng, 2000, 16, 4, 10, 1)
    out.append(("k_gg_true_d16_k512", X, X[rng.choice(len(X), 512, replace=False)], False))
    X = blobs(rng, 2000, 8, 8, 10, 1)
    C = X[rng.choice(len(X), 32, replace=False)]
    C[16:] = C[:16]
    out.append(("duplicate_centers_d8_k32", X, C, False))
    X = np.repeat(blobs(rng, 250, 8, 8, 10, 1), 8, axis=0)
    out.append(("duplicate_points_d8_k64", X, X[rng.choice(len(X), 64, replace=False)], False))
    X = blobs(rng, 7, 3, 2, 10, 1)
    out.append(("tiny_n7_d3_k5", X, X[:5].copy(), False))
    X = (blobs(rng, 2000, 8, 16, 10, 1) + 1000).astype(np.float32)
    out.append(("offset1000_d8_k64", X, X[rng.choice(len(X), 64, replace=False)], False))
    X = rng.random((1000, 128), dtype=np.float32) * 255
    out.append(("uniform255_d128_k64", X, X[rng.choice(len(X), 64, replace=False)], False))
    X = blobs(rng, 300, 960, 50, 1, 1)
    out.append(("high_d960_k16", X, X[rng.choice(len(X), 16, replace=False)], False))
    X = np.concatenate([blobs(rng, 1000, 64, 8, 10, 1), np.zeros((16, 64), np.float32)])[:1009]
    out.append(("zero_rows_tail_d64_k16", X, X[rng.choice(1000, 16, replace=False)], False))
    X = blobs(rng, 4000, 4, 16, 1, 0.3)
    X = ((X - X.mean(0)) / X.std(0)).astype(np.float32)
    out.append(("standardised_d4_k16", X, X[rng.choice(len(X), 16, replace=False)], False))
    X = blobs(rng, 3000, 1, 5, 10, 1)
    out.append(("d1_k7", X, X[rng.choice(len(X), 7, replace=False)], False))
    X = blobs(rng, 3000, 2, 4, 10, 1) + 1000
    out.append(("offset1000_d2_k4", X.astype(np.float32), X[rng.choice(len(X), 4, replace=False)].astype(np.float32),
                False))
    # exact float64 ties that are not duplicate centers: integer points, centers mirrored about them
    X = rng.integers(-4, 5, size=(2000, 6)).astype(np.float32)
    C = rng.integers(-4, 5, size=(12, 6)).astype(np.float32)
    C[6:] = -C[:6]
    out.append(("integer_grid_ties_d6_k12", X, C, False))
    X = blobs(rng, 1500, 33, 10, 3, 1)
    out.append(("ragged_d33_k40", X, X[rng.choice(len(X), 40, replace=False)], False))
    # relocation (core.py:2224-2236): clusters parked far away empty on the first step
    X = blobs(rng, 3000, 16, 8, 10, 1)
    C = np.concatenate([X[rng.choice(len(X), 24, replace=False)], rng.uniform(900, 1000, (8, 16)).astype(np.float32)])
    out.append(("relocation_8empty_d16_k32", X, C, True))
    X = blobs(rng, 3000, 12, 16, 10, 1)
    C = np.concatenate([X[rng.choice(len(X), 31, replace=False)], rng.uniform(900, 1000, (1, 12)).astype(np.float32)])
    out.append(("relocation_1empty_d12_k32", X, C, True))
    X = blobs(rng, 2000, 4, 4, 10, 1)
    C = np.concatenate([X[rng.choice(len(X), 12, replace=False)], rng.uniform(900, 1000, (4, 4)).astype(np.float32)])
    out.append(("relocation_4empty_d4_k16", X, C, True))
    # the two label rules apart: rows far from every center (float32 sums of ~2^20 lose the last bits that
    # separate the centers) around pairs of centers a few float32 ulps apart
    X = (blobs(rng, 3000, 16, 8, 1, 0.5) + 1000).astype(np.float32)
    C = X[rng.choice(len(X), 8, replace=False)].copy()
    C = np.concatenate([C, C + np.float32(2.0 ** -15) * rng.standard_normal(C.shape).astype(np.float32)])
    C = (C - 1000).astype(np.float32)
    out.append(("rules_apart_d16_k16", X, C, False))
    return out


def main():
    acc, core = _load_reference()
    rng = np.random.default_rng(20261201)
    index = []
    for name, X, C, reloc in cases(rng):
        X = np.ascontiguousarray(X, np.float32)
        C = np.ascontiguousarray(C, np.float32)
        labels, best_d = acc.reference(X, C)
        sums_np, counts_np, inertia_np = core.assign_numpy([X], C)
        labels32, best32 = rows_kernel_labels(X, C)
        rec = dict(X=X, C=C, labels=labels.astype(np.int64), best_d=best_d.astype(np.float64),
                   np_sums=sums_np, np_counts=counts_np, np_inertia=np.float64(inertia_np),
                   labels32=labels32, best32=best32)
        if reloc:
            C_new, n_empty = acc.reference_lloyd_step(X, C, labels)
            rec.update(C_new=C_new.astype(np.float64), n_empty=np.int64(n_empty))
        np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **rec)
        index.append(name)
        print(f"{name:32s} n={len(X):6d} d={X.shape[1]:4d} k={len(C):4d}  "
              f"rows whose float32-rule label differs: {int((labels32 != labels).sum())}")
    with open(os.path.join(OUT, "INDEX.txt"), "w") as f:
        f.write("\n".join(index) + "\n")


if __name__ == "__main__":
    main()
