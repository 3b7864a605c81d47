"""Float64 NumPy restatement of the reference's e-means reference (mlx_kmeans/emeans.py:192-295), the checker of the
GPU e-means.

TEST INFRASTRUCTURE ONLY: imported by tests/ as the checker; the product (mlx_kmeans_b200) never imports it.

emeans64(X, k, ...) follows emeans_reference step for step: float32 data computed on in float64; N = 1e-10,
S = N C at the start; per batch t (the seeded permutation's sorted cuts, emeans.py:121-136) the labels (its own
float64 nearest centre, lowest index on ties -- or, driven, the labels a fit recorded), counts and sums, the step
a(t) of the cosine schedule (emeans.py:80-82), N <- (1 - a) N + a count, S <- (1 - a) S + a sum, C <- S / N where N > 0;
after every fifth batch the revival of emeans.py:145-169 (or, driven, the decisions a fit recorded); the output is
the last epoch's exact mean per cluster (the moving-average centre for a cluster empty in that epoch).
Pinned against the reference's own runs in tests/golden/emeans/ (tests/test_emeans.py).
"""
import math

import numpy as np


def _batches(seed, e, n, B):
    """The rows of epoch e: stream (seed, 2, e)'s shuffle of range(n), cut into n // B sorted batches."""
    order = np.arange(n, dtype=np.uint32 if n <= 2 ** 32 else np.int64)
    np.random.default_rng([seed, 2, e]).shuffle(order)
    out = order[:(n // B) * B].reshape(n // B, B)
    out.sort(axis=1)
    return out


def _revive(N, seed, t, tau=0.1):
    """Dead clusters (N < tau mean N) and donors drawn from the live ones by Gumbel-top-m keys on log N."""
    u = np.random.default_rng([seed, 3, t]).random(len(N))
    below = N < tau * (N.sum() / len(N))
    dead, live = np.flatnonzero(below), np.flatnonzero(~below)
    m = min(len(dead), len(live))
    if m == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    with np.errstate(divide="ignore"):
        keys = np.log(N[live]) - np.log(-np.log(np.maximum(u[live], np.finfo(np.float64).tiny)))
    return dead[:m].astype(np.int64), live[np.argsort(-keys, kind="stable")[:m]].astype(np.int64)


def nearest64(x, C):
    """Float64 nearest centre, lowest index on ties: each row's distances summed over the columns in NumPy's
    order for a contiguous row, candidates first screened by the expanded form with a margin."""
    csq = (C * C).sum(1)
    approx = csq[None, :] - 2 * x @ C.T
    lo = approx.min(1, keepdims=True)
    win = 1e-9 * ((x * x).sum(1, keepdims=True) + csq[None, :]) + 1e-300
    dist = np.full(approx.shape, np.inf)
    r, c = np.nonzero(approx <= lo + 2 * win)
    dist[r, c] = ((x[r] - C[c]) ** 2).sum(1)
    lab = dist.argmin(1)
    return lab, dist[np.arange(len(x)), lab]


def emeans64(X, k, epochs, seed, B, a0, init, labels=None, revivals=None):
    """-> (centres float64 (k, d), dict(revived, train_mse, last_epoch_counts, trace)).  init: (k, d) starting
    centres; labels: per-batch label arrays to use instead of its own (driven); revivals: per-check (dead, donors)."""
    X64 = np.asarray(X, np.float32).astype(np.float64)
    n, d = X64.shape
    per = n // B
    M = epochs * per
    C = np.asarray(init, np.float32).astype(np.float64)
    N = np.full(k, 1e-10)
    S = C * 1e-10
    even = np.arange(d) % 2 == 0
    p, q = np.where(even, 1 + 2.0 ** -7, 1 - 2.0 ** -7), np.where(even, 1 - 2.0 ** -7, 1 + 2.0 ** -7)
    acc_c, acc_s = np.zeros(k), np.zeros((k, d))
    revived, mse, trace = [], [], []
    t = check = 0
    for e in range(epochs):
        cuts = _batches(seed, e, n, B)
        inertia = 0.0
        for i in range(per):
            rows = cuts[i].astype(np.int64)
            xb = X64[rows]
            if labels is None:
                lab, bd = nearest64(xb, C)
            else:
                lab = np.asarray(labels[t], np.int64)
                bd = ((xb - C[lab]) ** 2).sum(1)
            cnt = np.bincount(lab, minlength=k).astype(np.float64)
            sums = np.zeros((k, d))
            np.add.at(sums, lab, xb)
            a = a0 * (0.1 + 0.9 * 0.5 * (1.0 + math.cos(math.pi * t / M)))
            N = (1.0 - a) * N + a * cnt
            S = (1.0 - a) * S + a * sums
            has = N > 0
            C = np.where(has[:, None], S / np.where(has, N, 1.0)[:, None], C)
            inertia += float(bd.sum())
            if e == epochs - 1:
                acc_c += cnt
                acc_s += sums
            if (t + 1) % 5 == 0:
                dead, donors = _revive(N, seed, t) if revivals is None else \
                    (np.asarray(v, np.int64).reshape(-1) for v in revivals[check])
                check += 1
                revived.append(len(dead))
                if len(dead):
                    cd, half = C[donors], N[donors] * 0.5
                    N[dead], N[donors] = half, half
                    S[dead], S[donors] = (cd * p) * half[:, None], (cd * q) * half[:, None]
                    has = N > 0
                    C = np.where(has[:, None], S / np.where(has, N, 1.0)[:, None], C)
            trace.append(dict(C=C.copy(), N=N.copy()))
            t += 1
        mse.append(inertia / (per * B))
    out = C.copy()
    used = acc_c > 0
    out[used] = acc_s[used] / acc_c[used, None]
    return out, dict(revived=revived, train_mse=mse, last_epoch_counts=acc_c, trace=trace)
