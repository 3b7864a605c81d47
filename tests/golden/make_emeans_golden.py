#!/usr/bin/env python3
"""Fixtures of e-means from the reference's own NumPy code (mlx_kmeans/emeans.py, which imports MLX only inside
its GPU functions).

Run where the reference checkout is mounted, with its directory in REFERENCE_ROOT:

    REFERENCE_ROOT=<reference checkout> python tests/golden/make_emeans_golden.py

Writes tests/golden/emeans/:
  laws.json     batch_size / step0 / plan (emeans.py:60-105) on a grid of (n, k, T) and explicit overrides
  draws.npz     the seeded draws: _init_rows, _epoch_batches, _revive_plan (emeans.py:108-169)
  run_<case>.npz  emeans_reference (emeans.py:192-295, the float64 NumPy e-means) on a seeded case: its input,
                its centres and record, and per batch its labels and revival decisions (its trace)
"""
import json
import os
import sys

import numpy as np

REF = os.environ.get("REFERENCE_ROOT")
if not REF:
    sys.exit("set REFERENCE_ROOT to the reference checkout (kakollu/mlx-kmeans)")
OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "emeans")


def blobs(rng, n, d, true_k, spread, noise):
    centers = rng.uniform(-spread, spread, size=(true_k, d))
    return (centers[rng.integers(0, true_k, n)] + rng.normal(0, noise, (n, d))).astype(np.float32)


def main():
    sys.path.insert(0, REF)
    from mlx_kmeans import emeans as em
    os.makedirs(OUT, exist_ok=True)
    laws = []
    for n in (1_000, 50_000, 1_000_000, 2_000_001, 96_000_000):
        for k in (8, 256, 16384):
            for T in (1, 3, 10):
                if k > n:
                    continue
                B = em.batch_size(n, k, T)
                laws.append(dict(n=n, k=k, T=T, B=B, a0=em.step0(n, k, T, B), plan=em.plan(n, k, T)))
    overrides = [dict(n=1_000_000, k=16384, T=3, batch_size=10_000, step0=None),
                 dict(n=50_000, k=256, T=2, batch_size=None, step0=0.5),
                 dict(n=3_000, k=12, T=4, batch_size=256, step0=1.0)]
    for o in overrides:
        o["plan"] = em.plan(o["n"], o["k"], o["T"], o["batch_size"], o["step0"])
    json.dump(dict(laws=laws, overrides=overrides), open(os.path.join(OUT, "laws.json"), "w"), indent=1)

    draws = {"init_7_5000_20": em._init_rows(7, 5000, 20)}
    for e in range(3):
        draws[f"batches_7_{e}_5000_512"] = em._epoch_batches(7, e, 5000, 512)
    rng = np.random.default_rng(1)
    for i in range(6):
        N = rng.exponential(1.0, 24) * rng.choice([1.0, 1.0, 1e-3], 24)
        if i == 5:
            N[:20] = 0.0                                   # more dead clusters than live ones
        dead, donors = em._revive_plan(N, 11, 5 * i + 4)
        draws[f"revive_N_{i}"], draws[f"revive_dead_{i}"], draws[f"revive_donors_{i}"] = N, dead, donors
    np.savez_compressed(os.path.join(OUT, "draws.npz"), **draws)

    rng = np.random.default_rng(20261202)
    cases = []
    X = blobs(rng, 8000, 8, 16, 10, 1)
    cases.append(("blobs_d8_k16", X, dict(k=16, epochs=3, seed=0)))
    X = blobs(rng, 6000, 6, 6, 5, 1)
    C0 = np.concatenate([X[rng.choice(6000, 8, replace=False)],
                         rng.uniform(60, 80, (4, 6)).astype(np.float32)]).astype(np.float32)
    cases.append(("revive_d6_k12", X, dict(k=12, epochs=2, seed=3, batch_size=256, init=C0)))
    X = blobs(rng, 3000, 4, 5, 3, 1)
    cases.append(("a0one_d4_k10", X, dict(k=10, epochs=2, seed=5, batch_size=3000, step0=1.0)))
    for name, X, kw in cases:
        trace = []
        C, rec = em.emeans_reference(X, trace=trace, **kw)
        out = dict(X=X, centres=C, B=rec["B"], a0=rec["a0"], M=rec["M"], per=rec["batches_per_epoch"],
                   revived=np.array(rec["revived"], np.int64), train_mse=np.array(rec["train_mse"]),
                   last_epoch_counts=rec["last_epoch_counts"], last_labels=rec["last_labels"],
                   k=kw["k"], epochs=kw["epochs"], seed=kw["seed"],
                   batch_size=kw.get("batch_size", -1), step0=kw.get("step0", -1.0),
                   labels=np.stack([t["labels"] for t in trace]), rows=np.stack([t["rows"] for t in trace]))
        if "init" in kw:
            out["init"] = kw["init"]
        checks = [t for t in trace if t["N_check"] is not None]
        out["n_checks"] = len(checks)
        for i, t in enumerate(checks):
            out[f"dead_{i}"], out[f"donors_{i}"] = t["dead"], t["donors"]
        np.savez_compressed(os.path.join(OUT, f"run_{name}.npz"), **out)
        print(name, "B", rec["B"], "M", rec["M"], "revived", sum(rec["revived"]), "mse", rec["train_mse"])


if __name__ == "__main__":
    main()
