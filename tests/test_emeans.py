"""e-means (mlx_kmeans_b200.emeans) against the reference's own e-means (mlx_kmeans/emeans.py).

CPU tier (fixtures in tests/golden/emeans/, made by make_emeans_golden.py from the reference's NumPy code):
  - the batch and step laws and plan() on a grid of (n, k, T) and overrides, exactly;
  - the seeded draws (initial rows, epoch batches, revival donors), exactly;
  - the oracle's float64 restatement (oracle/emeans_port.py) against the reference's float64 e-means runs: centres,
    revivals, per-epoch MSE and last-epoch counts equal.
GPU tier, the reference's own bars (its tests/emeans.py: driven by the fit's labels and revival decisions, the
trajectory within 1e-5 and the last-epoch means within 1e-6 of the RMS coordinate; here tighter where the
arithmetic allows):
  - every batch's labels are the float64-nearest of the float32 centres the batch was assigned against (bit-exact
    to the oracle), and every revival decision is the shared draw on the N the fit read;
  - the oracle driven by the fit's labels and decisions follows the fit's centres to 1e-7 and ends at the same
    centres to 1e-6 of the RMS coordinate;
  - same seed, same bits; KMeans(algorithm="emeans") end to end.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

EM = os.path.join(GOLDEN, "emeans")
RUNS = sorted(f[4:-4] for f in os.listdir(EM) if f.startswith("run_"))


def _run(name):
    z = np.load(os.path.join(EM, f"run_{name}.npz"))
    return {k: z[k] for k in z.files}


def test_laws_and_plan():
    from mlx_kmeans_b200 import emeans as em
    f = json.load(open(os.path.join(EM, "laws.json")))
    for r in f["laws"]:
        B = em.batch_size(r["n"], r["k"], r["T"])
        assert B == r["B"] and em.step0(r["n"], r["k"], r["T"], B) == r["a0"]
        assert em.plan(r["n"], r["k"], r["T"]) == r["plan"]
    for o in f["overrides"]:
        assert em.plan(o["n"], o["k"], o["T"], o["batch_size"], o["step0"]) == o["plan"]
    for bad in [(0, 3, 1), (10, 20, 1), (10, 3, 0)]:
        with pytest.raises(ValueError):
            em.plan(*bad)
    with pytest.raises(ValueError):
        em.plan(100, 3, 1, step0_=1.5)


def test_seeded_draws():
    from mlx_kmeans_b200 import emeans as em
    z = np.load(os.path.join(EM, "draws.npz"))
    assert np.array_equal(em._init_rows(7, 5000, 20), z["init_7_5000_20"])
    for e in range(3):
        assert np.array_equal(em._epoch_batches(7, e, 5000, 512), z[f"batches_7_{e}_5000_512"])
    for i in range(6):
        dead, donors = em._revive_plan(z[f"revive_N_{i}"], 11, 5 * i + 4)
        assert np.array_equal(dead, z[f"revive_dead_{i}"]) and np.array_equal(donors, z[f"revive_donors_{i}"])


@pytest.mark.parametrize("name", RUNS)
def test_oracle_reproduces_the_reference_runs(name):
    from oracle.emeans_port import emeans64
    from mlx_kmeans_b200 import emeans as em
    r = _run(name)
    n = len(r["X"])
    init = r["init"] if "init" in r else r["X"][em._init_rows(int(r["seed"]), n, int(r["k"]))]
    C, rec = emeans64(r["X"], int(r["k"]), int(r["epochs"]), int(r["seed"]), int(r["B"]), float(r["a0"]), init)
    assert np.array_equal(C, r["centres"])
    assert rec["revived"] == r["revived"].tolist()
    assert np.array_equal(rec["train_mse"], r["train_mse"])
    assert np.array_equal(rec["last_epoch_counts"], r["last_epoch_counts"])


# ---------------------------------------------------------------- GPU

def _fit(name, device, assign="exact", trace=None):
    import torch
    from mlx_kmeans_b200 import emeans as em
    r = _run(name)
    kw = dict(k=int(r["k"]), epochs=int(r["epochs"]), seed=int(r["seed"]))
    if int(r["batch_size"]) > 0:
        kw["batch_size"] = int(r["batch_size"])
    if float(r["step0"]) > 0:
        kw["step0"] = float(r["step0"])
    if "init" in r:
        kw["init"] = r["init"]
    C, rec = em.emeans_fit([torch.from_numpy(r["X"]).to(device)], assign=assign, trace=trace, **kw)
    return r, C, rec


@pytest.mark.gpu
@pytest.mark.parametrize("name", RUNS)
def test_fit_against_the_driven_oracle(name, cuda_device):
    from oracle import oracle as O
    from oracle.emeans_port import emeans64, _revive
    trace = []
    r, C, rec = _fit(name, cuda_device, trace=trace)
    X = r["X"]
    assert rec["B"] == int(r["B"]) and rec["a0"] == float(r["a0"]) and rec["M"] == int(r["M"])
    X64 = X.astype(np.float64)
    rms = float(np.sqrt((X64 ** 2).mean()))
    for tr in trace:
        lab, _, _ = O.assign(X[tr["rows"]], tr["C_before"])
        assert np.array_equal(tr["labels"], lab), f"batch {tr['t']}"
        if tr["N_check"] is not None:
            dead, donors = _revive(tr["N_check"], rec["seed"], tr["t"])
            assert np.array_equal(dead, tr["dead"]) and np.array_equal(donors, tr["donors"])
    checks = [(tr["dead"], tr["donors"]) for tr in trace if tr["N_check"] is not None]
    Co, ro = emeans64(X, rec["k"], rec["epochs"], rec["seed"], rec["B"], rec["a0"], rec["init_centres"],
                      labels=[tr["labels"] for tr in trace], revivals=checks)
    drift = max(float(np.abs(tr["C"] - to["C"]).max()) for tr, to in zip(trace, ro["trace"]))
    # the batch sums are exact integers of each value, or (the fused low-d kernel) of per-lane float32 partials of
    # the residuals: the parity suite's sums bar, 1e-7 of the RMS coordinate (the reference's own: 1e-5)
    assert drift <= 1e-7 * rms, drift
    assert np.abs(C.astype(np.float64) - Co).max() <= 1e-6 * rms
    assert rec["revived"] == ro["revived"]
    assert np.array_equal(rec["last_epoch_counts"], ro["last_epoch_counts"])
    assert np.allclose(rec["train_mse"], ro["train_mse"], rtol=1e-6)


@pytest.mark.gpu
def test_same_seed_same_bits_and_estimator(cuda_device):
    import mlx_kmeans_b200 as km
    r = _run("blobs_d8_k16")
    _, C1, rec1 = _fit("blobs_d8_k16", cuda_device)
    _, C2, rec2 = _fit("blobs_d8_k16", cuda_device)
    assert np.array_equal(C1, C2) and rec1["train_mse"] == rec2["train_mse"]
    # the free-running fit ends near the reference's own float64 run (same draws; labels can differ only where the
    # float32 centres' rounding decides a tie)
    rms = float(np.sqrt((r["X"].astype(np.float64) ** 2).mean()))
    assert np.abs(C1 - r["centres"]).max() <= 1e-4 * rms
    m = km.KMeans(n_clusters=16, algorithm="emeans", epochs=3, random_state=0, n_init=2).fit(r["X"])
    assert m.n_iter_ == 3 and m.emeans_record_["B"] == int(r["B"])
    from oracle import oracle as O
    lab, _, best = O.assign(r["X"], m.cluster_centers_)
    assert np.array_equal(m.labels_, lab)
    assert abs(m.inertia_ - float(best.astype(np.float64).sum())) <= 1e-6 * m.inertia_
    with pytest.raises(ValueError):
        km.KMeans(n_clusters=4, algorithm="emeans", spherical=True).fit(r["X"])
    with pytest.raises(ValueError):
        km.KMeans(n_clusters=4, algorithm="emeans", batch_size=10**9).fit(r["X"])
