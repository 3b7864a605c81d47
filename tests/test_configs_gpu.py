"""Parity at the benchmark configurations' own shapes, and an audit of the tensor-core error window (-m gpu).

Shapes (rows are slices of each configuration's own generator; k, d as the configuration states):
  config 1   100k x 8, k=8: the reference's make_data_numpy recipe, k-means++ on a 16k-row sample, 20 exact
             Lloyd steps, every step against the oracle's step (labels bit-exact, centers and inertia 1e-6)
  config 2   200k x 32, k=64 (tensor-core pass)
  config 4   20k x 768, k=1024 (tensor-core pass)
  config 5   20k x 128, k=4096 (tensor-core pass)
Bars (the reference's tests/accuracy.py:86-99, tightened): labels bit-exact to the float64 oracle, counts exact,
sums within 1e-7 of the float64 sums (relative to the data RMS x count), inertia and centers within 1e-6.

The window audit reads the raw scores x.c of the tcgen05 pass (kmc_tc_dot) and checks the per-score error bound
the kernel's window is built from: |x.c_tc - x.c| <= E |x| |c| with E = 3.1 2^-16 + 3 dp 2^-24, on
configuration-4/5-shaped data, all-positive data (no cancellation, the accumulator's worst case) and rows of
mixed magnitude; and that rows constructed to be exact and near float64 ties get the oracle's labels.
"""
import numpy as np
import pytest

from oracle import oracle as O
from test_parity_gpu import _check_assign

pytestmark = pytest.mark.gpu


def _slice(cfg, n, device):
    from mlx_kmeans_b200.data import generate
    return generate(cfg, 0, n, device, rows_total=n)


@pytest.mark.parametrize("cfg,n,k", [(2, 200_000, 64), (4, 20_000, 1024), (5, 20_000, 4096)])
def test_tensor_core_configs_match_oracle(cfg, n, k, cuda_device):
    import torch
    import mlx_kmeans_b200 as km
    X = _slice(cfg, n, cuda_device)
    Xh = X.cpu().numpy()
    rng = np.random.default_rng(cfg)
    C = Xh[rng.choice(n, k, replace=False)].copy()
    # the centers moved off the rows a little, as after a Lloyd step
    C += (0.01 * rng.standard_normal(C.shape) * np.abs(Xh).mean()).astype(np.float32)
    ds = km.Dataset([X])
    assert ds.tensor_cores
    out = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True)
    labels_ref, _, _ = O.assign(Xh, C)
    _check_assign(Xh, C, out, labels_ref)
    # and one Lloyd step against the oracle's
    C_new, inertia, n_empty = km.lloyd_step(ds, C)
    C_ref, in_ref, ne_ref, _, _, _ = O.lloyd_step(Xh, C, labels_ref)
    rms = float(np.sqrt((Xh.astype(np.float64) ** 2).mean()))
    assert n_empty == ne_ref
    assert np.max(np.abs(C_new.astype(np.float64) - C_ref)) / rms <= 1e-6
    assert abs(inertia - in_ref) <= 1e-6 * in_ref


@pytest.mark.parametrize("cfg,n,k", [(3, 2_000_000, 16), (2, 200_000, 64), (4, 20_000, 1024), (5, 20_000, 4096)])
def test_both_label_rules_at_config_shapes(cfg, n, k, cuda_device):
    """Each label rule bit-exact to its oracle on a slice of the configuration; the rows where the rules
    disagree are counted (printed: -s)."""
    import torch
    import mlx_kmeans_b200 as km
    X = _slice(cfg, n, cuda_device)
    Xh = X.cpu().numpy()
    rng = np.random.default_rng(cfg + 10)
    C = Xh[rng.choice(n, k, replace=False)].copy()
    C += (0.01 * rng.standard_normal(C.shape) * np.abs(Xh).mean()).astype(np.float32)
    ds = km.Dataset([X])
    Ct = torch.from_numpy(C).to(cuda_device)
    got = {}
    for rule in ("float64", "float32"):
        ref, _, _ = O.assign(Xh, C, rule=rule)
        lab = ds.assign(Ct, return_labels=True, rule=rule)[3]
        assert np.array_equal(lab, ref), f"{rule}: {int((lab != ref).sum())} labels differ"
        got[rule] = lab
    print(f"config {cfg} slice {n} x {Xh.shape[1]}, k={k}: rows labelled differently by the two rules: "
          f"{int((got['float64'] != got['float32']).sum())}")


def test_config1_recipe_step_by_step(cuda_device):
    """Configuration 1 as specified: make_data_numpy(100k, 8, k_true=8, seed 0), k-means++ on a 16k-row sample,
    20 exact Lloyd steps; each step's labels, centers, inertia and empties against the oracle's step."""
    import torch
    import mlx_kmeans_b200 as km
    X = km.make_data_numpy(100_000, 8, 8, 0)[0]
    ds = km.Dataset([X])
    C = km.kmeans_pp_init(ds, len(X), 8, np.random.default_rng(0), sample=16_000)
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean()))
    for step in range(20):
        labels = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True)[3]
        C_ref, in_ref, ne_ref, _, labels_ref, _ = O.lloyd_step(X, C)
        assert np.array_equal(labels, labels_ref), f"step {step}"
        C_gpu, inertia, n_empty = km.lloyd_step(ds, C)
        assert n_empty == ne_ref
        assert np.max(np.abs(C_gpu.astype(np.float64) - C_ref)) / rms <= 1e-6, f"step {step}"
        assert abs(inertia - in_ref) <= 1e-6 * in_ref
        C = C_gpu


# ---------------------------------------------------------------- tensor-core error window

def _tc_scores(X, C, device):
    """(x.c as the tcgen05 pass accumulates it, n x k float32)."""
    import torch
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    n, d = X.shape
    k = C.shape[0]
    Xt = torch.from_numpy(np.ascontiguousarray(X)).to(device)
    Ct = torch.from_numpy(np.ascontiguousarray(C)).to(device)
    sb, cb = int(L.kmc_split_bytes(n, d)), int(L.kmc_csplit_bytes(d, k))
    sp = torch.empty(sb, dtype=torch.uint8, device=device)
    cs = torch.empty(cb, dtype=torch.uint8, device=device)
    out = torch.full((n, k), float("nan"), dtype=torch.float32, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    st = torch.cuda.current_stream().cuda_stream
    _lib.call("kmc_split_rows", Xt.data_ptr(), n, d, sp.data_ptr(), sb, st)
    _lib.call("kmc_tc_dot", Ct.data_ptr(), n, d, k, sp.data_ptr(), sb, cs.data_ptr(), cb, out.data_ptr(),
              err.data_ptr(), st)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out.cpu().numpy()


def _ratio(X, C, device):
    """max over rows and centers of |x.c_tc - x.c| / (|x| |c|), and the window's per-score bound E."""
    s = _tc_scores(X, C, device).astype(np.float64)
    X64, C64 = X.astype(np.float64), C.astype(np.float64)
    exact = X64 @ C64.T
    nx = np.linalg.norm(X64, axis=1)[:, None]
    nc = np.linalg.norm(C64, axis=1)[None, :]
    r = np.abs(s - exact) / np.maximum(nx * nc, 1e-300)
    dp = (X.shape[1] + 63) // 64 * 64
    E = 3.1 / 65536.0 + 3.0 * dp / 16777216.0
    return float(r.max()), E


def _audit_sets():
    rng = np.random.default_rng(17)
    sets = {}
    # configuration 4: unit-norm embeddings around 1024 directions, k = 1024
    dirs = rng.standard_normal((1024, 768))
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    X = dirs[rng.integers(0, 1024, 4096)] + 0.15 * rng.standard_normal((4096, 768))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    sets["config4"] = (X.astype(np.float32), X[:1024].astype(np.float32))
    # configuration 5: 4096-component mixture, k = 4096
    means = 2.0 * rng.standard_normal((4096, 128))
    X = means[rng.integers(0, 4096, 4096)] + rng.standard_normal((4096, 128))
    sets["config5"] = (X.astype(np.float32), (means + 0.1 * rng.standard_normal(means.shape)).astype(np.float32))
    # all products positive: no cancellation, the float32 accumulation's worst case relative to |x||c|
    X = rng.random((2048, 768))
    sets["positive768"] = (X.astype(np.float32), rng.random((512, 768)).astype(np.float32))
    # rows and centers over twenty binades
    X = rng.standard_normal((2048, 256)) * np.exp2(rng.integers(-10, 10, (2048, 1)))
    C = rng.standard_normal((512, 256)) * np.exp2(rng.integers(-10, 10, (512, 1)))
    sets["mixed256"] = (X.astype(np.float32), C.astype(np.float32))
    return sets


@pytest.mark.parametrize("name", ["config4", "config5", "positive768", "mixed256"])
def test_tc_score_error_within_window_bound(name, cuda_device):
    X, C = _audit_sets()[name]
    r, E = _ratio(X, C, cuda_device)
    print(f"{name}: max |x.c_tc - x.c| / (|x||c|) = {r:.3e} = {r / E:.3f} E (E = {E:.3e})")
    assert r <= E


def test_tc_exact_and_near_ties(cuda_device):
    """Rows equidistant in float64 from two centers (c = m +- delta u with exactly representable offsets), and
    rows a few float32 ulps off such ties: the float64 decision gives the oracle's labels, lowest index on ties."""
    import torch
    import mlx_kmeans_b200 as km
    rng = np.random.default_rng(23)
    d, pairs = 128, 64
    # multiples of 2^-10 below 8 in magnitude: m +- 2^-6 is exact in float32, so both distances are sum u_j^2
    M = (np.rint(rng.standard_normal((pairs, d)) * 1024) / 1024).clip(-7.9, 7.9).astype(np.float32)
    U = np.where(rng.random((pairs, d)) < 0.5, -1.0, 1.0).astype(np.float32) * np.float32(2.0 ** -6)
    C = np.concatenate([M + U, M - U, rng.standard_normal((128, d)).astype(np.float32) * 4])
    rows = [M]
    for ulps in (1, 2, 8, 64):
        P = M.copy()
        P[:, 0] = P[:, 0] + np.float32(ulps) * np.spacing(P[:, 0])
        rows.append(P)
    X = np.concatenate(rows + [rng.standard_normal((1000, d)).astype(np.float32)])
    labels_ref, d64, _ = O.assign(X, C)
    ties = sum(1 for i in range(pairs) if O.d64(X[i], C[i]) == O.d64(X[i], C[pairs + i]))
    assert ties == pairs                                   # the construction gives exact float64 ties
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    assert ds.tensor_cores
    out = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True)
    assert np.array_equal(out[3], labels_ref)
    assert np.array_equal(labels_ref[:pairs], np.arange(pairs))   # ties go to the lower index
