"""GPU parity: libkmc.so against the CPU oracle and the reference's golden outputs (run with -m gpu).

Bars (the reference's tests/accuracy.py:86-99, tightened where the design allows):
  labels   bit-exact to the float64 oracle (lowest index on exact ties)
  counts   exact
  sums     within 1e-7 of the float64 sums, relative to |data| RMS x count (reference bar: 1e-6 for centers)
  inertia  within 1e-6 relative of sum over rows of the float32 `best` in float64
  centers  (Lloyd step) within 1e-6 relative to the data RMS; relocated clusters bit-equal to their row
"""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import oracle as O

pytestmark = pytest.mark.gpu

CASES = golden_cases()


def _torch():
    import torch
    return torch


def _ds(X, device, parts=1):
    import mlx_kmeans_b200 as km
    torch = _torch()
    Xt = torch.from_numpy(np.ascontiguousarray(X, np.float32)).to(device)
    if parts == 1:
        return km.Dataset([Xt])
    cuts = np.linspace(0, len(X), parts + 1).astype(int)
    return km.Dataset([Xt[a:b].contiguous() for a, b in zip(cuts[:-1], cuts[1:])])


def _check_assign(X, C, out, labels_ref, rule="float64"):
    sums, counts, inertia, labels = out
    assert np.array_equal(labels, labels_ref), f"{int((labels != labels_ref).sum())} labels differ"
    k, d = C.shape
    ref_counts = np.bincount(labels_ref, minlength=k)
    assert np.array_equal(counts, ref_counts)
    ref_sums = np.zeros((k, d))
    np.add.at(ref_sums, labels_ref, X.astype(np.float64))
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean())) or 1.0
    err = np.abs(sums - ref_sums) / (rms * np.maximum(ref_counts, 1)[:, None])
    assert err.max() <= 1e-7
    _, _, best = O.assign(X, C, rule=rule)
    ref_inertia = float(best.astype(np.float64).sum())
    assert abs(inertia - ref_inertia) <= 1e-6 * max(ref_inertia, 1e-30)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("path", ["auto", "generic", "tensor_cores"])
def test_float32_rule_matches_golden(name, path, cuda_device):
    """label_rule="float32" (the reference's rows kernel, core.py:263-274) on every path: labels bit-exact to the
    NumPy restatement recorded in the fixtures (and so to the oracle's float32 rule)."""
    g = load_golden(name)
    ds = _ds(g["X"], cuda_device)
    if path == "tensor_cores":
        ds.tensor_cores = True
    C = _torch().from_numpy(g["C"]).to(cuda_device)
    out = ds.assign(C, return_labels=True, generic=(path == "generic"), rule="float32")
    _check_assign(g["X"], g["C"], out, g["labels32"], rule="float32")


def _rules_apart_lowd(n, d, k, seed):
    """Low-d rows around pairs of centers a few float32 ulps apart: the two centers' distances differ by about
    their float32 rounding, so the float32 direct sum and the float64 distance pick different centers for a
    share of the rows."""
    rng = np.random.default_rng(seed)
    base = rng.uniform(-4, 4, (k // 2, d)).astype(np.float32)
    step = (rng.integers(1, 4, base.shape) * np.where(rng.random(base.shape) < 0.5, -1, 1)).astype(np.float32)
    C = np.concatenate([base, base + step * np.spacing(base)]).astype(np.float32)
    X = (base[rng.integers(0, k // 2, n)] + 0.5 * rng.standard_normal((n, d))).astype(np.float32)
    return X, C


@pytest.mark.parametrize("d,k", [(4, 16), (2, 32), (8, 8), (3, 6)])
def test_float32_rule_low_d_fused_bounded_generic(d, k, cuda_device):
    """The fused low-d kernel, the bounded pass (after a step whose bounds are then used) and the generic kernel
    under the float32 rule against the oracle's, on data where the two rules disagree."""
    import mlx_kmeans_b200 as km
    torch = _torch()
    X, C = _rules_apart_lowd(60_000, d, k, d * 100 + k)
    l64, _, _ = O.assign(X, C)
    l32, _, _ = O.assign(X, C, rule="float32")
    assert (l64 != l32).sum() > 0
    ds = _ds(X, cuda_device)
    Ct = torch.from_numpy(C).to(cuda_device)
    for generic in (False, True):
        out = ds.assign(Ct, return_labels=True, generic=generic, rule="float32")
        _check_assign(X, C, out, l32, rule="float32")
    # bounded steps: the first writes the bounds, the second (same centers, zero drift) keeps labels by them
    bd = _ds(X, cuda_device)
    bd.label_rule = "float32"
    for _ in range(2):
        bd.step(Ct, bounded=True)
    assert np.array_equal(_word_labels(bd, k), l32)
    C_ref, in_ref, ne_ref, _, _, _ = O.lloyd_step(X, C, rule="float32")
    C_new, inertia, n_empty = km.lloyd_step(bd, C, label_rule="float32")
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean()))
    assert n_empty == ne_ref
    assert np.max(np.abs(C_new.astype(np.float64) - C_ref)) / rms <= 1e-6
    assert abs(inertia - in_ref) <= 1e-6 * in_ref


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("generic", [False, True])
def test_assign_matches_golden(name, generic, cuda_device):
    g = load_golden(name)
    ds = _ds(g["X"], cuda_device)
    C = _torch().from_numpy(g["C"]).to(cuda_device)
    out = ds.assign(C, return_labels=True, generic=generic)
    _check_assign(g["X"], g["C"], out, g["labels"])


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("relocation")] + ["separated_d8_k16",
                                                                                   "offset1000_d8_k64"])
def test_lloyd_step_matches_oracle(name, cuda_device):
    import mlx_kmeans_b200 as km
    g = load_golden(name)
    X, C = g["X"], g["C"]
    C_ref, inertia_ref, ne_ref, pairs, _, _ = O.lloyd_step(X, C)
    ds = _ds(X, cuda_device)
    C_new, inertia, n_empty = km.lloyd_step(ds, C)
    assert n_empty == ne_ref
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean()))
    assert np.max(np.abs(C_new.astype(np.float64) - C_ref)) / rms <= 1e-6
    assert abs(inertia - inertia_ref) <= 1e-6 * inertia_ref
    for c, row in pairs:
        assert np.array_equal(C_new[c], X[row]), f"relocated cluster {c} is not row {row}"
    if "C_new" in g:       # and against the reference's own float64 Lloyd step
        assert np.max(np.abs(C_new - g["C_new"])) / rms <= 1e-6


def test_slices_give_the_same_bits(cuda_device):
    g = load_golden("separated_d8_k16")
    C = _torch().from_numpy(g["C"]).to(cuda_device)
    one = _ds(g["X"], cuda_device).assign(C, return_labels=True)
    three = _ds(g["X"], cuda_device, parts=3).assign(C, return_labels=True)
    for a, b in zip(one, three):
        assert np.array_equal(np.asarray(a), np.asarray(b))


def test_refit_is_bit_identical(cuda_device):
    """tests/reuse.py:64-68: a refit on the same data gives the same bits."""
    import mlx_kmeans_b200 as km
    rng = np.random.default_rng(7)
    A = rng.standard_normal((40_000, 8)).astype(np.float32)
    m1 = km.KMeans(n_clusters=16, max_iter=5, random_state=0).fit(A)
    m2 = km.KMeans(n_clusters=16, max_iter=5, random_state=0).fit(A.copy())
    assert m1.inertia_ == m2.inertia_
    assert np.array_equal(m1.cluster_centers_, m2.cluster_centers_)
    assert np.array_equal(m1.labels_, m2.labels_)


def test_pp_init_matches_oracle(cuda_device):
    import mlx_kmeans_b200 as km
    torch = _torch()
    rng = np.random.default_rng(11)
    S = (rng.uniform(-10, 10, (32, 6))[rng.integers(0, 32, 5000)] + rng.standard_normal((5000, 6))).astype(np.float32)
    for k in (1, 2, 33, 100):
        seeds = rng.integers(2**63 - 1, size=max(k - 1, 0)).astype(np.uint64)
        picks_ref, C_ref = O.pp_init(S, k, 123, seeds)
        C = km.pp_init_device(torch.from_numpy(S).to(cuda_device), k, 123, seeds)
        picks = km.pp_init_device.last_picks.cpu().numpy()
        assert np.array_equal(picks, picks_ref), f"k={k}"
        assert np.array_equal(C.cpu().numpy(), C_ref)


def test_fit_matches_oracle_loop(cuda_device):
    """KMeans.fit against the oracle's Lloyd loop from the same device k-means++ start."""
    import mlx_kmeans_b200 as km
    X = km.make_data_numpy(20_000, 5, 12, 3)[0]
    m = km.KMeans(n_clusters=12, max_iter=8, tol=0.0, random_state=4).fit(X)
    # the same start, then the oracle's steps
    ds = km.Dataset([X])
    C = km.kmeans_pp_init(ds, len(X), 12, np.random.default_rng(4))
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean()))
    for _ in range(m.n_iter_):
        C_ref, _, _, _, _, _ = O.lloyd_step(X, C)
        C_gpu, _, _ = km.lloyd_step(ds, C)
        assert np.max(np.abs(C_gpu - C_ref)) / rms <= 1e-6
        C = C_gpu
    assert np.array_equal(C, m.cluster_centers_)
    labels, _, best = O.assign(X, m.cluster_centers_)
    assert np.array_equal(m.labels_, labels)
    assert abs(m.inertia_ - float(best.astype(np.float64).sum())) <= 1e-6 * m.inertia_


def test_errors_match_the_reference(cuda_device):
    import mlx_kmeans_b200 as km
    rng = np.random.default_rng(0)
    m = km.KMeans(n_clusters=8, max_iter=2, random_state=0).fit(rng.standard_normal((5000, 8)).astype(np.float32))
    with pytest.raises(ValueError, match="features"):
        m.predict(rng.standard_normal((300, 16)).astype(np.float32))
    with pytest.raises(ValueError, match="tiles"):
        km.assign_mlx([rng.standard_normal((3000, 12)).astype(np.float32)], np.zeros((100, 12), np.float32),
                      method="tiles")
    bad = rng.standard_normal((1000, 4)).astype(np.float32)
    bad[7, 2] = np.nan
    with pytest.raises(ValueError, match="NaN"):
        km.KMeans(n_clusters=4, max_iter=2, random_state=0).fit(bad)
    huge = rng.standard_normal((1000, 4)).astype(np.float32)
    huge[3, 1] = 3e37
    with pytest.raises(ValueError, match="largest coordinate"):
        km.KMeans(n_clusters=4, max_iter=2, random_state=0).fit(huge)
    with pytest.raises(ValueError, match="n_clusters"):
        km.KMeans(n_clusters=50).fit(rng.standard_normal((10, 3)).astype(np.float32))


# ---------------------------------------------------------------- the fused low-dimensional kernel

def _oracle_totals(X, labels, k):
    sums = np.zeros((k, X.shape[1]))
    np.add.at(sums, labels, X.astype(np.float64))
    return sums, np.bincount(labels, minlength=k)


def test_config1_full_fused_vs_generic_vs_oracle(cuda_device):
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200.data import generate
    torch = _torch()
    X = generate(1, 0, 100_000, cuda_device)
    Xh = X.cpu().numpy()
    C = Xh[np.random.default_rng(0).choice(len(Xh), 8, replace=False)].copy()
    ds = km.Dataset([X])
    Cd = torch.from_numpy(C).to(cuda_device)
    fused = ds.assign(Cd, return_labels=True)
    generic = ds.assign(Cd, return_labels=True, generic=True)
    ref_labels, _, best = O.assign(Xh, C)
    _check_assign(Xh, C, fused, ref_labels)
    _check_assign(Xh, C, generic, ref_labels)
    assert np.array_equal(fused[1], generic[1])


def test_config3_slice_matches_oracle(cuda_device):
    """2M rows of the 96M-row configuration (same generator, standardised over the slice)."""
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200.data import generate
    torch = _torch()
    X = generate(3, 0, 2_000_000, cuda_device, rows_total=2_000_000)
    Xh = X.cpu().numpy()
    C = Xh[np.random.default_rng(3).choice(len(Xh), 16, replace=False)].copy()
    ds = km.Dataset([X])
    b = ds.run_pass(torch.from_numpy(C).to(cuda_device), labels=True)
    labels = b["labels"][0].cpu().numpy()
    best = b["best"][0].cpu().numpy()
    ref_labels, _, ref_best = O.assign(Xh, C)
    assert np.array_equal(labels, ref_labels)
    assert np.array_equal(best.view(np.uint32), ref_best.view(np.uint32)), "best must be bit-exact"
    out = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True)
    _check_assign(Xh, C, out, ref_labels)


def test_fused_is_deterministic_and_block_split_invariant(cuda_device):
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200 import _lib
    from mlx_kmeans_b200.data import generate
    torch = _torch()
    blk = int(_lib.load().kmc_row_block(0))
    n = 37 * blk + 1234
    X = generate(3, 0, n, cuda_device, rows_total=n)
    C = X[torch.arange(0, 16, device=cuda_device) * 997].contiguous()
    a = km.Dataset([X]).assign(C, return_labels=True)
    b = km.Dataset([X]).assign(C, return_labels=True)
    cuts = [0, 5 * blk, 21 * blk, n]
    c = km.Dataset([X[lo:hi] for lo, hi in zip(cuts[:-1], cuts[1:])]).assign(C, return_labels=True)
    for u, v, w in zip(a, b, c):
        assert np.array_equal(np.asarray(u), np.asarray(v))
        assert np.array_equal(np.asarray(u), np.asarray(w))


@pytest.mark.parametrize("bounded", [False, True])
def test_large_blocks_are_split_invariant(bounded, cuda_device):
    """From 64M rows in all the fused kernels fold 160 rows per lane (20480-row blocks, kmc_row_block): passes
    over one slice and over three slices cut at block multiples, with the global row count of such a dataset,
    give the same totals bit for bit (plain and bounded kernels, the bounded one after a pass that built its
    bounds), and the labels of the 8192-row-block pass."""
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200 import _lib
    from mlx_kmeans_b200.data import generate
    torch = _torch()
    L = _lib.load()
    n_total = 64_000_000
    blk = int(L.kmc_row_block(n_total))
    assert blk == 20480 and int(L.kmc_row_block(n_total - 1)) == 8192
    n = 37 * blk + 1234
    X = generate(3, 0, n, cuda_device, rows_total=n)
    C = X[torch.arange(0, 16, device=cuda_device) * 997].contiguous()
    ds = km.Dataset([X])
    ref_labels = ds.assign(C, return_labels=True)[3]
    cm, b = ds.colmax, ds.buffers(16)
    st = torch.cuda.current_stream().cuda_stream
    lab = torch.empty(n, dtype=torch.int32, device=cuda_device)

    def run(cuts):
        tot = torch.zeros((16, 6), dtype=torch.int64, device=cuda_device)
        for i, (lo, hi) in enumerate(zip(cuts[:-1], cuts[1:])):
            flags = _lib.KMC_PASS_ACCUMULATE if i else 0
            if bounded:
                nb = int(L.kmc_bounds_bytes(hi - lo, 4, 16))
                bb = torch.zeros(nb, dtype=torch.uint8, device=cuda_device)
                for _ in range(2):          # the first pass writes the bounds, the second uses them
                    t2 = torch.zeros_like(tot)
                    _lib.call("kmc_pass_bounded", X[lo:hi].data_ptr(), hi - lo, 4, C.data_ptr(), 16, cm.data_ptr(),
                              n_total, t2.data_ptr(), 0, bb.data_ptr(), nb, b["ws"].data_ptr(), b["wsb"], st)
                tot += t2
            else:
                _lib.call("kmc_pass", X[lo:hi].data_ptr(), hi - lo, 4, C.data_ptr(), 16, cm.data_ptr(), n_total,
                          tot.data_ptr(), lab[lo:hi].data_ptr(), None, flags, b["ws"].data_ptr(), b["wsb"], st)
        torch.cuda.synchronize()
        return tot.cpu().numpy()

    one = run([0, n])
    three = run([0, 5 * blk, 21 * blk, n])
    assert np.array_equal(one, three)
    assert one[:, 0].sum() == n
    if not bounded:
        assert np.array_equal(lab.cpu().numpy().astype(np.int64), ref_labels)


def test_window_rows_are_rescored(cuda_device):
    """Exact float64 ties (integer grid, mirrored centers) must reach the float64 re-scoring."""
    import mlx_kmeans_b200 as km
    g = load_golden("integer_grid_ties_d6_k12")
    ds = _ds(g["X"], cuda_device)
    C = _torch().from_numpy(g["C"]).to(cuda_device)
    _, s = ds.step(C)
    assert s["rescored"] > 50
    labels = ds.assign(C, return_labels=True)[3]
    assert np.array_equal(labels, g["labels"])


# ---------------------------------------------------------------- per-row bounds (kmc_pass_bounded)

def _word_labels(ds, k):
    """Labels stored in the low bits of the bound words of a one-slice Dataset."""
    from mlx_kmeans_b200 import _lib
    buf, nbytes = ds.bounds(k)[0]
    n, d = ds.parts[0].shape
    a256 = lambda v: (v + 255) // 256 * 256
    off = 256 + a256(k * d * 4)            # after the drift record and the centers of the last pass
    words = buf[off:off + n * 4].view(torch_int32()).cpu().numpy().view(np.uint32)
    kp = next(v for v in (2, 4, 8, 16, 32) if v >= k)
    return (words & (kp - 1)).astype(np.int64)


def torch_int32():
    import torch
    return torch.int32


@pytest.mark.parametrize("cfg,n", [(3, 1_000_000), (1, 100_000)])
def test_bounded_steps_match_full_steps(cfg, n, cuda_device):
    """Lloyd steps with per-row bounds against full steps from the same start: identical counts, empties,
    labels (read back from the bound words), inertia within 1e-7 relative and centers within one float32 ulp
    (plus 1e-7 of the data RMS) at every step."""
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200.data import CONFIGS, generate
    torch = _torch()
    X = generate(cfg, 0, n, cuda_device, rows_total=n)
    k = CONFIGS[cfg]["k"]
    rng = np.random.default_rng(1)
    C0 = X[torch.from_numpy(rng.choice(n, k, replace=False)).to(cuda_device)].contiguous()
    rms = float(torch.sqrt((X.double() ** 2).mean()))
    a, b = km.Dataset([X]), km.Dataset([X])
    Ca, Cb = C0.clone(), C0.clone()
    screened = []
    for step in range(8):
        Na, sa = a.step(Ca, bounded=True)
        Nb, sb = b.step(Cb, bounded=False)
        assert sa["n_empty"] == sb["n_empty"]
        # per-lane float32 partials of `best` are summed in another order once rows are queued
        assert abs(sa["inertia"] - sb["inertia"]) <= 1e-7 * sb["inertia"]
        lab_full = b.assign(Cb, return_labels=True)[3]
        assert np.array_equal(_word_labels(a, k), lab_full), f"step {step}: labels differ"
        assert np.array_equal(a.assign(Ca)[1], b.assign(Cb)[1])
        # the same holds for the per-lane partial sums of x (and the float32 fold of the lanes): the last
        # float32 bit of a center may move -- one unit in the last place of the center, or 1e-7 of the data RMS
        # for a center near zero
        tol = torch.abs(Nb).double() * 2.0 ** -23 + 1e-7 * rms
        assert bool(((Na - Nb).abs().double() <= tol).all())
        screened.append(sa["screened"])
        Ca, Cb = Na.clone(), Nb.clone()
    assert screened[0] == n                       # the first pass compares every row
    assert min(screened[3:]) < n // 2             # later passes keep most labels from their bounds


def test_bounds_survive_a_jump_of_the_centers(cuda_device):
    """Centers replaced by unrelated ones (a restart without reset): the drift makes every bound fail and
    the pass is still exact."""
    import mlx_kmeans_b200 as km
    from mlx_kmeans_b200.data import generate
    torch = _torch()
    n, k = 300_000, 16
    X = generate(3, 0, n, cuda_device, rows_total=n)
    ds = km.Dataset([X])
    C = X[:k].contiguous()
    for _ in range(3):
        C, _ = ds.step(C, bounded=True)
        C = C.clone()
    C2 = X[1000:1000 + k].contiguous() * 0.5
    _, s = ds.step(C2, bounded=True)
    ref = km.Dataset([X]).assign(C2, return_labels=True)[3]
    assert np.array_equal(_word_labels(ds, k), ref)
