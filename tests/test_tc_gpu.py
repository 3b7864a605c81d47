"""Tensor-core pass (kmc_pass_split: tcgen05 MMA on bf16 hi / lo splits, float64 decision of the rows inside
the error window) against the float64 oracle, the reference's golden outputs and the CUDA-core pass (-m gpu).

Bars: labels bit-exact to the float64 oracle; counts and sums bit-identical to the CUDA-core pass for the
same data (both quantise each value on its own onto the same grid); inertia within 1e-6 of it; sums and
inertia against the oracle as in test_parity_gpu.py.
"""
import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import oracle as O
from test_parity_gpu import _check_assign

pytestmark = pytest.mark.gpu


def _dims(name):
    return int(name.split("_d")[1].split("_")[0]) if "_d" in name else 0


TC_CASES = [c for c in golden_cases() if _dims(c) >= 32]


def _ds(X, device, tc=True, parts=1):
    import torch
    import mlx_kmeans_b200 as km
    Xt = torch.from_numpy(np.ascontiguousarray(X, np.float32)).to(device)
    if parts == 1:
        return km.Dataset([Xt], tensor_cores=tc)
    cuts = np.linspace(0, len(X), parts + 1).astype(int)
    return km.Dataset([Xt[a:b].contiguous() for a, b in zip(cuts[:-1], cuts[1:])], tensor_cores=tc)


def _totals(ds, C):
    import torch
    b = ds.run_pass(torch.from_numpy(np.ascontiguousarray(C)).to(ds.device))
    return b["totals"].cpu().numpy().copy()


@pytest.mark.parametrize("name", TC_CASES)
def test_tc_matches_golden(name, cuda_device):
    import torch
    g = load_golden(name)
    ds = _ds(g["X"], cuda_device)
    out = ds.assign(torch.from_numpy(g["C"]).to(cuda_device), return_labels=True)
    _check_assign(g["X"], g["C"], out, g["labels"])


@pytest.mark.parametrize("name", ["separated_d8_k16", "tiny_n7_d3_k5", "integer_grid_ties_d6_k12", "d1_k7",
                                  "duplicate_centers_d8_k32", "duplicate_points_d8_k64"])
def test_tc_forced_at_low_d(name, cuda_device):
    """Columns padded to 64 and tiny n: the tensor-core pass still gives the oracle's labels."""
    import torch
    g = load_golden(name)
    ds = _ds(g["X"], cuda_device)
    ds.tensor_cores = True
    out = ds.assign(torch.from_numpy(g["C"]).to(cuda_device), return_labels=True)
    _check_assign(g["X"], g["C"], out, g["labels"])


def _embeddings(n, d, k_true, seed):
    """Unit-norm rows around random unit directions (the shape of configuration 4)."""
    rng = np.random.default_rng(seed)
    dirs = rng.standard_normal((k_true, d))
    dirs /= np.linalg.norm(dirs, axis=1, keepdims=True)
    X = dirs[rng.integers(0, k_true, n)] + 0.15 * rng.standard_normal((n, d))
    X /= np.linalg.norm(X, axis=1, keepdims=True)
    return X.astype(np.float32)


@pytest.mark.parametrize("n,d,k", [(20_000, 768, 300), (3_001, 100, 600), (50_000, 128, 512), (4_000, 64, 64),
                                   (30_000, 32, 64), (5_000, 20, 40), (8_000, 64, 2100), (5_000, 72, 4096)])
def test_tc_matches_cuda_core_pass(n, d, k, cuda_device):
    """Ragged row tiles, padded columns, several (padded) center tiles: labels and totals identical to the
    CUDA-core pass, labels identical to the float64 oracle."""
    X = _embeddings(n, d, max(k // 2, 2), n + d)
    C = X[np.random.default_rng(k).choice(n, k, replace=False)].copy()
    tc, cc = _ds(X, cuda_device, tc=True), _ds(X, cuda_device, tc=False)
    import torch
    Ct = torch.from_numpy(C).to(cuda_device)
    lab_tc = tc.assign(Ct, return_labels=True)[3]
    lab_cc = cc.assign(Ct, return_labels=True, generic=True)[3]
    assert np.array_equal(lab_tc, lab_cc), f"{int((lab_tc != lab_cc).sum())} labels differ"
    ta, tb = _totals(tc, C), _generic_totals(cc, C)
    assert np.array_equal(ta[:, [0] + list(range(2, d + 2))], tb[:, [0] + list(range(2, d + 2))])
    # inertia: float64 row distances here, float32 `best` in the CUDA-core pass
    assert abs(int(ta[:, 1].sum()) - int(tb[:, 1].sum())) <= 1e-6 * abs(int(tb[:, 1].sum()))
    if n * k * d <= 2e9:
        ref, _, _ = O.assign(X, C)
        assert np.array_equal(lab_tc, ref)


def _generic_totals(ds, C):
    import torch
    b = ds.run_pass(torch.from_numpy(np.ascontiguousarray(C)).to(ds.device), generic=True)
    return b["totals"].cpu().numpy().copy()


def test_tc_window_flags_few_rows(cuda_device):
    """The error window sends only a small share of embedding rows to float64."""
    import torch
    X = _embeddings(40_000, 768, 200, 3)
    C = X[np.random.default_rng(1).choice(len(X), 256, replace=False)].copy()
    ds = _ds(X, cuda_device)
    C_new, s = ds.step(torch.from_numpy(C).to(cuda_device), bounded=False)
    assert s["rescored"] < 0.05 * len(X), s


def test_tc_lloyd_step_and_slices(cuda_device):
    """A Lloyd step with relocation on the tensor-core path, one slice and three: the same bits, and the
    oracle's step."""
    import mlx_kmeans_b200 as km
    g = load_golden("relocation_8empty_d16_k32")
    X, C = g["X"], g["C"]
    C_ref, inertia_ref, ne_ref, pairs, _, _ = O.lloyd_step(X, C)
    rms = float(np.sqrt((X.astype(np.float64) ** 2).mean()))
    outs = []
    for parts in (1, 3):
        ds = _ds(X, cuda_device, parts=parts)
        ds.tensor_cores = True
        C_new, inertia, n_empty = km.lloyd_step(ds, C)
        assert n_empty == ne_ref
        assert np.max(np.abs(C_new.astype(np.float64) - C_ref)) / rms <= 1e-6
        assert abs(inertia - inertia_ref) <= 1e-6 * inertia_ref
        for c, row in pairs:
            assert np.array_equal(C_new[c], X[row])
        outs.append(C_new)
    assert np.array_equal(outs[0], outs[1])


@pytest.mark.parametrize("k,copies", [(40, [3, 9, 10, 17, 30, 31]), (2500, [3, 9, 10, 700, 2047, 2400]),
                                      (2500, [5, 6]), (2500, [5, 1500]), (4096, [4095, 31, 32, 2048])])
def test_tc_many_equal_centers(k, copies, cuda_device):
    """Copies of one center: rows near it have exact ties.  Two copies are two candidates (decided in float64
    between them, or in full when the per-chunk tracker of many centers finds both in one 32-column chunk), more
    than two take the full float64 decision; the label is the lowest index, as in the oracle.  With 2048 centers
    and more the kernel keeps its top two a chunk at a time (copies in one chunk, in neighbouring chunks, in the
    last and first chunks of the row)."""
    import torch
    rng = np.random.default_rng(5)
    X = rng.standard_normal((5_000, 64)).astype(np.float32)
    C = rng.standard_normal((k, 64)).astype(np.float32) * (1.0 + 0.01 * (k > 100))
    C[copies] = 0.05 * rng.standard_normal(64).astype(np.float32)
    ds = _ds(X, cuda_device)
    out = ds.assign(torch.from_numpy(C).to(cuda_device), return_labels=True)
    ref, _, _ = O.assign(X, C)
    assert np.array_equal(out[3], ref)
    low = min(copies)
    assert (ref == low).sum() > 0 and not np.isin(ref, [c for c in copies if c != low]).any()


@pytest.mark.parametrize("d", [3, 7, 8, 31, 32, 100, 128, 129, 136, 200, 255, 513, 768, 1000, 4096])
def test_d64_warp_bit_identical(d, cuda_device):
    """kmc_d64 (a warp per pair: the leaves' partial chains across lanes, the reference's combination order)
    returns the float64 bits of the oracle's NumPy-pairwise D64, at leaf-only, split and ragged-tail sizes."""
    import torch
    from mlx_kmeans_b200 import _lib
    rng = np.random.default_rng(d)
    m = 64
    X = rng.standard_normal((m, d)).astype(np.float32) * rng.uniform(0.01, 100.0, size=(m, 1)).astype(np.float32)
    C = X + rng.standard_normal((m, d)).astype(np.float32) * np.float32(1e-3)
    C[::7] = X[::7]                                     # zero distances
    Xt, Ct = torch.from_numpy(X).to(cuda_device), torch.from_numpy(C).to(cuda_device)
    out = torch.empty(m, dtype=torch.float64, device=cuda_device)
    L = _lib.load()
    _lib.check(L.kmc_d64(Xt.data_ptr(), Ct.data_ptr(), d, m, out.data_ptr(),
                         torch.cuda.current_stream().cuda_stream))
    got = out.cpu().numpy()
    want = np.array([O.d64(X[i], C[i]) for i in range(m)])
    assert np.array_equal(got.view(np.int64), want.view(np.int64))
