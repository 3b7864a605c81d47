"""The CPU oracle, pinned against the reference's own outputs (CPU tier, no GPU).

Golden fixtures in tests/golden/ were produced by the reference's float64 test oracle (tests/accuracy.py:31-51,
108-129) and its CPU path (core.py:197-215); tests/golden/make_golden.py regenerates them.
"""
import math

import numpy as np
import pytest

from conftest import golden_cases, load_golden
from oracle import oracle as O
from oracle.assign_numpy_port import assign_numpy

CASES = golden_cases()


def test_fixture_set_present():
    assert len(CASES) >= 18


@pytest.mark.parametrize("name", CASES)
def test_labels_and_distances_bit_exact(name):
    g = load_golden(name)
    labels, d64, best = O.assign(g["X"], g["C"])
    assert np.array_equal(labels, g["labels"]), "labels differ from tests/accuracy.py::reference"
    assert np.array_equal(d64, g["best_d"]), "float64 distances differ in the last bit"
    # best is the float32 distance to the same center
    assert best.dtype == np.float32 and np.all(np.isfinite(best))


@pytest.mark.parametrize("name", CASES)
def test_cpu_path_port_matches_reference_assign_numpy(name):
    g = load_golden(name)
    sums, counts, inertia = assign_numpy([g["X"]], g["C"])
    assert np.array_equal(counts, g["np_counts"])
    assert np.array_equal(sums, g["np_sums"])
    assert inertia == float(g["np_inertia"])


@pytest.mark.parametrize("name", [c for c in CASES if c.startswith("relocation")])
def test_lloyd_step_with_relocation(name):
    g = load_golden(name)
    C_new, inertia, n_empty, pairs, labels, best = O.lloyd_step(g["X"], g["C"])
    assert n_empty == int(g["n_empty"]) > 0
    assert len(pairs) == n_empty
    scale = float(np.sqrt((g["X"].astype(np.float64) ** 2).mean()))
    assert np.max(np.abs(C_new - g["C_new"])) / scale <= 1e-6
    # relocated clusters are exactly their far row, farthest first, ascending cluster index
    for c, row in pairs:
        assert np.array_equal(C_new[c], g["X"][row])
    far = [row for _, row in pairs]
    assert all(best[far[i]] >= best[far[i + 1]] for i in range(len(far) - 1))
    assert [c for c, _ in pairs] == sorted(c for c, _ in pairs)


def test_exact_ties_go_to_lowest_index():
    g = load_golden("integer_grid_ties_d6_k12")
    X, C = g["X"], g["C"]
    X64, C64 = X.astype(np.float64), C.astype(np.float64)
    D = ((X64[:, None, :] - C64[None]) ** 2).sum(2)
    ties = (D == D.min(1, keepdims=True)).sum(1) > 1
    assert ties.sum() > 50, "the fixture must hold exact float64 ties"
    labels, _, _ = O.assign(X, C)
    assert np.array_equal(labels[ties], D[ties].argmin(1))


def test_duplicate_centers_never_use_the_higher_copy():
    g = load_golden("duplicate_centers_d8_k32")
    labels, _, _ = O.assign(g["X"], g["C"])
    assert labels.max() < 16


# (includes every length tests/test_tc_gpu.py::test_d64_warp_bit_identical compares the GPU's D64 at)
@pytest.mark.parametrize("d", [1, 2, 3, 7, 8, 9, 15, 16, 17, 31, 32, 64, 100, 127, 128, 129, 136, 200, 255, 256,
                               513, 768, 960, 1000, 1537, 4096])
def test_d64_is_numpy_pairwise(d):
    rng = np.random.default_rng(d)
    for _ in range(40):
        x = (rng.standard_normal(d) * 10.0 ** rng.integers(-6, 6, d)).astype(np.float32)
        c = (rng.standard_normal(d) * 10.0 ** rng.integers(-6, 6, d)).astype(np.float32)
        ref = ((x.astype(np.float64)[None] - c.astype(np.float64)[None]) ** 2).sum(1)[0]
        assert O.d64(x, c) == ref


def test_philox_known_answers():
    # Random123 known-answer vectors for Philox4x32-10
    assert list(O.philox([0, 0, 0, 0], [0, 0])) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    assert list(O.philox([0xffffffff] * 4, [0xffffffff] * 2)) == [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]
    assert list(O.philox([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], [0xa4093822, 0x299f31d0])) == \
        [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]


def test_log_accuracy():
    rng = np.random.default_rng(3)
    for v in np.concatenate([rng.random(2000), 10.0 ** rng.uniform(-300, 300, 500)]):
        if v <= 0:
            continue
        a, b = O.log(v), math.log(v)
        assert abs(a - b) <= 2e-15 * max(abs(b), 1.0)   # a few ulp: it only shapes a sampling distribution


def test_pp_init_properties():
    rng = np.random.default_rng(5)
    S = rng.standard_normal((3000, 5)).astype(np.float32)
    seeds = rng.integers(2**63 - 1, size=63).astype(np.uint64)
    picks, C = O.pp_init(S, 64, 17, seeds)
    assert picks[0] == 17
    assert len(set(picks.tolist())) == 64
    assert np.array_equal(C, S[picks])
    picks2, _ = O.pp_init(S, 64, 17, seeds)
    assert np.array_equal(picks, picks2)


def test_pp_init_spreads_over_clusters():
    """Greedy k-means++ on well-separated blobs takes one seed per blob (core.py:65-69 motivation)."""
    rng = np.random.default_rng(9)
    centers = rng.uniform(-100, 100, (8, 4))
    lab = rng.integers(0, 8, 4000)
    S = (centers[lab] + rng.standard_normal((4000, 4))).astype(np.float32)
    seeds = rng.integers(2**63 - 1, size=7).astype(np.uint64)
    picks, _ = O.pp_init(S, 8, 0, seeds)
    assert len(set(lab[picks].tolist())) == 8


@pytest.mark.parametrize("name", CASES)
def test_float32_rule_matches_the_rows_kernel_restatement(name):
    """The oracle's float32 label rule against the NumPy restatement of the reference's rows kernel
    (core.py:263-274) recorded in the fixtures: labels and the float32 distances bit-exact."""
    g = load_golden(name)
    labels, _, best = O.assign(g["X"], g["C"], rule="float32")
    assert np.array_equal(labels, g["labels32"])
    assert np.array_equal(best.view(np.uint32), g["best32"].view(np.uint32))


def test_the_label_rules_disagree_only_inside_the_float32_rounding():
    """Where the two rules pick different centers, the float32 direct sums of both centers are within the sum's
    relative error bound gamma_{d+2} of each other (and the float64 distances differ by at most that too)."""
    g = load_golden("rules_apart_d16_k16")
    X, C = g["X"], g["C"]
    l64, l32 = g["labels"], g["labels32"]
    diff = np.nonzero(l64 != l32)[0]
    assert len(diff) > 0
    d = X.shape[1]
    gam = (d + 2) * 2.0 ** -24 / (1 - (d + 2) * 2.0 ** -24)
    for i in diff:
        a, b = O.d64(X[i], C[l64[i]]), O.d64(X[i], C[l32[i]])
        assert a <= b <= a * (1 + gam) / (1 - gam)
