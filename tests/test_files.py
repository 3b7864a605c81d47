"""The file workflow (mlx_kmeans_b200.files) against the reference's own cluster_file (mlx_kmeans/files.py).

CPU tier: the fixtures in tests/golden/files/ are the reference's outputs, made by tests/golden/make_files_golden.py
with a deterministic stand-in estimator (files_stub.StubKMeans); this build's cluster_file runs on the same inputs
with the same stand-in and must write the same files: labeled.csv and cluster_summary.csv byte for byte, run.json
and model.npz equal (paths and timings aside), and the same error messages for rejected calls.
GPU tier: one case end to end with the real KMeans: the exported labels are the oracle's for the fitted centers.
"""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN

FILES = os.path.join(GOLDEN, "files")
CASES = sorted(d for d in os.listdir(FILES) if os.path.isdir(os.path.join(FILES, d)))
VOLATILE = ("input", "preparation_s", "fit_including_labels_s")


def _input(case):
    d = os.path.join(FILES, case)
    return os.path.join(d, next(f for f in os.listdir(d) if f.startswith("input.")))


@pytest.fixture
def stub(monkeypatch):
    import sys
    sys.path.insert(0, GOLDEN)
    from files_stub import StubKMeans
    from mlx_kmeans_b200 import estimator
    monkeypatch.setattr(estimator, "KMeans", StubKMeans)


@pytest.mark.parametrize("case", CASES)
def test_outputs_match_the_reference(case, tmp_path, stub):
    from mlx_kmeans_b200 import files
    d = os.path.join(FILES, case)
    want = json.load(open(os.path.join(d, "run.json")))
    res = files.cluster_file(_input(case), output=str(tmp_path / "out"), **want["kwargs"])
    out = tmp_path / "out"
    for fn in ("labeled.csv", "cluster_summary.csv"):
        assert (out / fn).read_bytes() == open(os.path.join(d, fn), "rb").read(), fn
    run = json.load(open(out / "run.json"))
    for key in VOLATILE:
        run.pop(key)
    assert run == want["run"]
    got, ref = np.load(out / "model.npz"), np.load(os.path.join(d, "model.npz"))
    assert sorted(got.files) == sorted(ref.files)
    for key in ref.files:
        assert np.array_equal(got[key], ref[key]), key
    assert res["run"]["clustered_rows"] == want["run"]["clustered_rows"]


def test_errors_match_the_reference(tmp_path, stub):
    from mlx_kmeans_b200 import files
    want = json.load(open(os.path.join(FILES, "errors.json")))
    base = os.path.join(FILES, "drop_missing")
    calls = {
        "missing_error": dict(path=os.path.join(base, "input.csv"), columns=["spend", "visits"], k=4),
        "absent_column": dict(path=os.path.join(base, "input.csv"), columns=["spend", "nope"], k=4, missing="drop"),
        "bad_k": dict(path=os.path.join(base, "input.csv"), columns=["spend"], k=0),
        "bad_tol": dict(path=os.path.join(base, "input.csv"), columns=["spend"], k=2, tol=-1.0),
        "bad_missing": dict(path=os.path.join(base, "input.csv"), columns=["spend"], k=2, missing="zero"),
        "columns_str": dict(path=os.path.join(base, "input.csv"), columns="spend", k=2),
        "too_few_rows": dict(path=os.path.join(base, "input.csv"), columns=["spend", "visits"], k=5000,
                             missing="drop"),
        "all_constant": dict(path=os.path.join(FILES, "tsv_collision", "input.tsv"), columns=["const"], k=2),
        "not_found": dict(path=os.path.join(base, "absent.csv"), columns=["spend"], k=2),
        "bad_suffix": dict(path=os.path.join(GOLDEN, "INDEX.txt"), columns=["spend"], k=2),
    }
    assert sorted(calls) == sorted(want)
    for name, kw in calls.items():
        path = kw.pop("path")
        with pytest.raises(ValueError) as e:
            files.cluster_file(path, output=str(tmp_path / name), **kw)
        assert str(e.value).replace(os.path.dirname(path), "<dir>") == want[name], name
        assert not (tmp_path / name).exists()


def test_existing_output_is_never_overwritten(tmp_path, stub):
    from mlx_kmeans_b200 import files
    (tmp_path / "taken").mkdir()
    with pytest.raises(ValueError, match="already exists"):
        files.cluster_file(_input("raw_units"), output=str(tmp_path / "taken"), columns=["spend"], k=2)


def test_inspect_file_and_read_table():
    from mlx_kmeans_b200 import files
    head = files.inspect_file(_input("drop_missing"))
    assert list(head.columns) == ["id", "spend", "visits", "segment", "note"] and len(head) == 5
    table = files.read_table(_input("tsv_collision"))
    assert list(table.columns) == ["cluster", "x", "y", "const"] and len(table) == 200


@pytest.mark.gpu
def test_cluster_file_end_to_end(tmp_path, cuda_device):
    """The real fit: every exported label is the oracle's nearest fitted center of the standardised row."""
    import pandas as pd
    from mlx_kmeans_b200 import files
    from oracle import oracle as O
    res = files.cluster_file(_input("drop_missing"), output=str(tmp_path / "o"), columns=["spend", "visits"], k=4,
                             missing="drop", n_init=2)
    run = res["run"]
    table = pd.read_csv(tmp_path / "o" / "labeled.csv")
    kept = table[["spend", "visits"]].apply(pd.to_numeric, errors="coerce").to_numpy(np.float64)
    valid = np.isfinite(kept).all(1)
    X = ((kept[valid] - np.array(run["feature_mean"])) / np.array(run["feature_scale"])).astype(np.float32)
    centers = np.load(tmp_path / "o" / "model.npz")["centers"]
    labels, _, best = O.assign(X, centers)
    assert np.array_equal(table[run["label_column"]].to_numpy()[valid].astype(np.int64), labels + 1)
    assert table[run["label_column"]].isna().sum() == run["excluded_rows"]
    assert abs(run["inertia"] - float(best.astype(np.float64).sum())) <= 1e-6 * run["inertia"]
