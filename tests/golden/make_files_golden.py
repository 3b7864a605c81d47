#!/usr/bin/env python3
"""Fixtures of the file workflow from the reference's own cluster_file (mlx_kmeans/files.py:95-180).

Run where the reference checkout is mounted, with its directory in REFERENCE_ROOT:

    REFERENCE_ROOT=<reference checkout> python tests/golden/make_files_golden.py

Each case writes an input table under tests/golden/files/<case>/input.*, runs the reference's cluster_file on it
with files_stub.StubKMeans in place of its estimator (which needs MLX), and keeps its outputs (labeled.csv,
cluster_summary.csv, run.json without paths and timings, model.npz) beside the input. errors.json holds the
reference's error message for each rejected call.
"""
import json
import os
import shutil
import sys
import tempfile

import numpy as np

REF = os.environ.get("REFERENCE_ROOT")
if not REF:
    sys.exit("set REFERENCE_ROOT to the reference checkout (kakollu/mlx-kmeans)")
HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "files")
sys.path.insert(0, HERE)
VOLATILE = ("input", "preparation_s", "fit_including_labels_s")


def tables(rng):
    """(case, file name, text, cluster_file kwargs)"""
    out = []
    n = 300
    a = rng.normal(50, 10, n).round(3)
    b = rng.exponential(3, n).round(4)
    c = rng.integers(0, 9, n)
    ids = [f"id{i:04d}" for i in range(n)]
    lines = ["id,spend,visits,segment,note"]
    for i in range(n):
        spend = "" if i % 37 == 5 else ("n/a" if i % 53 == 7 else f"{a[i]}")
        lines.append(f"{ids[i]},{spend},{b[i]},{c[i]},\"text, {i}\"")
    body = "\n".join(lines) + "\n"
    out.append(("drop_missing", "input.csv", body, dict(columns=["spend", "visits"], k=4, missing="drop")))
    out.append(("raw_units", "input.csv", body.replace(",\"text, ", ",\"t ").replace("n/a", "7.5").replace(",,", ",1,"),
                dict(columns=["spend", "visits", "segment"], k=5, standardize=False)))
    lines = ["cluster\tx\ty\tconst"]
    for i in range(200):
        lines.append(f"c{i}\t{rng.normal():.5f}\t{rng.normal() * 100:.3f}\t2.5")
    out.append(("tsv_collision", "input.tsv", "﻿" + "\n".join(lines) + "\n",
                dict(columns=["x", "y", "const"], k=3)))
    return out


def errors(case_dir):
    """(name, kwargs) of calls the reference rejects, on the drop_missing table."""
    p = os.path.join(case_dir, "input.csv")
    return [
        ("missing_error", dict(path=p, columns=["spend", "visits"], k=4)),
        ("absent_column", dict(path=p, columns=["spend", "nope"], k=4, missing="drop")),
        ("bad_k", dict(path=p, columns=["spend"], k=0)),
        ("bad_tol", dict(path=p, columns=["spend"], k=2, tol=-1.0)),
        ("bad_missing", dict(path=p, columns=["spend"], k=2, missing="zero")),
        ("columns_str", dict(path=p, columns="spend", k=2)),
        ("too_few_rows", dict(path=p, columns=["spend", "visits"], k=5000, missing="drop")),
        ("all_constant", dict(path=os.path.join(OUT, "tsv_collision", "input.tsv"), columns=["const"], k=2)),
        ("not_found", dict(path=os.path.join(case_dir, "absent.csv"), columns=["spend"], k=2)),
        ("bad_suffix", dict(path=os.path.join(HERE, "INDEX.txt"), columns=["spend"], k=2)),
    ]


def main():
    sys.path.insert(0, REF)
    import mlx_kmeans.estimator as est
    import mlx_kmeans.files as files
    from files_stub import StubKMeans
    est.KMeans = StubKMeans
    shutil.rmtree(OUT, ignore_errors=True)
    os.makedirs(OUT)
    rng = np.random.default_rng(20261202)
    for case, name, text, kw in tables(rng):
        d = os.path.join(OUT, case)
        os.makedirs(d)
        with open(os.path.join(d, name), "w", encoding="utf-8", newline="") as f:
            f.write(text)
        with tempfile.TemporaryDirectory() as tmp:
            res = files.cluster_file(os.path.join(d, name), output=os.path.join(tmp, "out"), **kw)
            for fn in ("labeled.csv", "cluster_summary.csv", "model.npz"):
                shutil.copy(os.path.join(tmp, "out", fn), os.path.join(d, fn))
            run = json.load(open(os.path.join(tmp, "out", "run.json")))
        for key in VOLATILE:
            run.pop(key)
        json.dump(dict(kwargs=kw, run=run), open(os.path.join(d, "run.json"), "w"), indent=1)
        print(case, res["run"]["clustered_rows"], "rows clustered")
    msgs = {}
    for name, kw in errors(os.path.join(OUT, "drop_missing")):
        kw = dict(kw)
        path = kw.pop("path")
        try:
            with tempfile.TemporaryDirectory() as tmp:
                files.cluster_file(path, output=os.path.join(tmp, "o"), **kw)
            msgs[name] = None
        except ValueError as e:
            msgs[name] = str(e).replace(os.path.dirname(path), "<dir>")
    json.dump(msgs, open(os.path.join(OUT, "errors.json"), "w"), indent=1)
    print(json.dumps(msgs, indent=1))


if __name__ == "__main__":
    main()
