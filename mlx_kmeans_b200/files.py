"""Clustering a local CSV / TSV / XLSX file: the step before the Lloyd path (the reference's mlx_kmeans/files.py).

    cluster_file("customers.csv", columns=["spend", "visits"], k=5)

Same entry points, arguments, outputs and error messages as the reference (files.py:9-180):
  batches(path, sheet)    the table as 10,000-row string DataFrames (.csv / .tsv as UTF-8 with an optional BOM,
                          .xlsx through openpyxl when it is installed); the header must be unique and nonempty
  inspect_file(path)      its first five rows
  read_table(path)        the whole table, refused when it would not fit a conservative share of the host's RAM
  cluster_file(...)       numeric feature columns -> (optional) standardisation with the float64 mean and the
                          population standard deviation -> KMeans on the GPU -> a new folder holding
                          labeled.csv (every input row, 1-based cluster ids, blank for excluded rows),
                          cluster_summary.csv, run.json and model.npz; nothing existing is overwritten.
Missing / non-numeric / non-finite selected values are an error by default; missing="drop" keeps those rows in
the export with a blank label. The fit reuses the device copy of the rows for every restart (n_init).
"""
import csv
import datetime
import json
import time
from pathlib import Path

CHUNK_ROWS = 10_000
MEMORY_SHARE = 0.35          # of installed RAM that a table may take (read_table's estimate)
AVAILABLE_SHARE = 0.7        # of currently available RAM


def dependencies():
    """pandas and psutil, or the reference's install hint."""
    try:
        import pandas as pd
        import psutil
    except ImportError as e:
        raise ValueError('Install file support: python -m pip install ".[files]"') from e
    return pd, psutil


def check_header(header):
    names = [str(h) for h in header]
    if not names or any(not n.strip() for n in names) or len(set(names)) != len(names):
        raise ValueError('The first row must have unique, nonempty column names.')


def _delimited(path, sep):
    pd, _ = dependencies()
    with path.open(encoding='utf-8-sig', newline='') as f:
        check_header(next(csv.reader(f, delimiter=sep), []))
    with pd.read_csv(path, sep=sep, dtype=str, keep_default_na=False, encoding='utf-8-sig',
                     chunksize=CHUNK_ROWS) as chunks:
        for chunk in chunks:
            yield chunk


def _workbook(path, sheet):
    pd, _ = dependencies()
    try:
        from openpyxl import load_workbook
    except ImportError as e:
        raise ValueError('XLSX support needs openpyxl: install ".[files]"') from e
    book = load_workbook(path, read_only=True, data_only=True)
    try:
        if sheet is not None and sheet not in book.sheetnames:
            raise ValueError(f'Sheet {sheet!r} not found. Available: {", ".join(book.sheetnames)}')
        ws = book[sheet] if sheet else book.worksheets[0]
        cells = ws.iter_rows(values_only=True)
        header = ['' if v is None else str(v) for v in next(cells, ())]
        check_header(header)
        pending = []
        for row in cells:
            pending.append(['' if v is None else str(v) for v in row])
            if len(pending) == CHUNK_ROWS:
                yield pd.DataFrame(pending, columns=header)
                pending = []
        if pending:
            yield pd.DataFrame(pending, columns=header)
    finally:
        book.close()


def batches(path, sheet=None):
    """The table at `path` as DataFrames of at most 10,000 rows of strings."""
    path = Path(path).expanduser()
    if not path.is_file():
        raise ValueError(f'Local file not found: {path}')
    ext = path.suffix.lower()
    if ext in ('.csv', '.tsv'):
        yield from _delimited(path, '\t' if ext == '.tsv' else ',')
    elif ext == '.xlsx':
        yield from _workbook(path, sheet)
    else:
        raise ValueError('Use a .csv, .tsv, or .xlsx file. Export older Excel files as CSV or XLSX.')


def inspect_file(path, sheet=None):
    """The first five data rows (for choosing the feature columns)."""
    it = batches(path, sheet)
    try:
        first = next(it, None)
    finally:
        it.close()
    if first is None:
        raise ValueError('The file has no data rows.')
    return first.head(5)


def read_table(path, sheet=None):
    """The whole table, chunk by chunk, refused once its estimated footprint passes the budget: MEMORY_SHARE of
    the installed RAM, or AVAILABLE_SHARE of what is available now."""
    pd, psutil = dependencies()
    budget = int(psutil.virtual_memory().total * MEMORY_SHARE)
    parts, nbytes, nrows = [], 0, 0
    for chunk in batches(path, sheet):
        nbytes += int(chunk.memory_usage(index=True, deep=True).sum())
        nrows += len(chunk)
        estimate = 256 * 2 ** 20 + 4 * nbytes + 32 * nrows * len(chunk.columns)
        if estimate > budget or estimate > AVAILABLE_SHARE * psutil.virtual_memory().available:
            raise ValueError('This file exceeds the conservative in-memory budget. Nothing was sampled. '
                             'Close heavy apps or export a smaller file/fewer columns and retry.')
        parts.append(chunk)
    if not parts:
        raise ValueError('The file has no data rows.')
    return pd.concat(parts, ignore_index=True)


def _check_args(columns, k, n_init, max_iter, tol, missing):
    import numpy as np
    for name, value in (('k', k), ('n_init', n_init), ('max_iter', max_iter)):
        if isinstance(value, bool) or not isinstance(value, (int, np.integer)) or value < 1:
            raise ValueError(f'{name} must be a positive integer')
    if not np.isfinite(tol) or tol < 0:
        raise ValueError('tol must be finite and nonnegative')
    if missing not in ('error', 'drop'):
        raise ValueError('missing must be error or drop')
    if isinstance(columns, str) or not columns or len(set(columns)) != len(columns):
        raise ValueError('Pass a list of unique feature column names, e.g. columns=["spend", "visits"].')


def _features(frame, columns, k, missing, standardize):
    """-> (X float32 rows to cluster, kept float64 values, valid row mask, center, scale, constant columns)."""
    import numpy as np
    pd, _ = dependencies()
    absent = [c for c in columns if c not in frame.columns]
    if absent:
        raise ValueError(f'Columns not found: {absent}. Available: {list(frame.columns)}')
    values = frame[list(columns)].apply(pd.to_numeric, errors='coerce').to_numpy(dtype=np.float64)
    finite = np.isfinite(values)
    valid = finite.all(axis=1)
    excluded = int((~valid).sum())
    if excluded and missing == 'error':
        per_column = {c: int((~finite[:, i]).sum()) for i, c in enumerate(columns) if not finite[:, i].all()}
        raise ValueError(f'{excluded} rows have missing/non-numeric/nonfinite selected values: {per_column}. '
                         'Clean the file or explicitly choose --missing drop / missing="drop".')
    kept = values[valid]
    if len(kept) < k:
        raise ValueError(f'Only {len(kept)} usable rows for k={k}.')
    mean, std = kept.mean(axis=0), kept.std(axis=0)
    constant = [c for c, s in zip(columns, std) if s == 0]
    if len(constant) == len(columns):
        raise ValueError('All selected features are constant; they cannot separate rows into clusters.')
    if standardize:
        center, scale = mean, np.where(std > 0, std, 1.0)
    else:
        center, scale = np.zeros(len(columns)), np.ones(len(columns))
    with np.errstate(over='ignore', invalid='ignore'):
        X = np.ascontiguousarray((kept - center) / scale, dtype=np.float32)
    if not np.isfinite(X).all():
        raise ValueError('Feature values exceed float32 range; rescale the data before clustering.')
    return X, kept, valid, excluded, center, scale, constant


def _summary(kept, labels, columns, k):
    """Per cluster (1..k): rows, share of the clustered rows, and the mean of every feature in original units."""
    import numpy as np
    pd, _ = dependencies()
    table = pd.DataFrame(kept, columns=columns).groupby(labels).mean()
    table.index.name = 'cluster'
    table = table.rename(columns={c: 'mean_' + c for c in columns}).reindex(range(1, k + 1))
    counts = np.bincount(labels, minlength=k + 1)[1:]
    table.insert(0, 'rows', counts)
    table.insert(1, 'share', counts / len(kept))
    return table.reset_index()


def cluster_file(path, *, columns, k, output=None, n_init=10, max_iter=300, tol=1e-4, seed=0, standardize=True,
                 missing='error', sheet=None):
    """Cluster the selected numeric columns of a local file and write the results to a new folder.

    Returns dict(output=folder, summary=DataFrame, run=metadata). Labels in the export are 1-based group ids
    (arbitrary, not ranked); rows excluded by missing="drop" get a blank label.
    """
    import numpy as np
    from .estimator import KMeans
    pd, _ = dependencies()
    _check_args(columns, k, n_init, max_iter, tol, missing)
    path = Path(path).expanduser().resolve()
    if output:
        destination = Path(output).expanduser()
    else:
        stamp = datetime.datetime.now().strftime('%Y%m%d-%H%M%S-%f')
        destination = path.with_name(f'{path.stem}-clusters-{stamp}')
    if destination.exists():
        raise ValueError(f'Output already exists: {destination}. Choose a new folder; nothing overwritten.')
    t0 = time.perf_counter()
    frame = read_table(path, sheet)
    X, kept, valid, excluded, center, scale, constant = _features(frame, columns, k, missing, standardize)
    prepare_s = time.perf_counter() - t0
    t1 = time.perf_counter()
    model = KMeans(n_clusters=k, n_init=n_init, max_iter=max_iter, tol=tol, random_state=seed).fit(X)
    fit_s = time.perf_counter() - t1
    labels = np.asarray(model.labels_) + 1
    summary = _summary(kept, labels, list(columns), k)
    label_name = 'cluster'
    while label_name in frame.columns:
        label_name = 'kmeans_' + label_name
    exported = pd.Series(pd.NA, index=frame.index, dtype='Int64')
    exported.loc[valid] = labels
    frame[label_name] = exported
    run = dict(input=str(path), columns=list(columns), sheet=sheet, k=k, n_init=n_init, max_iter=max_iter, tol=tol,
               tol_definition='relative inertia change (not R or sklearn center-shift tolerance)', seed=seed,
               standardize=standardize, scale_ddof=0, missing=missing, input_rows=len(frame),
               clustered_rows=len(kept), excluded_rows=excluded, label_column=label_name,
               labels='1-based, arbitrary group IDs, not ranked', constant_features=constant,
               inertia=model.inertia_, iterations=model.n_iter_, preparation_s=prepare_s,
               fit_including_labels_s=fit_s, feature_mean=center.tolist(), feature_scale=scale.tolist())
    # the folder is made only once everything above succeeded; an existing one is never reused
    destination.mkdir(parents=True, exist_ok=False)
    frame.to_csv(destination / 'labeled.csv', index=False)
    summary.to_csv(destination / 'cluster_summary.csv', index=False)
    (destination / 'run.json').write_text(json.dumps(run, indent=2))
    np.savez(destination / 'model.npz', centers=model.cluster_centers_, mean=center, scale=scale,
             columns=np.array(columns))
    return dict(output=destination.resolve(), summary=summary, run=run)
