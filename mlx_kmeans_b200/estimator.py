"""scikit-learn-shaped KMeans on the B200 Lloyd path (the reference's mlx_kmeans/estimator.py API).

    KMeans(n_clusters=64).fit(X).cluster_centers_

Same constructor, attributes and errors as the reference (estimator.py:52-65, 180-230): n_clusters, n_init,
max_iter, tol (relative inertia change), random_state, verbose, spherical, accumulate, exact, and the e-means
options (algorithm="emeans", epochs, batch_size: mlx_kmeans_b200.emeans), plus label_rule. The Lloyd loop keeps
its centers on the device and, on one GPU with the CUDA-core pass, runs whole on the device (kmc_lloyd: the tol test
in the finish kernel, one host read at the end); elsewhere each step reads back one 64-byte statistics record.
"""
import numpy as np
import torch

from . import core


class KMeans:
    """Exact k-means on B200 GPUs: every label is the float64-nearest center, lowest index on ties.

    label_rule="float64" (default) labels every row with its float64-nearest center; "float32" reproduces the
    reference's exact-mode kernels bit for bit (their float32 direct sum, strict < in index order, core.py:263-274).
    The two differ only on rows whose float32 sums to two centers are within their rounding of each other.

    exact=False takes the approximate kernel from 64 dims up on the tensor-core path (x.c from one bf16 product,
    the smallest score's center without an error window: the reference's approximate assignment, core.py:859-1088);
    below that it runs exactly, as the reference does below its crossover. Counts, sums and inertia are exact for
    the labels it gives. accumulate="atomic" also runs the
    deterministic accumulation: totals here are exact integers, so there is no faster non-deterministic mode to
    opt into.
    """

    def __init__(self, n_clusters=8, n_init=1, max_iter=300, tol=1e-4, random_state=None, verbose=False,
                 spherical=False, accumulate="auto", exact=True, algorithm="lloyd", epochs=3, batch_size=None,
                 label_rule="float64"):
        self.n_clusters = n_clusters
        self.n_init = n_init
        self.max_iter = max_iter
        self.tol = tol
        self.random_state = random_state
        self.verbose = verbose
        self.spherical = spherical
        self.accumulate = accumulate
        self.exact = exact
        self.algorithm = algorithm
        self.epochs = epochs
        self.batch_size = batch_size
        self.label_rule = label_rule

    @property
    def _method(self):
        return "auto" if self.exact else "approx"

    @classmethod
    def from_centers(cls, centers, **kwargs):
        """A fitted model from centers saved earlier (estimator.py:71-79)."""
        centers = np.ascontiguousarray(centers, dtype=np.float32)
        if not np.isfinite(centers).all():
            raise ValueError("centers contain NaN or infinity")
        model = cls(n_clusters=len(centers), **kwargs)
        model.cluster_centers_ = centers
        return model

    @staticmethod
    def _explain_nonfinite(ds):
        """Say why a pass came back non-finite, then raise (estimator.py:81-106)."""
        peak = ds.absmax()
        if not np.isfinite(peak):
            raise ValueError(
                "input contains NaN or infinity, which would produce nan centers rather than an error. "
                "Drop or impute those rows first (the file workflow's missing='drop' does this).")
        limit = float(np.sqrt(np.finfo(np.float32).max / (4.0 * ds.d)))
        if peak > limit:
            raise ValueError(
                f"largest coordinate is {peak:.3e}, above the {limit:.3e} this many dimensions allow: "
                f"a squared distance would overflow float32 and return nan. Standardise the features "
                f"(see the README) or rescale before fitting.")
        raise ValueError("clustering produced a non-finite result, but the input values look usable; "
                         "please report this with the data shape and dtype.")

    @staticmethod
    def _parts(X):
        """-> a core.Dataset (device-resident rows), from NumPy, pandas, lists, CUDA tensors or a Dataset."""
        if isinstance(X, core.Dataset):
            return X
        if isinstance(X, list) and X and isinstance(X[0], torch.Tensor):
            return core.Dataset(X)
        if isinstance(X, torch.Tensor):
            if X.ndim != 2 or not all(X.shape):
                raise ValueError(f"expected a nonempty 2-D (rows, dims) array, got shape {tuple(X.shape)}")
            return core.Dataset([X])
        if not isinstance(X, np.ndarray):
            X = np.asarray(X.to_numpy() if hasattr(X, "to_numpy") else X)
        X = np.ascontiguousarray(X, dtype=np.float32)
        if X.ndim != 2 or not all(X.shape):
            raise ValueError(f"expected a nonempty 2-D (rows, dims) array, got shape {X.shape}")
        return core.Dataset([X])

    @staticmethod
    def _normalise(C):
        n = torch.linalg.vector_norm(C.double(), dim=1, keepdim=True)
        return (C.double() / torch.where(n > 0, n, torch.ones_like(n))).float()

    def _one_run(self, ds, rows, seed):
        """estimator.py:132-150 with the centers kept on the device between steps."""
        rng = np.random.default_rng(seed)
        C = torch.from_numpy(core.kmeans_pp_init(ds, rows, self.n_clusters, rng)).to(ds.device)
        ds.reset_bounds()                  # a restart: the previous run's per-row bounds say nothing useful
        if self.spherical:
            C = self._normalise(C)
        generic = self._method == "generic"
        approx = self._method == "approx"
        if not self.spherical and not self.verbose and ds.device_loop_ok(generic) and \
                not ds.uses_approx(approx):
            # the whole loop on the device: one host read at the end (estimator.py:132-150's stopping rule)
            C, inertia, iters, flags = ds.lloyd_loop(C, self.max_iter, self.tol, generic=generic,
                                                     rule=self.label_rule)
            if flags & 1 or not np.isfinite(inertia):
                self._explain_nonfinite(ds)
            return C.clone(), inertia, iters
        prev = None
        inertia = float("nan")
        it = 0
        for it in range(self.max_iter):
            C_new, s = ds.step(C, generic=generic, rule=self.label_rule, approx=approx)
            C = C_new.clone()
            inertia = s["inertia"]
            if s["flags"] & 1 or not np.isfinite(inertia):
                self._explain_nonfinite(ds)
            if self.spherical:
                C = self._normalise(C)
            if self.verbose:
                n_empty = s["n_empty"]
                print(f"iter {it + 1}: inertia {inertia:.6e}" + (f", {n_empty} empty relocated" if n_empty else ""))
            if prev is not None and abs(prev - inertia) <= self.tol * prev:
                break
            prev = inertia
        return C, inertia, it + 1

    # e-means keeps its own exact accumulation; the reference's accumulator names map onto it
    _EMEANS_ACCUMULATE = {"auto": "auto", "lanes": "lanes", "blocks": "blocks", "sorted": "segments"}

    def _check_algorithm(self):
        """algorithm="lloyd" (default) or "emeans" with its options (estimator.py:155-170)."""
        algorithm = getattr(self, "algorithm", "lloyd")
        if algorithm not in ("lloyd", "emeans"):
            raise ValueError(f"algorithm must be 'lloyd' or 'emeans', got {algorithm!r}")
        if algorithm != "emeans":
            return
        if isinstance(self.epochs, bool) or not isinstance(self.epochs, (int, np.integer)) or self.epochs < 1:
            raise ValueError("epochs must be a positive integer")
        if self.batch_size is not None and (isinstance(self.batch_size, bool) or
                                            not isinstance(self.batch_size, (int, np.integer)) or self.batch_size < 1):
            raise ValueError("batch_size must be None or a positive integer")
        if self.spherical:
            raise ValueError("spherical=True is not offered with algorithm='emeans'")
        if self.accumulate not in self._EMEANS_ACCUMULATE:
            raise ValueError(f"accumulate={self.accumulate!r} is not offered with algorithm='emeans' "
                             f"(use one of {sorted(self._EMEANS_ACCUMULATE)})")

    def _one_run_emeans(self, ds, rows, seed):
        from . import emeans
        if self.batch_size is not None and self.batch_size > rows:
            raise ValueError(f"batch_size ({self.batch_size}) cannot exceed the number of rows ({rows})")
        C, record = emeans.emeans_fit(ds, self.n_clusters, epochs=self.epochs, seed=seed, batch_size=self.batch_size,
                                      assign="exact" if self.exact else "approx",
                                      accumulate=self._EMEANS_ACCUMULATE[self.accumulate], verbose=self.verbose)
        return torch.from_numpy(C).to(ds.device), record

    def fit(self, X, y=None):
        for name in ['n_clusters', 'n_init', 'max_iter']:
            value = getattr(self, name)
            if isinstance(value, bool) or not isinstance(value, (int, np.integer)) or value < 1:
                raise ValueError(f'{name} must be a positive integer')
        if not np.isfinite(self.tol) or self.tol < 0:
            raise ValueError('tol must be finite and nonnegative')
        self._check_algorithm()
        if self.accumulate not in core.ACCUMULATE_METHODS:
            raise ValueError(f"unknown accumulate {self.accumulate!r}")
        core._check_rule(self.label_rule)
        ds = self._parts(X)
        rows = ds.n_total
        if rows < self.n_clusters:
            raise ValueError('n_clusters cannot exceed the number of rows')
        emeans = getattr(self, "algorithm", "lloyd") == "emeans"
        best = None
        for run in range(self.n_init):                  # every start runs on the same device-resident Dataset
            seed = None if self.random_state is None else self.random_state + run
            record = None
            if emeans:
                C, record = self._one_run_emeans(ds, rows, seed)
                iters = self.epochs
            else:
                C, inertia, iters = self._one_run(ds, rows, seed)
            # the last step's inertia belongs to the centers it started from; one more pass scores the returned ones
            # (estimator.py:201-204)
            _, _, inertia, labels = ds.assign(C, return_labels=True, rule=self.label_rule,
                                              approx=self._method == "approx")
            if emeans and not np.isfinite(inertia):
                self._explain_nonfinite(ds)
            if self.verbose and self.n_init > 1:
                print(f"start {run + 1}/{self.n_init}: inertia {inertia:.6e} after {iters} "
                      f"{'epochs' if emeans else 'iterations'}")
            if best is None or inertia < best[1]:
                best = (C.cpu().numpy(), inertia, iters, labels, record)
        self.cluster_centers_, self.inertia_, self.n_iter_, self.labels_ = best[:4]
        if emeans:
            self.emeans_record_ = best[4]
        return self

    def predict(self, X):
        """Cluster index for every row of X (any array-like)."""
        ds = self._parts(X)
        if ds.d != self.cluster_centers_.shape[1]:
            raise ValueError(f"X has {ds.d} features but this model was fitted with "
                             f"{self.cluster_centers_.shape[1]}")
        C = torch.from_numpy(np.ascontiguousarray(self.cluster_centers_, dtype=np.float32)).to(ds.device)
        _, _, inertia, labels = ds.assign(C, return_labels=True, rule=self.label_rule,
                                          approx=self._method == "approx")
        if not np.isfinite(inertia):
            self._explain_nonfinite(ds)
        return labels

    def fit_predict(self, X, y=None):
        return self.fit(X).labels_
