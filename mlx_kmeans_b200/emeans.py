"""e-means: mini-batch k-means with exponential moving averages (the reference's mlx_kmeans/emeans.py), on this
library's exact batch pass.

The algorithm (the reference's statement of arXiv:2611.09501, emeans.py:1-30): per cluster j a count N_j and a sum
S_j, the centre S_j / N_j. Each epoch permutes the rows and cuts them into batches of B (the remainder dropped);
every batch is assigned to the current centres and each cluster's state moves toward the batch's count and sum by
a step a(t) on a cosine schedule from a0 down to 0.1 a0. After every fifth batch, clusters whose N fell under a
tenth of the mean are revived by splitting a donor drawn in proportion to N. The output is the exact mean of each
cluster over the last epoch's assignments (a cluster empty in the last epoch keeps its moving-average centre).
B and a0 come from the paper's fitted laws unless given.

The laws, the schedule and the seeded draws (permutation, initial rows, revival donors) are the reference's
definitions and give the same numbers (they define the algorithm's output). The fit runs on the GPU: a batch is
gathered on the device, assigned by kmc_pass (every label the float64-nearest centre of the batch's float32
centres, lowest index on ties; counts and sums exact integers), and N, S, C are kept in float64 on the device
(the reference's own float64 reference keeps them in float64 too; its GPU fit in float32). The host reads N
once per revival check (every fifth batch), as the reference does. Like the reference it is APPROXIMATE: its
centres are not a fixed point of Lloyd's iteration, and Lloyd stays the default.
"""
import math
import time

import numpy as np
import torch

from . import _lib, core

# Batch law (paper Eq. 7 as the reference states it, emeans.py:44-45): B = c k^bk n^bn T^bt, /8 above 2M rows.
BATCH_C, BATCH_K, BATCH_N, BATCH_T = 0.035, 0.13, 0.88, 0.81
BATCH_BIG_N, BATCH_BIG_DIV = 2_000_000, 8
# Step law (paper Eq. 6, emeans.py:46-47): a0 = min(c k^ak B^ab n^an T^at, 1).
STEP_C, STEP_K, STEP_B, STEP_N, STEP_T = 0.824, -0.46, 0.90, -0.45, -0.11
COSINE_FLOOR = 0.1
REVIVE_EVERY = 5
REVIVE_TAU = 0.1
SPLIT_DELTA = 2.0 ** -7
INIT_COUNT = 1e-10


def _positive_int(name, v):
    if isinstance(v, bool) or not isinstance(v, (int, np.integer)) or v < 1:
        raise ValueError(f"{name} must be a positive integer, got {v!r}")
    return int(v)


# ---------------------------------------------------------------- laws and schedule (emeans.py:60-105)

def batch_size(n, k, T):
    """The batch law: B_raw = 0.035 k^0.13 n^0.88 T^0.81 (divided by 8 above 2,000,000 rows), rounded to the
    nearest power of two in log2 (half up), at most n."""
    n, k, T = _positive_int("n", n), _positive_int("k", k), _positive_int("T", T)
    raw = BATCH_C * k ** BATCH_K * n ** BATCH_N * T ** BATCH_T
    if n > BATCH_BIG_N:
        raw /= BATCH_BIG_DIV
    e = max(0, int(math.floor(math.log2(raw) + 0.5)))
    return int(min(2 ** e, n))


def step0(n, k, T, B):
    """The peak step at batch size B: min(0.824 k^-0.46 B^0.90 n^-0.45 T^-0.11, 1)."""
    n, k, T, B = (_positive_int(nm, v) for nm, v in (("n", n), ("k", k), ("T", T), ("B", B)))
    return float(min(STEP_C * k ** STEP_K * B ** STEP_B * n ** STEP_N * T ** STEP_T, 1.0))


def schedule(t, M, a0):
    """The step of batch t of M (counted across epochs): cosine from a0 down to COSINE_FLOOR a0."""
    return a0 * (COSINE_FLOOR + (1.0 - COSINE_FLOOR) * 0.5 * (1.0 + math.cos(math.pi * t / M)))


def plan(n, k, epochs, batch_size_=None, step0_=None):
    """-> dict(B, a0, per_epoch, M) for these inputs; explicit B / a0 override the laws."""
    n, k, epochs = _positive_int("n", n), _positive_int("k", k), _positive_int("epochs", epochs)
    if k > n:
        raise ValueError(f"k = {k} cannot exceed the number of rows ({n})")
    if batch_size_ is None:
        B = batch_size(n, k, epochs)
    else:
        B = _positive_int("batch_size", batch_size_)
        if B > n:
            raise ValueError(f"batch_size = {B} is larger than the number of rows ({n})")
    if step0_ is None:
        a0 = step0(n, k, epochs, B)
    else:
        a0 = float(step0_)
        if not 0.0 < a0 <= 1.0:
            raise ValueError(f"step0 must be in (0, 1], got {step0_!r}")
    return dict(B=B, a0=a0, per_epoch=n // B, M=epochs * (n // B))


# ---------------------------------------------------------------- seeded draws (emeans.py:108-169)

def _seed(seed):
    if seed is None:
        return int(np.random.SeedSequence().entropy)        # fresh, and recorded so the run can be repeated
    if isinstance(seed, bool) or not isinstance(seed, (int, np.integer)) or seed < 0:
        raise ValueError(f"seed must be a nonnegative integer or None, got {seed!r}")
    return int(seed)


def _init_rows(seed, n, k):
    """init="random": k distinct rows, centre j from the j-th draw (stream (seed, 1))."""
    return np.random.default_rng([seed, 1]).choice(n, size=k, replace=False)


def _epoch_batches(seed, e, n, B):
    """(n // B, B) row indices of epoch e: stream (seed, 2, e)'s permutation of range(n) (a shuffle of an integer
    range draws the same way whatever its dtype), the remainder dropped, each batch sorted ascending."""
    per = n // B
    order = np.arange(n, dtype=np.uint32 if n <= 2 ** 32 else np.int64)
    np.random.default_rng([seed, 2, e]).shuffle(order)
    cut = order[:per * B].reshape(per, B)
    cut.sort(axis=1)
    return cut


def _split_factors(d):
    """A revived cluster gets its donor's centre times p = (1+delta, 1-delta, ...), the donor keeps it times q."""
    even = np.arange(d) % 2 == 0
    return np.where(even, 1.0 + SPLIT_DELTA, 1.0 - SPLIT_DELTA), np.where(even, 1.0 - SPLIT_DELTA, 1.0 + SPLIT_DELTA)


def _revive_plan(N, seed, t, tau=REVIVE_TAU):
    """(dead, donors) after batch t: dead = clusters with N below tau times the mean; donors drawn from the live
    ones without replacement in proportion to N by Gumbel-top-m keys (stream (seed, 3, t), one uniform per
    cluster); m = min(#dead, #live), the lowest-indexed dead first."""
    N = np.asarray(N, dtype=np.float64)
    u = np.random.default_rng([seed, 3, t]).random(len(N))
    below = N < tau * (N.sum() / len(N))
    dead, live = np.flatnonzero(below), np.flatnonzero(~below)
    m = min(len(dead), len(live))
    if m == 0:
        return np.zeros(0, np.int64), np.zeros(0, np.int64)
    with np.errstate(divide="ignore"):
        keys = np.log(N[live]) - np.log(-np.log(np.maximum(u[live], np.finfo(np.float64).tiny)))
    pick = np.argsort(-keys, kind="stable")[:m]
    return dead[:m].astype(np.int64), live[pick].astype(np.int64)


# ---------------------------------------------------------------- the batch pass on the device

class _Batches:
    """The device side of the batches: one (B, d) buffer the batch rows are gathered into, and a Dataset over it
    that keeps the parent's fixed-point grid (its column maxima and row count), so the integer totals of every
    batch of the last epoch add up exactly."""

    def __init__(self, ds, B):
        self.ds = ds
        self.buf = torch.empty((B, ds.d), dtype=torch.float32, device=ds.device)
        self.bds = core.Dataset([self.buf], label_rule=ds.label_rule)
        self.bds._colmax = ds.colmax
        self.bds.n_total = ds.n_total
        self.offsets = np.concatenate([[0], np.cumsum([p.shape[0] for p in ds.parts])]).astype(np.int64)

    def gather(self, rows):
        """Rows (sorted global indices) into the buffer."""
        B = len(rows)
        at = 0
        for i, p in enumerate(self.ds.parts):
            lo, hi = np.searchsorted(rows, [self.offsets[i], self.offsets[i + 1]])
            if hi > lo:
                idx = torch.from_numpy(np.asarray(rows[lo:hi], np.int64) - self.offsets[i]).to(self.ds.device)
                torch.index_select(p, 0, idx, out=self.buf[at:at + hi - lo])
                at += hi - lo
        assert at == B

    def run(self, C32, approx, labels=False):
        """One batch pass -> the Dataset's buffers (totals, labels)."""
        if self.bds.tensor_cores:                      # the bf16 split of this batch's rows
            (sp, nb), = self.bds.split()
            _lib.call("kmc_split_rows", self.buf.data_ptr(), self.buf.shape[0], self.ds.d, sp.data_ptr(), nb,
                      torch.cuda.current_stream().cuda_stream)
        return self.bds.run_pass(C32, labels=labels, approx=approx)

    def unpack(self, totals, k):
        """(sums float64 (k, d), counts float64 (k), inertia (1,)) on the device, from integer totals."""
        b = self.bds.buffers(k)
        sums = torch.empty((k, self.ds.d), dtype=torch.float64, device=self.ds.device)
        counts = torch.empty(k, dtype=torch.int64, device=self.ds.device)
        inertia = torch.empty(1, dtype=torch.float64, device=self.ds.device)
        _lib.call("kmc_totals_unpack", totals.data_ptr(), k, self.ds.d, sums.data_ptr(), counts.data_ptr(),
                  inertia.data_ptr(), b["ws"].data_ptr(), b["wsb"], torch.cuda.current_stream().cuda_stream)
        return sums, counts.double(), inertia


def emeans_fit(parts, k, epochs=3, seed=0, batch_size=None, step0=None, init="random", assign="exact",
               method="auto", accumulate="auto", trace=None, verbose=False):
    """e-means on the GPU -> (centres float32 (k, d), record) (emeans.py:558-616).

    parts: a Dataset, CUDA tensors, or NumPy arrays (copied to the device once). init: "random" (k distinct rows),
    "k-means++" (kmeans_pp_init with the generator of stream (seed, 1)) or a (k, d) array. assign: "exact" or
    "approx" (exact=False's tensor-core pass where it applies, as for Lloyd). method / accumulate: accepted for
    the reference's signature ("auto" and its names); this library has one exact batch pass and one exact
    accumulation. trace: a list that gets one dict of host copies per batch (a host read every batch).
    The record: n, d, k, epochs, B, a0, M, batches_per_epoch, dropped_per_epoch, seed, init, assign, revived (per
    check), train_mse (per epoch: mean float32 distance of the epoch's batch rows to the centre each was assigned
    to), last_epoch_counts, last_epoch_empty, timings.
    """
    t_start = time.perf_counter()
    ds = core._dataset(parts)
    n, d = ds.n_total, ds.d
    k = _positive_int("k", k)
    seed = _seed(seed)
    P = plan(n, k, epochs, batch_size, step0)
    B, a0, per, M = P["B"], P["a0"], P["per_epoch"], P["M"]
    if assign not in ("exact", "approx"):
        raise ValueError(f"assign must be 'exact' or 'approx', got {assign!r}")
    if method not in ("auto", "rows", "pairs", "tiles", "tiles1", "onehot"):
        raise ValueError(f"method must be auto, rows, pairs, tiles, tiles1 or onehot, got {method!r}")
    if accumulate not in ("auto", "lanes", "blocks", "segments"):
        raise ValueError(f"accumulate must be auto, lanes, blocks or segments, got {accumulate!r}")
    if isinstance(init, str):
        if init == "random":
            C0 = core.take_rows(ds, _init_rows(seed, n, k))
        elif init == "k-means++":
            C0 = core.kmeans_pp_init(ds, n, k, np.random.default_rng([seed, 1]))
        else:
            raise ValueError(f"init must be 'random', 'k-means++' or a (k, d) array, got {init!r}")
    else:
        C0 = np.array(init, dtype=np.float32)
        if C0.shape != (k, d):
            raise ValueError(f"init centres must have shape {(k, d)}, got {C0.shape}")
    C0 = np.ascontiguousarray(C0, dtype=np.float32)
    t_init = time.perf_counter()

    dev = ds.device
    bat = _Batches(ds, B)
    approx = assign == "approx" and bat.bds.uses_approx(True)
    pn, qn = _split_factors(d)
    p_d, q_d = torch.from_numpy(pn).to(dev), torch.from_numpy(qn).to(dev)
    C = torch.from_numpy(C0).to(dev).double()
    N = torch.full((k,), INIT_COUNT, dtype=torch.float64, device=dev)
    S = C * INIT_COUNT
    last_tot = torch.zeros((k, d + 2), dtype=torch.int64, device=dev)
    batch_inertia = []
    revived = []
    t = 0
    for e in range(epochs):
        batches = _epoch_batches(seed, e, n, B)
        last = e == epochs - 1
        for i in range(per):
            rows = batches[i]
            bat.gather(rows)
            C32 = C.float()
            b = bat.run(C32, approx, labels=trace is not None)
            sums, cnt, inert = bat.unpack(b["totals"], k)
            a = schedule(t, M, a0)
            N = (1.0 - a) * N + a * cnt
            S = (1.0 - a) * S + a * sums
            has = N > 0
            C = torch.where(has[:, None], S / torch.where(has, N, torch.ones_like(N))[:, None], C)
            batch_inertia.append(inert)
            if last:
                last_tot += b["totals"]
            dead = donors = Nh = None
            if (t + 1) % REVIVE_EVERY == 0:
                Nh = N.cpu().numpy()                   # the counts the decision is made from (one host read)
                dead, donors = _revive_plan(Nh, seed, t)
                revived.append(len(dead))
                if len(dead):
                    di = torch.from_numpy(dead).to(dev)
                    oi = torch.from_numpy(donors).to(dev)
                    cd = C[oi]
                    half = N[oi] * 0.5
                    N[di] = half
                    N[oi] = half
                    S[di] = (cd * p_d) * half[:, None]
                    S[oi] = (cd * q_d) * half[:, None]
                    has = N > 0
                    C = torch.where(has[:, None], S / torch.where(has, N, torch.ones_like(N))[:, None], C)
            if trace is not None:
                trace.append(dict(t=t, epoch=e, rows=np.asarray(rows, np.int64), a=a,
                                  labels=b["labels"][0].cpu().numpy().astype(np.int64), C_before=C32.cpu().numpy(),
                                  counts=cnt.cpu().numpy(), sums=sums.cpu().numpy(), N=N.cpu().numpy(),
                                  C=C.cpu().numpy(), N_check=Nh, dead=dead, donors=donors))
            t += 1
    t_train = time.perf_counter()
    sums, cnt, _ = bat.unpack(last_tot, k)
    out = C.clone()
    used = cnt > 0                                     # a cluster empty in the last epoch keeps its EMA centre
    out[used] = sums[used] / cnt[used][:, None]
    out = out.float().cpu().numpy()
    inert = torch.cat(batch_inertia).cpu().numpy() if batch_inertia else np.zeros(0)
    train_mse = [float(inert[e * per:(e + 1) * per].sum() / (per * B)) for e in range(epochs)]
    cnt_h = cnt.cpu().numpy()
    t_end = time.perf_counter()
    rec = dict(n=n, d=d, k=k, epochs=epochs, B=B, a0=a0, batches_per_epoch=per, M=M, dropped_per_epoch=n - per * B,
               seed=seed, init=init if isinstance(init, str) else "given", assign="approx" if approx else "exact",
               method="exact batch pass" if not approx else "approx", revived=revived, train_mse=train_mse,
               last_epoch_counts=cnt_h, last_epoch_empty=int((cnt_h == 0).sum()),
               init_centres=C0 if trace is not None else None,
               timings=dict(init_s=t_init - t_start, train_s=t_train - t_init, finish_s=t_end - t_train,
                            total_s=t_end - t_start))
    if verbose:
        print(f"e-means: B={B} a0={a0:.4f} M={M} ({per} batches x {epochs} epochs, {n - per * B} rows dropped per "
              f"epoch); train MSE by epoch " + ", ".join(f"{v:.6e}" for v in train_mse) +
              f"; revived {sum(revived)} in {len(revived)} checks")
    return out, rec
