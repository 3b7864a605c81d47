"""Multi-rank host logic of the package on CPU ranks (gloo, world size 2, no GPU).

The ranks run the package's own multi-rank code on CPU tensors: Dataset(group=...)'s shard plan
(core.shard_plan), the MAX all-reduce of the column maxima (core.allreduce_colmax), Dataset.allreduce_totals
(the exact int64 SUM all-reduce of the fixed-point totals; the peer-memory exchange is switched off with
KMC_EXCHANGE=nccl, so the CUDA buffers are never opened) and the relocation candidates' gather
(core.gather_candidates). Their results are checked against the one-process values: shards contiguous and
covering, totals bit-identical, and the gathered candidate lists -- merged by the relocation rule of
core.py:2227-2229 -- equal to the global far-row order.
"""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

WORLD = 2
E = 5


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _quantised_totals(X, labels, best, k, shift_x, shift_i):
    """Totals in the library's format: [count, sum q(best), sum q(x_j)] with q(v) = rint(v * 2^shift)."""
    n, d = X.shape
    tot = np.zeros((k, d + 2), np.int64)
    np.add.at(tot[:, 0], labels, 1)
    np.add.at(tot[:, 1], labels, np.rint(np.ldexp(best.astype(np.float64), shift_i)).astype(np.int64))
    for j in range(d):
        np.add.at(tot[:, 2 + j], labels, np.rint(np.ldexp(X[:, j].astype(np.float64), shift_x[j])).astype(np.int64))
    return tot


def _case():
    rng = np.random.default_rng(3)
    X = (rng.standard_normal((5000, 3)) * [1, 10, 100]).astype(np.float32)
    C = X[:7].copy()
    from oracle import oracle as O
    labels, _, best = O.assign(X, C)
    return X, C, labels, best


def _shifts(gmax, n):
    L = int(np.ceil(np.log2(n)))
    return [61 - L - int(np.ceil(np.log2(float(m)))) for m in gmax], 40


def _records(X, labels, best, rows):
    """kmc_far_rows' record layout: [best, global row lo, global row hi, label, x_0 .. x_{d-1}] as 32-bit words."""
    d = X.shape[1]
    out = np.zeros((len(rows), d + 4), np.uint32)
    for r, i in enumerate(rows):
        out[r, 0] = np.float32(best[i]).view(np.uint32)
        out[r, 1], out[r, 2], out[r, 3] = i & 0xFFFFFFFF, i >> 32, labels[i]
        out[r, 4:] = X[i].view(np.uint32)
    return out.view(np.int32)


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD),
                      KMC_EXCHANGE="nccl")
    import sys
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from mlx_kmeans_b200 import core
        from mlx_kmeans_b200.data import shard_range
        X, C, labels, best = _case()
        n, d = X.shape
        k = len(C)
        lo, hi = shard_range(n, rank, WORLD, align=512)
        # the package's shard plan, from this rank's rows
        ds = core.Dataset([torch.from_numpy(X[lo:hi])], group=dist.group.WORLD, device="cpu")
        plan = (ds.rank, ds.world, ds.row0, ds.n_total, lo)
        # column grids from the GLOBAL maxima
        cm = torch.from_numpy(np.abs(X[lo:hi]).max(0).astype(np.float32).view(np.int32).copy())
        core.allreduce_colmax(cm, dist.group.WORLD)
        gmax = cm.numpy().view(np.float32)
        shift_x, shift_i = _shifts(gmax, n)
        # the exact totals: this rank's int64 sums through Dataset.allreduce_totals
        b = {"totals": torch.from_numpy(_quantised_totals(X[lo:hi], labels[lo:hi], best[lo:hi], k, shift_x,
                                                           shift_i))}
        ds.allreduce_totals(b, k)
        # relocation candidates: this rank's top E (what kmc_far_rows returns), gathered in rank order
        mine = sorted(range(lo, hi), key=lambda i: (-best[i], i))[:E]
        local = torch.from_numpy(_records(X, labels, best, mine))
        gathered = core.gather_candidates(local, dist.group.WORLD, WORLD)
        if rank == 0:
            out.put((plan, gmax.tolist(), b["totals"].numpy().tolist(), gathered.numpy().tolist(),
                     ds._xch.get(k)))
        else:
            out.put(("plan", plan))
    finally:
        dist.destroy_process_group()


def _merge(gathered, ranks):
    """The relocation merge of the concatenated lists (farthest first, lower global row on ties), as k_finish
    takes them: one sorted list of E records per rank."""
    recs = np.asarray(gathered, np.int32).view(np.uint32).reshape(ranks, E, -1)
    heads = [0] * ranks
    order = []
    for _ in range(E):
        pick = None
        for r in range(ranks):
            if heads[r] >= E:
                continue
            rec = recs[r, heads[r]]
            b = float(rec[0:1].view(np.float32)[0])
            g = int(rec[1]) | (int(rec[2]) << 32)
            if pick is None or b > pick[1] or (b == pick[1] and g < pick[2]):
                pick = (r, b, g)
        heads[pick[0]] += 1
        order.append(pick[2])
    return order


def test_two_cpu_ranks_reproduce_the_single_process_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(WORLD)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    other = next(r[1] for r in res if r[0] == "plan")
    plan0, gmax, tot, gathered, xch = next(r for r in res if r[0] != "plan")
    X, C, labels, best = _case()
    n = len(X)
    # shard plan: rank 0 first, rows contiguous, covering, on the block grid
    assert plan0[:4] == (0, WORLD, 0, n) and other[:4] == (1, WORLD, other[4], n)
    assert other[2] == other[4] and other[2] % 512 == 0 and 0 < other[2] < n
    # global maxima and all-reduced integer totals equal the one-process values bit for bit
    assert np.array_equal(np.float32(gmax), np.abs(X).max(0))
    shift_x, shift_i = _shifts(np.abs(X).max(0), n)
    assert np.array_equal(np.array(tot, np.int64), _quantised_totals(X, labels, best, len(C), shift_x, shift_i))
    assert xch is False                       # the NCCL-style all-reduce ran, not the peer-memory exchange
    # the gathered lists, merged by the relocation rule, give the global far-row order
    assert _merge(gathered, WORLD) == sorted(range(n), key=lambda i: (-best[i], i))[:E]
