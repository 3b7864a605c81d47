"""Multi-rank host logic on CPU ranks (gloo, world size 2): shard plan, exact all-reduce of the fixed-point
totals, and the far-row candidate merge used by relocation. No GPU."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import ROOT

WORLD = 2


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


def _worker(rank, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(WORLD))
    import sys
    sys.path.insert(0, ROOT)
    dist.init_process_group("gloo", rank=rank, world_size=WORLD)
    try:
        from mlx_kmeans_b200.data import shard_range
        X, C, labels, best = _case()
        n, d = X.shape
        k = len(C)
        # the shard plan covers every row once, on the block grid
        lo, hi = shard_range(n, rank, WORLD, align=512)
        cover = torch.tensor([lo, hi], dtype=torch.int64)
        allc = [torch.zeros_like(cover) for _ in range(WORLD)]
        dist.all_gather(allc, cover)
        # column grids from the GLOBAL maxima (MAX all-reduce of the local ones)
        cm = torch.from_numpy(np.abs(X[lo:hi]).max(0).astype(np.float32).view(np.int32).copy())
        dist.all_reduce(cm, op=dist.ReduceOp.MAX)
        gmax = cm.numpy().view(np.float32)
        L = int(np.ceil(np.log2(n)))
        shift_x = [61 - L - int(np.ceil(np.log2(float(m)))) for m in gmax]
        shift_i = 40
        # exact totals: local int64 sums, SUM all-reduce
        t = torch.from_numpy(_quantised_totals(X[lo:hi], labels[lo:hi], best[lo:hi], k, shift_x, shift_i))
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        # relocation candidates: local top-E by (best desc, global row asc), all-gathered, merged the same way
        E = 5
        order = sorted(range(lo, hi), key=lambda i: (-best[i], i))[:E]
        cand = torch.tensor([[float(best[i]), i] for i in order], dtype=torch.float64)
        gathered = [torch.zeros_like(cand) for _ in range(WORLD)]
        dist.all_gather(gathered, cand)
        merged = sorted([tuple(r) for g in gathered for r in g.tolist()], key=lambda r: (-r[0], r[1]))[:E]
        if rank == 0:
            out.put(([c.tolist() for c in allc], t.numpy().tolist(), [int(r[1]) for r in merged], shift_x, shift_i))
    finally:
        dist.destroy_process_group()


def test_two_cpu_ranks_reproduce_the_single_process_step():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, q)) for r in range(WORLD)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    allc, tot, far, shift_x, shift_i = res
    X, C, labels, best = _case()
    n = len(X)
    # shards: contiguous, aligned, covering
    assert allc[0][0] == 0 and allc[-1][1] == n and allc[0][1] == allc[1][0] and allc[0][1] % 512 == 0
    # all-reduced integer totals equal the one-process totals bit for bit
    single = _quantised_totals(X, labels, best, len(C), shift_x, shift_i)
    assert np.array_equal(np.array(tot, np.int64), single)
    # merged candidates equal the global far-row order (core.py:2227-2229)
    want = sorted(range(n), key=lambda i: (-best[i], i))[:5]
    assert far == want
