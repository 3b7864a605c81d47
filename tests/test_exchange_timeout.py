"""Failure detection of the peer-memory all-reduce, on one GPU and without a fault (-m gpu).

A rank of a sharded Lloyd step waits for its peers' flags for at most KMC_EXCHANGE_TIMEOUT_MS milliseconds; a
peer that never arrives makes the wait give up, the kernel sets statistics flag 2 and keeps the rank's own
totals, and Dataset.step raises RuntimeError. Here "the peer" is a second exchange buffer on the same GPU whose
flag nothing raises (world = 2, rank 0), with a 200 ms limit; afterwards the GPU context is still usable.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

K, D, N = 16, 4, 200_000


def _setup(device):
    import torch
    from mlx_kmeans_b200 import _lib
    L = _lib.load()
    nb = int(L.kmc_exchange_bytes(K, D))
    own = torch.zeros(nb, dtype=torch.uint8, device=device)
    peer = torch.zeros(nb, dtype=torch.uint8, device=device)        # a peer that never publishes
    peers = torch.tensor([own.data_ptr(), peer.data_ptr()], dtype=torch.int64, device=device)
    rng = np.random.default_rng(2)
    X = rng.standard_normal((N, D)).astype(np.float32)
    return L, _lib, own, peer, peers, X


def test_exchange_gives_up_on_a_missing_peer(cuda_device, monkeypatch):
    import torch
    monkeypatch.setenv("KMC_EXCHANGE_TIMEOUT_MS", "200")
    L, lib, own, peer, peers, X = _setup(cuda_device)
    import mlx_kmeans_b200 as km
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    C = ds.parts[0][:K].contiguous()
    b = ds.run_pass(C)
    mine = b["totals"].clone()
    st = torch.cuda.current_stream().cuda_stream
    # kmc_exchange_sum alone, then the finish that reports its flag
    lib.check(L.kmc_exchange_sum(b["totals"].data_ptr(), K, D, peers.data_ptr(), 2, 0, 0, b["ws"].data_ptr(),
                                 b["wsb"], st), "kmc_exchange_sum")
    lib.check(L.kmc_finish(b["totals"].data_ptr(), K, D, None, 0, 1, b["C_new"].data_ptr(), b["stats"].data_ptr(),
                           b["ws"].data_ptr(), b["wsb"], st), "kmc_finish")
    s = ds.read_stats(b)
    assert s["flags"] & 2, s
    assert torch.equal(b["totals"], mine)                # the rank's own totals are kept
    # this rank raised its flag in the peer's buffer (flag slot 0 = rank 0) before waiting
    assert int(peer[:8].view(torch.int64)[0]) == 1


def test_sharded_step_raises_when_a_peer_never_arrives(cuda_device, monkeypatch):
    import torch
    monkeypatch.setenv("KMC_EXCHANGE_TIMEOUT_MS", "200")
    L, lib, own, peer, peers, X = _setup(cuda_device)
    import mlx_kmeans_b200 as km
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    ds.colmax                                            # (the column maxima of this one-GPU Dataset, computed now)
    # a sharded Dataset's exchange state, with the stand-in peer: the step takes the fused exchange + finish
    ds.group, ds.world, ds.rank = object(), 2, 0
    ds._xch[K] = dict(dev=peers, step=0)
    with pytest.raises(RuntimeError, match="timed out"):
        ds.step(ds.parts[0][:K].contiguous())
    # the context is still usable: a plain pass on the same data
    fresh = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    _, counts, _ = fresh.assign(fresh.parts[0][:K].contiguous())
    assert counts.sum() == N


@pytest.mark.parametrize("k,d", [(512, 62), (4096, 128)])
def test_wide_exchange_gives_up_on_a_missing_peer(k, d, cuda_device, monkeypatch):
    """Wide totals (k (d + 2) >= 16384 values) take the multi-CTA exchange, one flag row per CTA: every CTA
    raises its flag in the peer's row and gives up on its own; flag 2 is reported and the totals are kept."""
    import torch
    from mlx_kmeans_b200 import _lib
    import mlx_kmeans_b200 as km
    monkeypatch.setenv("KMC_EXCHANGE_TIMEOUT_MS", "200")
    L = _lib.load()
    nb = int(L.kmc_exchange_bytes(k, d))
    own = torch.zeros(nb, dtype=torch.uint8, device=cuda_device)
    peer = torch.zeros(nb, dtype=torch.uint8, device=cuda_device)
    peers = torch.tensor([own.data_ptr(), peer.data_ptr()], dtype=torch.int64, device=cuda_device)
    rng = np.random.default_rng(3)
    X = rng.standard_normal((20_000, d)).astype(np.float32)
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    b = ds.run_pass(ds.parts[0][:k].contiguous())
    mine = b["totals"].clone()
    st = torch.cuda.current_stream().cuda_stream
    _lib.check(L.kmc_exchange_finish(b["totals"].data_ptr(), k, d, peers.data_ptr(), 2, 0, 0, b["C_new"].data_ptr(),
                                     b["stats"].data_ptr(), b["ws"].data_ptr(), b["wsb"], st), "kmc_exchange_finish")
    s = ds.read_stats(b)
    assert s["flags"] & 2, s
    assert torch.equal(b["totals"], mine)
    W = k * (d + 2)
    ctas = min(64, (W + 4095) // 4096)
    flags = peer[: 64 * 64 * 8].view(torch.int64).view(64, 64).cpu().numpy()
    assert (flags[:ctas, 0] == 1).all() and (flags[ctas:, :] == 0).all() and (flags[:, 1:] == 0).all()


@pytest.mark.parametrize("k,d", [(16, 4), (512, 62), (1000, 129)])
def test_exchange_of_one_rank_keeps_the_totals(k, d, cuda_device):
    """world = 1: the one-CTA and multi-CTA exchanges copy every range into the slot and sum it back unchanged
    (ragged last range included), over several steps (both slots)."""
    import torch
    from mlx_kmeans_b200 import _lib
    import mlx_kmeans_b200 as km
    L = _lib.load()
    own = torch.zeros(int(L.kmc_exchange_bytes(k, d)), dtype=torch.uint8, device=cuda_device)
    peers = torch.tensor([own.data_ptr()], dtype=torch.int64, device=cuda_device)
    rng = np.random.default_rng(4)
    X = rng.standard_normal((20_000, d)).astype(np.float32)
    ds = km.Dataset([torch.from_numpy(X).to(cuda_device)])
    b = ds.run_pass(ds.parts[0][:k].contiguous())
    mine = b["totals"].clone()
    st = torch.cuda.current_stream().cuda_stream
    for step in range(3):
        _lib.check(L.kmc_exchange_sum(b["totals"].data_ptr(), k, d, peers.data_ptr(), 1, 0, step, b["ws"].data_ptr(),
                                      b["wsb"], st), "kmc_exchange_sum")
        torch.cuda.synchronize()
        assert torch.equal(b["totals"], mine)
