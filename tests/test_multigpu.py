"""Sharded Lloyd steps over 2 GPUs (totals summed through peer memory) against one GPU: the centers, inertia and
counts after several steps must be bit-identical (exact int64 totals, shards on the block grid), on the low-d
bounded pass (config 3), the CUDA-core pass (config 1) and the tensor-core pass with wide totals (config 5's
shape on 1.5M rows). Skipped with fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

N_ROWS = 1_500_000
STEPS = 4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(rank, world, port, out, cfg):
    import sys
    sys.path.insert(0, ROOT)
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    group = None
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        group = dist.group.WORLD
    try:
        from mlx_kmeans_b200 import core
        from mlx_kmeans_b200.data import CONFIGS, generate, shard_range
        lo, hi = shard_range(N_ROWS, rank, world)
        X = generate(cfg, lo, hi - lo, dev, rows_total=N_ROWS, group=group)
        ds = core.Dataset([X], group=group)
        rng = np.random.default_rng(0)
        k = CONFIGS[cfg]["k"]
        C = torch.from_numpy(rng.standard_normal((k, CONFIGS[cfg]["dims"])).astype(np.float32)).to(dev)
        hist = []
        for _ in range(STEPS):
            C_new, s = ds.step(C)
            C = C_new.clone()
            hist.append((s["inertia"], s["n_empty"]))
        sums, counts, inertia = ds.assign(C)
        if rank == 0:
            out.put((C.cpu().numpy(), hist, counts, inertia))
    finally:
        if group is not None:
            dist.destroy_process_group()


def _spawn(world, cfg):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_run, args=(r, world, port, q, cfg)) for r in range(world)]
    for p in procs:
        p.start()
    res = q.get(timeout=300)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.parametrize("cfg", [3, 1, 5])        # 5: wide totals (k = 4096, d = 128), the multi-CTA exchange
def test_two_gpus_match_one_gpu_bit_for_bit(cfg):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    one = _spawn(1, cfg)
    two = _spawn(2, cfg)
    assert np.array_equal(one[0], two[0]), "centers differ between 1 and 2 GPUs"
    assert one[1] == two[1], "per-step inertia / empties differ"
    assert np.array_equal(one[2], two[2]) and one[3] == two[3]
