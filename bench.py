#!/usr/bin/env python3
"""Benchmark: exact Lloyd passes on B200 (the reference's hot path), one JSON line on rank 0.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config 3] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...        (one rank per GPU, NCCL)

A step is one Lloyd pass of the workload -- nearest center for every row, exact per-cluster totals, the
all-reduce of the totals over ranks, the on-device center update -- with the centers chained from step to step
as in a fit. The default workload is configuration 3 of the benchmark (96M x 4 float32, k=16), the 96M-row
shape the targets are set on; its rows are split over the GPUs (strong scaling), generated on each GPU from the
global row index. Inputs (1.5 GB) are larger than L2 (126 MB), so no flush is needed between steps.

  value      rows/s of the whole job, K device-timed steps (CUDA events, max over ranks), inputs in HBM
  e2e        the same metric through the public API (mlx_kmeans_b200.lloyd_step) with the rows copied from
             pinned host memory every step and the new centers read back
  roofline   the pass kernel: one read of X (4 n d bytes per GPU) per launch / its CUDA-event time, against
             MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the reference's CPU path (NumPy assign_numpy + center update, restated in oracle/) on a
             leading sample of the workload, rank 0 at N=1 only
--impl reference runs only that CPU path (the reference itself is MLX/Metal and cannot run here).
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "ms per Lloyd pass & rows/s at 1/2/4/8 B200; % of HBM or tensor roofline"
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=400)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--config", type=int, default=3)
    p.add_argument("--rows", type=int, default=None, help="override the configuration's row count (profiling)")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--e2e-steps", type=int, default=10)
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--no-e2e", action="store_true")
    p.add_argument("--generic", action="store_true", help="force the any-shape kernel (diagnostic)")
    p.add_argument("--no-bounds", action="store_true", help="compare every row with every center each pass")
    p.add_argument("--cascade", action="store_true",
                   help="the prefix-pruning cascade (kmc_pass_cascade; 128-256 dims, k >= 256)")
    p.add_argument("--column-decay", type=float, default=None,
                   help="scale column j's spread by R^p(j) (p a seeded permutation): data with variance structure, "
                        "the cascade's case (SIFT-like)")
    p.add_argument("--approx", action="store_true",
                   help="exact=False: the approximate tensor-core pass (one bf16 product per score; d >= 64)")
    return p.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return json.load(f), "measured"
    except (OSError, ValueError):
        return dict(PEAKS_FALLBACK), "fallback"


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"kmc_clocks_{os.getpid()}.csv")

    def _lines(self):
        try:
            with open(self.path) as f:
                return f.read().count("\n")
        except OSError:
            return 0

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        # nvidia-smi can take a while to start (several ranks start it at once): the timed region (short at
        # 8 GPUs) begins only once sampling runs, at most 5 s later
        t = time.time()
        while self._lines() == 0 and time.time() - t < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"], "samples": 0}
        # one sample after the timed region too
        n, t = self._lines(), time.time()
        while self._lines() <= n and time.time() - t < 0.5 and self.proc.poll() is None:
            time.sleep(0.01)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


def cpu_baseline(cfg, budget_s=12.0, rows=4_000_000):
    """The reference's CPU Lloyd pass (oracle/assign_numpy_port.py, core.py:197-215) on a leading sample: at most
    `rows` rows, fewer where a pass of them would take more than a quarter of the budget (a probe pass on 20k rows
    sets the rate)."""
    from oracle.assign_numpy_port import cpu_lloyd_pass
    from mlx_kmeans_b200.data import CONFIGS, host_sample
    c = CONFIGS[cfg]
    probe = host_sample(cfg, min(20_000, c["rows"]), seed_offset=1)
    cpu_lloyd_pass([probe], probe[:c["k"]].copy())
    t = time.perf_counter()
    cpu_lloyd_pass([probe], probe[:c["k"]].copy())
    rate = len(probe) / (time.perf_counter() - t)
    n = int(max(10_000, min(rows, c["rows"], rate * budget_s / 4)))
    X = host_sample(cfg, n)
    rng = np.random.default_rng(0)
    C = X[rng.choice(n, c["k"], replace=False)].copy()
    cpu_lloyd_pass([X], C)                                   # warm-up (BLAS threads, page faults)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
        t = time.perf_counter()
        C, _, _ = cpu_lloyd_pass([X], C)
        times.append(time.perf_counter() - t)
    med = statistics.median(times)
    try:
        from threadpoolctl import threadpool_info
        blas = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        blas = os.cpu_count()
    return {"value": n / med, "unit": "rows/s", "cores": int(blas), "kind": "port",
            "sample": f"{n} rows of {c['rows']} ({'config %d' % cfg}), median of {len(times)} passes, "
                      f"{med * 1e3:.1f} ms/pass; NumPy restatement of the reference's assign_numpy + center update",
            "ms_per_pass_sample": med * 1e3, "extrapolated_ms_per_pass_full": med * 1e3 * c["rows"] / n}


def run_reference(args):
    """--impl reference: the reference's CPU path on the box's host cores (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from threadpoolctl import threadpool_limits
    threadpool_limits(os.cpu_count())          # torchrun sets OMP_NUM_THREADS=1; the baseline uses every core
    from mlx_kmeans_b200.data import CONFIGS, DESCRIPTION, host_sample
    from oracle.assign_numpy_port import cpu_lloyd_pass
    cfg = args.config
    c = CONFIGS[cfg]
    # size each step so the whole run stays within ~2 minutes
    probe_n = min(500_000, c["rows"])
    Xp = host_sample(cfg, probe_n, seed_offset=1)
    Cp = Xp[:c["k"]].copy()
    cpu_lloyd_pass([Xp], Cp)
    t = time.perf_counter()
    cpu_lloyd_pass([Xp], Cp)
    rate = probe_n / (time.perf_counter() - t)
    per_step = 100.0 / max(1, args.steps + args.warmup)
    n = int(max(10_000, min(4_000_000, c["rows"], rate * per_step)))
    X = host_sample(cfg, n)
    rng = np.random.default_rng(0)
    C = X[rng.choice(n, c["k"], replace=False)].copy()
    for _ in range(args.warmup):
        C, _, _ = cpu_lloyd_pass([X], C)
    times = []
    for _ in range(args.steps):
        t = time.perf_counter()
        C, _, _ = cpu_lloyd_pass([X], C)
        times.append(time.perf_counter() - t)
    total = sum(times)
    value = n * args.steps / total
    try:
        from threadpoolctl import threadpool_info
        cores = max((i.get("num_threads", 1) for i in threadpool_info()), default=1)
    except Exception:
        cores = os.cpu_count()
    sample = (f"{n} rows per step of the {c['rows']}-row workload (NumPy restatement of the reference's "
              f"assign_numpy + center update, core.py:197-215)")
    line = {"metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total / args.steps * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "impl": "reference",
            "config": {"workload": DESCRIPTION[cfg], "rows_per_step": n, "dims": c["dims"], "k": c["k"]},
            "cpu_baseline": {"value": value, "unit": "rows/s", "cores": int(cores), "kind": "port",
                             "sample": sample},
            "e2e": {"value": value, "unit": "rows/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist
    from mlx_kmeans_b200 import _lib, core
    from mlx_kmeans_b200.data import CONFIGS, DESCRIPTION, column_scales, generate, shard_range

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    group = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        group = dist.group.WORLD

    cfg = args.config
    c = dict(CONFIGS[cfg])
    if args.rows:
        c["rows"] = args.rows
    n_total, d, k = c["rows"], c["dims"], c["k"]
    lo, hi = shard_range(n_total, rank, world)
    X = generate(cfg, lo, hi - lo, dev, rows_total=n_total, group=group)
    if args.column_decay:
        X.mul_(torch.from_numpy(column_scales(d, args.column_decay, c["seed"])).to(dev))
    ds = core.Dataset([X], group=group)
    ds.cascade = args.cascade

    # identical initial centers on every rank: greedy k-means++ on the first rows, broadcast from rank 0
    m = min(n_total, c["pp_sample"] or 20_000, hi - lo if world == 1 else n_total)
    S = X[:m].contiguous() if rank == 0 else torch.empty((m, d), dtype=torch.float32, device=dev)
    if world > 1:
        dist.broadcast(S, src=0)
    rng = np.random.default_rng(c["seed"])
    C = core.pp_init_device(S, k, int(rng.integers(m)), rng.integers(2**63 - 1, size=k - 1).astype(np.uint64))

    # warm-up: full Lloyd steps (relocation handled)
    for _ in range(max(args.warmup, 3)):
        C_new, s = ds.step(C, generic=args.generic, bounded=not args.no_bounds, approx=args.approx,
                           cascade=args.cascade)
        C = C_new.clone()

    L = _lib.load()
    b = ds.buffers(k)
    cm = ds.colmax
    st = torch.cuda.current_stream()
    sp = st.cuda_stream
    K = args.steps
    stats = torch.zeros((K, _lib.STATS_BYTES), dtype=torch.uint8, device=dev)
    Cs = [C.clone(), torch.empty_like(C)]
    # per-row bounds carried over from the warm-up steps (the fit's own state)
    tc = ds.tensor_cores and not args.generic       # d >= 32: the tensor-core pass (kmc_pass_split)
    bounded = not args.no_bounds and not args.generic and not tc
    bb, bbytes = ds.bounds(k)[0] if bounded else (None, 0)
    approx = args.approx and tc and ds.uses_approx(True)
    elk = None
    casc = None
    if tc and args.cascade and ds.cascade_ok(k, forced=True):
        casc = ds.cascade_state(k)                    # prefix split and state built by the warm-up steps
        Cm = torch.empty((k, casc["m"]), dtype=torch.float32, device=dev)
    if tc:
        (spl, splb), (csp, cspb) = ds.split()[0], ds.csplit(k)
        # per-center bounds (kmc_pass_elkan) built by the warm-up steps, used by every timed step
        e = ds._elkan.get(k)
        if not args.no_bounds and not approx and e is not None and e["valid"]:
            elk = e["bufs"][0]
    flags = _lib.KMC_PASS_GENERIC if args.generic else 0
    if approx:
        flags |= _lib.KMC_PASS_APPROX
    xch = ds._exchange(k) if world > 1 else False
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = Clocks(vis.split(",")[local] if vis else str(local))

    clocks.start()
    time.sleep(0.2)
    # the barrier right before the first timed launch: a rank that starts late would otherwise keep the others
    # waiting in the first step's exchange, and that start-up skew would count as step time
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    t0.record(st)
    h0 = time.perf_counter()
    for i in range(K):
        Cin, Cout = Cs[i % 2], Cs[(i + 1) % 2]
        ev[i][0].record(st)
        if casc is not None:
            torch.index_select(Cin, 1, casc["cols"], out=Cm)
            (ms, mb), (cbuf, cbytes) = casc["msplits"][0], casc["bufs"][0]
            _lib.check(L.kmc_pass_cascade(X.data_ptr(), X.shape[0], d, Cin.data_ptr(), k, cm.data_ptr(), n_total,
                                          b["totals"].data_ptr(), None, None, flags, spl.data_ptr(), splb,
                                          csp.data_ptr(), cspb, Cm.data_ptr(), casc["m"], ms.data_ptr(), mb,
                                          casc["mcsplit"][0].data_ptr(), casc["mcsplit"][1], cbuf.data_ptr(), cbytes,
                                          b["ws"].data_ptr(), b["wsb"], sp))
        elif elk is not None:
            _lib.check(L.kmc_pass_elkan(X.data_ptr(), X.shape[0], d, Cin.data_ptr(), k, cm.data_ptr(), n_total,
                                        b["totals"].data_ptr(), None, None, flags, spl.data_ptr(), splb,
                                        csp.data_ptr(), cspb, elk[0].data_ptr(), elk[1], b["ws"].data_ptr(),
                                        b["wsb"], sp))
        elif tc:
            _lib.check(L.kmc_pass_split(X.data_ptr(), X.shape[0], d, Cin.data_ptr(), k, cm.data_ptr(), n_total,
                                        b["totals"].data_ptr(), None, None, flags, spl.data_ptr(), splb,
                                        csp.data_ptr(), cspb, b["ws"].data_ptr(), b["wsb"], sp))
        elif bounded:
            _lib.check(L.kmc_pass_bounded(X.data_ptr(), X.shape[0], d, Cin.data_ptr(), k, cm.data_ptr(), n_total,
                                          b["totals"].data_ptr(), flags, bb.data_ptr(), bbytes, b["ws"].data_ptr(),
                                          b["wsb"], sp))
        else:
            _lib.check(L.kmc_pass(X.data_ptr(), X.shape[0], d, Cin.data_ptr(), k, cm.data_ptr(), n_total,
                                  b["totals"].data_ptr(), None, None, flags, b["ws"].data_ptr(), b["wsb"], sp))
        ev[i][1].record(st)
        if xch:      # the all-reduce over peer memory and the finish in one launch
            _lib.check(L.kmc_exchange_finish(b["totals"].data_ptr(), k, d, xch["dev"].data_ptr(), world, rank,
                                             xch["step"], Cout.data_ptr(), stats[i].data_ptr(), b["ws"].data_ptr(),
                                             b["wsb"], sp))
            xch["step"] += 1
        else:
            ds.allreduce_totals(b, k)
            _lib.check(L.kmc_finish(b["totals"].data_ptr(), k, d, None, 0, 1, Cout.data_ptr(), stats[i].data_ptr(),
                                    b["ws"].data_ptr(), b["wsb"], sp))
    t1.record(st)
    host_ms = (time.perf_counter() - h0) * 1e3 / K      # host time to issue one step (the GPU must not wait)
    torch.cuda.synchronize()
    clk = clocks.stop()
    if world > 1:
        dist.barrier()
    total_ms = t0.elapsed_time(t1)
    pass_ms = statistics.mean(a.elapsed_time(z) for a, z in ev)
    st_host = stats.cpu().numpy().view(np.int64).reshape(K, 8)
    reloc_steps = int((st_host[:, 3] != 0).sum())
    rescored = float(st_host[:, 5].mean())
    screened = float(st_host[:, 6].mean()) / max(1, hi - lo)
    if world > 1:
        t = torch.tensor([total_ms, pass_ms], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        total_ms, pass_ms = float(t[0]), float(t[1])
    ms_per_step = total_ms / K
    value = n_total / (ms_per_step * 1e-3)

    # end to end through the public API: pinned host rows -> device, lloyd_step, centers back to the host
    e2e = None
    if not args.no_e2e:
        import mlx_kmeans_b200 as km
        Xh = torch.empty(X.shape, dtype=torch.float32, pin_memory=True)
        Xh.copy_(X)
        Xd = torch.empty_like(X)
        Ch = Cs[K % 2].cpu().numpy()
        E = max(1, args.e2e_steps)
        for it in range(E + 2):
            if it == 2:
                if world > 1:
                    dist.barrier()
                torch.cuda.synchronize()
                a0 = torch.cuda.Event(enable_timing=True)
                a0.record(st)
            Xd.copy_(Xh, non_blocking=True)
            Ch, inertia, n_empty = km.lloyd_step(core.Dataset([Xd], group=group), Ch,
                                                 method="approx" if args.approx else "auto")
        a1 = torch.cuda.Event(enable_timing=True)
        a1.record(st)
        torch.cuda.synchronize()
        e_ms = a0.elapsed_time(a1) / E
        if world > 1:
            t = torch.tensor([e_ms], dtype=torch.float64, device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
            e_ms = float(t[0])
        e2e = {"value": n_total / (e_ms * 1e-3), "unit": "rows/s", "ms_per_step": e_ms, "steps": E,
               "h2d_bytes_per_step": int(X.numel() * 4), "d2h_bytes_per_step": int(k * d * 4 + 64),
               "api": "mlx_kmeans_b200.lloyd_step(Dataset([rows copied from pinned host memory]), C)"}

    pk, src = peaks()
    bytes_per_launch = (hi - lo) * d * 4
    flops_per_launch = 2.0 * (hi - lo) * k * d
    achieved = bytes_per_launch / (pass_ms * 1e-3) / 1e9
    # the roofline is the slower of one read of X at HBM bandwidth and the distance GEMM at tensor peak (the
    # sustained bf16 figure: the pass runs in a long loop); the split pass issues three bf16 MMAs per product,
    # so its own ceiling is a third of that peak
    tpeak = pk.get("bf16_tflops_sustained", pk.get("bf16_tflops"))
    tensor_bound = tc and flops_per_launch / (tpeak * 1e12) > bytes_per_launch / (pk["hbm_gbs"] * 1e9)
    mmas = 1 if approx else 3             # bf16 MMAs per product: the pass's own ceiling is peak / mmas
    if casc is not None:
        mmas = 3.0 * casc["m"] / d        # the cascade multiplies the prefix columns only
    traffic = None
    tpath = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(tpath):
        try:
            traffic = json.load(open(tpath)).get(f"config{cfg}_{world}gpu")
        except ValueError:
            traffic = None
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world, "steps": K, "warmup": args.warmup,
        "ms_per_step": ms_per_step, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": DESCRIPTION[cfg] + ("" if n_total == CONFIGS[cfg]["rows"] else
                                                   f" (rows overridden: {n_total})"),
                   "rows": n_total, "dims": d, "k": k,
                   "parallelism": f"rows sharded dp{world}, int64 totals all-reduced " +
                                  ("(peer memory, kmc_exchange_finish)" if world > 1 and ds._xch.get(k) else "(NCCL)"),
                   "l2": "inputs larger than L2 (%.2f GB per GPU), no flush" % (bytes_per_launch / 1e9),
                   "relocation_steps_in_timed_region": reloc_steps,
                   "rows_rescored_in_float64_per_pass": rescored,
                   "per_row_bounds": bounded,
                   "per_center_bounds": elk is not None,
                   "fraction_of_rows_compared_with_every_center": screened if bounded else 1.0,
                   "fraction_of_row_center_pairs_visited": (screened / k) if (elk is not None or casc is not None)
                                                           else None,
                   "column_decay": args.column_decay,
                   "kernel": "generic" if args.generic else (("tensor cores (" +
                                                               ("kmc_pass_cascade, prefix of %d columns)" % casc["m"]
                                                                if casc is not None else
                                                                "kmc_pass_split" +
                                                                (", exact=False)" if approx else ")")))
                                                              if tc else "auto")},
        "roofline": ({"bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
                      "frac": achieved / pk["hbm_gbs"], "traffic": traffic,
                      "kernel_ms": pass_ms, "algorithmic_bytes_per_launch": bytes_per_launch,
                      "peak_source": f"{src} hbm_gbs (MEASURED_PEAKS.json)" if src == "measured" else "fallback"}
                     if not tensor_bound else
                     {"bound": "tensor", "achieved": flops_per_launch / (pass_ms * 1e-3) / 1e12, "peak": tpeak,
                      "unit": "TFLOP/s", "frac": flops_per_launch / (pass_ms * 1e-3) / 1e12 / tpeak,
                      "frac_of_split_ceiling": mmas * flops_per_launch / (pass_ms * 1e-3) / 1e12 / tpeak,
                      "bf16_mmas_per_product": mmas,
                      "traffic": traffic, "kernel_ms": pass_ms, "algorithmic_flops_per_launch": flops_per_launch,
                      "peak_source": (f"{src} bf16_tflops_sustained (MEASURED_PEAKS.json)" if src == "measured"
                                      else "fallback")}),
        "clocks": clk,
        # per step: k_prepare, the pass (tensor cores: k_split_centers, k_assign_tc and the seven kernels of the
        # float64 decision and the per-cluster reduction), k_finish (it runs the all-reduce over peer memory first
        # on several GPUs; with NCCL instead, NCCL's own kernel, not counted) and, above 32768 center values,
        # k_finish_centers
        # (with per-center bounds: k_elkan_drift and k_elkan in place of k_assign_tc)
        "gpu_launches": ((11 + (1 if elk is not None else 0) + (1 if k * d > 32768 else 0)) if tc else 3) * K,
        "host_enqueue_ms_per_step": host_ms,
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu:
        line["cpu_baseline"] = cpu_baseline(cfg)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
