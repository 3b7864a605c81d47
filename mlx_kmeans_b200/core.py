"""Host side of the Lloyd hot path: the functions of the reference's mlx_kmeans/core.py that sit on the
path, with the same names, arguments, return values and errors, running on libkmc.so.

    lloyd_step(parts, C)            core.py:2209-2242
    assign_mlx(parts, C, ...)       core.py:2200-2206
    kmeans_pp_init(parts, rows, k, rng, sample=None)   core.py:153-192
    kmeans(parts, rows, k, ...)     core.py:2247-2273
    take_rows, slice_rows, make_data_numpy               core.py:19-40, 132-143

`parts` are float32 (rows, dims) CUDA tensors (torch is the device-memory plumbing), NumPy arrays (copied to
the device once per call), or a Dataset, which keeps the per-dataset state (column maxima, workspaces) between
passes the way the reference keeps its per-array caches (core.py:548-578). Multi-GPU: a Dataset built with a
torch.distributed process group holds this rank's contiguous row shard; the per-cluster totals are summed over
ranks with one all-reduce per pass (int64, exact).
"""
import ctypes
import os
import weakref

import numpy as np
import torch

from . import _lib

SLICE_ROWS = 100_000_000            # kept for API parity: the kernels use 64-bit offsets, so slices are optional
PART_MAX_ELEMENTS = 2**62           # no 32-bit addressing limit here (core.py:19-20 has 2**32 - 1)

EXACT_METHODS = ("auto", "rows", "pairs", "tiles", "tiles1", "cascade", "onehot", "fused", "generic")
ACCUMULATE_METHODS = ("auto", "blocks", "sorted", "lanes", "atomic")


def slice_rows(dims):
    """Rows per slice (core.py:23-25). Kept for callers that slice; the library needs no slicing."""
    return SLICE_ROWS


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


# ---------------------------------------------------------------- data

def make_data_numpy(rows, dims, k, seed):
    """Points scattered around k hidden centers (the reference's make_data_numpy, core.py:30-40, same draws)."""
    rng = np.random.default_rng(seed)
    true_centers = rng.uniform(-10, 10, size=(k, dims)).astype(np.float32)
    X = np.empty((rows, dims), dtype=np.float32)
    chunk = 10_000_000
    for s in range(0, rows, chunk):
        e = min(s + chunk, rows)
        labels = rng.integers(0, k, size=e - s)
        X[s:e] = true_centers[labels] + rng.standard_normal((e - s, dims), dtype=np.float32)
    return [X]


def _as_part(p, device):
    """One slice as a contiguous float32 CUDA tensor, with the reference's shape errors (core.py:2022-2027)."""
    if isinstance(p, torch.Tensor):
        if p.ndim != 2:
            raise ValueError(f"each part must be 2-D (rows, dims), got {p.ndim}-D")
        t = p
        if t.device.type != "cuda":
            t = t.to(device)
        if t.dtype != torch.float32:
            t = t.float()
        return t.contiguous()
    a = np.asarray(p.to_numpy() if hasattr(p, "to_numpy") else p)
    if a.ndim != 2:
        raise ValueError(f"each part must be 2-D (rows, dims), got {a.ndim}-D")
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(device)


class Dataset:
    """Device-resident rows plus the state one Lloyd pass after another reuses.

    parts: list of (n_i, d) float32 CUDA tensors held by reference (never modified).
    group: torch.distributed process group when the rows are sharded over ranks (this rank's parts are a
    contiguous block of rows starting at global row `row0`); None on one GPU.
    """

    TC_MIN_DIMS = 32                # from here up the assign runs on the tensor cores (kmc_pass_split)
    APPROX_MIN_DIMS = 64            # exact=False from here up (core.py:1030-1034 / 2036-2041: below, exact is as fast)
    # per-center bounds (kmc_pass_elkan) on request (Dataset.elkan = True): while n k halves fit, and dropped by a
    # pass that visits more than 5% of the (row, center) pairs (the reference's BOUNDS_MAX_BYTES / BOUNDS_MAX_VISITED,
    # core.py:513-516).  Not by default: the bounded pass computes each visited distance on CUDA cores from the
    # center's float32 vector, which at configuration 4 costs more than the dense tensor-core pass until far fewer
    # than 1% of the pairs are visited (measured: 93% visited at step 5 of a fit, 2.7% at step 20, 16.9 ms against
    # 4.1 ms for the dense pass there)
    ELKAN_MAX_BYTES = 16 << 30
    ELKAN_MAX_VISITED = 0.05
    # the prefix-pruning cascade (kmc_pass_cascade) where the reference offers it (core.py:486-491: 128 to 256 dims,
    # k >= 256) and while its bounds fit; dropped once more than 15% of the (row, center) pairs survive.  Offered
    # when Dataset.cascade is True, or for one call by method="cascade" (the reference's accuracy suite forces it
    # that way); not by default: the dense tensor-core pass is faster on B200 at the shapes measured
    CASCADE_MIN_DIMS = 128
    CASCADE_MAX_DIMS = 256
    CASCADE_MIN_K = 256
    CASCADE_MAX_SURVIVORS = 0.15
    CASCADE_MAX_BYTES = 48 << 30    # the survivor bits, one per (row, center)

    def __init__(self, parts, group=None, device=None, tensor_cores=None, label_rule="float64"):
        if isinstance(parts, (torch.Tensor, np.ndarray)) or not isinstance(parts, (list, tuple)):
            parts = [parts]
        if not parts:
            raise ValueError("expected a nonempty 2-D (rows, dims) array")
        self.device = torch.device(device) if device is not None else (
            parts[0].device if isinstance(parts[0], torch.Tensor) and parts[0].is_cuda
            else torch.device("cuda", torch.cuda.current_device()))
        self.parts = [_as_part(p, self.device) for p in parts]
        d = self.parts[0].shape[1]
        for p in self.parts:
            if p.shape[1] != d:
                raise ValueError(f"data has {p.shape[1]} columns but the first slice has {d}")
        if d > _lib.KMC_MAX_DIMS:
            raise ValueError(f"{d} dims is above the supported maximum {_lib.KMC_MAX_DIMS}")
        self.d = d
        self.label_rule = _check_rule(label_rule)
        self.group = group
        self.n_local = sum(p.shape[0] for p in self.parts)
        if group is not None:
            self.rank, self.world, self.row0, self.n_total = shard_plan(self.n_local, group, self.device)
        else:
            self.rank, self.world, self.row0, self.n_total = 0, 1, 0, self.n_local
        self._ws = {}
        self._colmax = None
        self._bounds = {}
        # tensor_cores: None = by dims (d >= TC_MIN_DIMS), True / False to force
        self.tensor_cores = (d >= self.TC_MIN_DIMS) if tensor_cores is None else bool(tensor_cores)
        self._split = None
        self._csplit = {}
        self._xch = {}                  # per k: peer-memory exchange of the totals (multi-GPU), or False: NCCL
        self._elkan = {}                # per k: per-center bounds of the tensor-core pass and their policy state
        self.elkan = False              # True: per-center bounds between bounded tensor-core passes
        self._cascade = {}              # per k: the cascade's prefix, bounds and policy state
        self.cascade = False            # True: the prefix-pruning cascade where it applies
        self._split_ready = False       # a tensor-core pass has left labels and the grouped order in the splits

    # -- per-dataset state
    @property
    def colmax(self):
        """Global per-column max |x| (float32 bits as int32): the fixed-point grid of the totals."""
        if self._colmax is None:
            cm = torch.zeros(self.d, dtype=torch.int32, device=self.device)
            flags = 0
            for p in self.parts:
                _lib.call("kmc_colmax", _ptr(p), p.shape[0], self.d, _ptr(cm), flags, _stream())
                flags = _lib.KMC_PASS_ACCUMULATE
            if self.group is not None:
                allreduce_colmax(cm, self.group)
            self._colmax = cm
        return self._colmax

    def absmax(self):
        """max |x| over all rows and columns (host float; NaN / inf if the data holds them)."""
        bits = self.colmax.cpu().numpy().astype(np.uint32)
        vals = bits.view(np.float32)
        if (bits > 0x7F800000).any():
            return float("nan")
        return float(vals.max())

    def buffers(self, k):
        """Workspace, totals, stats and C_new buffers for k centers (reused across passes)."""
        b = self._ws.get(k)
        if b is None:
            L = _lib.load()
            wsb = int(L.kmc_workspace_bytes(self.d, k))
            b = dict(
                ws=torch.empty(wsb, dtype=torch.uint8, device=self.device), wsb=wsb,
                totals=torch.zeros((k, self.d + 2), dtype=torch.int64, device=self.device),
                stats=torch.zeros(_lib.STATS_BYTES, dtype=torch.uint8, device=self.device),
                C_new=torch.empty((k, self.d), dtype=torch.float32, device=self.device),
                labels=None, best=None)
            self._ws[k] = b
        return b

    def _label_buffers(self, b):
        if b["labels"] is None:
            b["labels"] = [torch.empty(p.shape[0], dtype=torch.int32, device=self.device) for p in self.parts]
            b["best"] = [torch.empty(p.shape[0], dtype=torch.float32, device=self.device) for p in self.parts]
        return b["labels"], b["best"]

    # -- per-row bounds kept between passes (kmc_pass_bounded), one buffer per slice and k
    def bounds(self, k):
        bb = self._bounds.get(k)
        if bb is None:
            L = _lib.load()
            bb = []
            for p in self.parts:
                nb = int(L.kmc_bounds_bytes(p.shape[0], self.d, k))
                bb.append((torch.zeros(nb, dtype=torch.uint8, device=self.device), nb))
            self._bounds[k] = bb
        return bb

    # -- tensor-core operands: bf16 hi / lo copies of the rows (once per dataset), the centers' (per k)
    def split(self):
        if self._split is None:
            L = _lib.load()
            sp = []
            for p in self.parts:
                nb = int(L.kmc_split_bytes(p.shape[0], self.d))
                t = torch.empty(nb, dtype=torch.uint8, device=self.device)
                _lib.call("kmc_split_rows", _ptr(p), p.shape[0], self.d, _ptr(t), nb, _stream())
                sp.append((t, nb))
            self._split = sp
        return self._split

    def csplit(self, k):
        cs = self._csplit.get(k)
        if cs is None:
            nb = int(_lib.load().kmc_csplit_bytes(self.d, k))
            cs = (torch.empty(nb, dtype=torch.uint8, device=self.device), nb)
            self._csplit[k] = cs
        return cs

    def reset_bounds(self):
        """Forget the per-row bounds: the next bounded pass compares every row with every center."""
        for bb in self._bounds.values():
            for t, _ in bb:
                _lib.call("kmc_bounds_reset", _ptr(t), _stream())
        for e in self._elkan.values():
            e["valid"], e["cool"], e["wait"] = False, 0, 0

    # -- per-center bounds of the tensor-core shapes (kmc_pass_elkan), one buffer per slice and k
    def elkan_ok(self, k):
        return (self.elkan is True and self.tensor_cores and k % 8 == 0 and
                self.n_local * k * 2 <= self.ELKAN_MAX_BYTES)

    def elkan_state(self, k):
        e = self._elkan.get(k)
        if e is None:
            L = _lib.load()
            bufs = []
            for p in self.parts:
                nb = int(L.kmc_elkan_bytes(p.shape[0], self.d, k))
                bufs.append((torch.empty(nb, dtype=torch.uint8, device=self.device), nb))
            e = dict(bufs=bufs, valid=False, cool=0, wait=0, used=False)
            self._elkan[k] = e
        return e

    def elkan_after(self, k, stats):
        """After a step: drop bounds that visited too many pairs, and wait longer each time that happens (1, 3,
        7 passes) before building them again -- on data where they cannot pay they cost a build now and then."""
        e = self._elkan.get(k)
        if e is None or not e["used"]:
            return
        if stats["screened"] > self.ELKAN_MAX_VISITED * self.n_local * k:
            e["valid"] = False
            e["cool"] = min(2 * e["cool"] + 1, 7)
            e["wait"] = e["cool"]
        else:
            e["cool"] = 0

    # -- the prefix-pruning cascade (kmc_pass_cascade): core.py:1198-1210 and 2085-2109
    def cascade_m(self):
        """Prefix width: half the dimensions in multiples of 8, 8 to 96 (core.py:1198-1200)."""
        return min(96, max(8, (self.d // 2) // 8 * 8))

    def cascade_ok(self, k, forced=False):
        """Whether a pass with k centers takes the cascade: the reference's shape rule (core.py:1203-1204) even when
        forced (core.py:2086, 2110: a forced cascade that does not apply falls through to the usual pass)."""
        if not (self.tensor_cores and k % 8 == 0 and self.n_local * k // 8 <= self.CASCADE_MAX_BYTES and
                self.CASCADE_MIN_DIMS <= self.d <= self.CASCADE_MAX_DIMS and k >= self.CASCADE_MIN_K):
            return False
        if forced:
            return True
        if self.cascade is not True:
            return False
        st = self._cascade.get(k)
        return st is None or st["ok"]

    def cascade_state(self, k):
        """The columns by decreasing variance (on a strided sample of the first slice, as core.py:2096-2098), the
        prefix of every slice split for the tensor cores, and the bounds buffers; built once per (dataset, k)."""
        st = self._cascade.get(k)
        if st is not None:
            return st
        L = _lib.load()
        m = self.cascade_m()
        step = max(1, self.parts[0].shape[0] // 65536)
        var = self.parts[0][::step].var(dim=0, unbiased=False)
        order = np.argsort(-var.cpu().numpy(), kind="stable").astype(np.int64)
        cols = torch.from_numpy(order[:m].copy()).to(self.device)
        msplits, bufs = [], []
        for p in self.parts:
            xm = p.index_select(1, cols).contiguous()
            nb = int(L.kmc_split_bytes(p.shape[0], m))
            t = torch.empty(nb, dtype=torch.uint8, device=self.device)
            _lib.call("kmc_split_rows", _ptr(xm), p.shape[0], m, _ptr(t), nb, _stream())
            msplits.append((t, nb))
            eb = int(L.kmc_cascade_bytes(p.shape[0], k))
            bufs.append((torch.empty(eb, dtype=torch.uint8, device=self.device), eb))
        del xm
        mcb = int(L.kmc_csplit_bytes(m, k))
        st = dict(m=m, order=order, cols=cols, msplits=msplits, bufs=bufs,
                  mcsplit=(torch.empty(mcb, dtype=torch.uint8, device=self.device), mcb), ok=True, used=False)
        self._cascade[k] = st
        return st

    def cascade_after(self, k, stats):
        """After a step: stop offering the cascade once a pass kept more than CASCADE_MAX_SURVIVORS of the pairs
        (core.py:2155-2156: the data has no variance structure the prefix can use)."""
        st = self._cascade.get(k)
        if st is not None and st["used"] and stats["screened"] > self.CASCADE_MAX_SURVIVORS * self.n_local * k:
            st["ok"] = False

    # -- the all-reduce of the totals over the ranks
    def _exchange(self, k):
        """Peer-memory exchange buffers for k centers: one per rank, mapped by every peer through CUDA IPC
        (kmc_exchange_*); False when the ranks cannot map each other's memory (then NCCL is used).  One set per
        (process group, k, d), shared by every Dataset of that group and held until the process exits: a peer
        may still be reading this rank's buffer when a Dataset goes away, so a buffer is never freed mid-run."""
        x = self._xch.get(k)
        if x is not None:
            return x
        key = (id(self.group), k, self.d)
        hit = _exchanges.get(key)
        if hit is not None:
            self._xch[k] = hit[1]
            return hit[1]
        x = self._open_exchange(k)
        _exchanges[key] = (self.group, x)          # (the group is kept so that its id is not reused)
        self._xch[k] = x
        return x

    def _open_exchange(self, k):
        import torch.distributed as dist
        L = _lib.load()
        x = False
        own = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(64)
        ok = os.environ.get("KMC_EXCHANGE", "peer") != "nccl" and \
            L.kmc_exchange_alloc(int(L.kmc_exchange_bytes(k, self.d)), ctypes.byref(own), handle) == 0
        oks = [None] * self.world
        dist.all_gather_object(oks, ok, group=self.group)
        if all(oks):
            handles = [None] * self.world
            dist.all_gather_object(handles, handle.raw, group=self.group)
            ptrs, opened = [], []
            for r in range(self.world):
                if r == self.rank:
                    ptrs.append(own.value)
                    continue
                p = ctypes.c_void_p()
                if L.kmc_exchange_open(handles[r], ctypes.byref(p)) != 0:
                    break
                ptrs.append(p.value)
                opened.append(p.value)
            oks = [None] * self.world
            dist.all_gather_object(oks, len(ptrs) == self.world, group=self.group)
            if all(oks):
                x = dict(dev=torch.tensor(ptrs, dtype=torch.int64, device=self.device), step=0)
            else:
                _close_exchange(opened, own.value)
        elif own.value:
            L.kmc_exchange_close(own, 1)
        return x

    def allreduce_totals(self, b, k):
        """Sum the int64 totals over the ranks: one peer-memory kernel (kmc_exchange_sum) when the ranks can map
        each other's buffers, else an NCCL all-reduce.  Either way the result is the exact integer sum."""
        if self.group is None:
            return
        x = self._exchange(k)
        if x:
            _lib.call("kmc_exchange_sum", _ptr(b["totals"]), k, self.d, _ptr(x["dev"]), self.world, self.rank,
                      x["step"], _ptr(b["ws"]), b["wsb"], _stream())
            x["step"] += 1
        else:
            import torch.distributed as dist
            dist.all_reduce(b["totals"], op=dist.ReduceOp.SUM, group=self.group)

    # -- one pass
    def uses_approx(self, approx):
        """Whether an exact=False pass takes the approximate kernel here (tensor-core shapes from
        APPROX_MIN_DIMS dims up; elsewhere it runs exactly, as the reference does below its crossover)."""
        return bool(approx) and self.tensor_cores and self.d >= self.APPROX_MIN_DIMS

    def run_pass(self, C, labels=False, generic=False, bounded=False, reduce=True, rule=None, approx=False,
                 cascade=False):
        """kmc_pass over every local slice, then (reduce) the all-reduce of the totals. C: (k, d) float32 CUDA.
        bounded: use and refresh the per-row bounds (kmc_pass_bounded; no labels). rule: the label rule ("float64"
        or "float32"; None: the Dataset's). approx: exact=False (one bf16 product per score, no window) where
        uses_approx allows it. cascade: force the prefix-pruning cascade for this pass (method="cascade") where the
        tensor-core pass runs; the Dataset's `cascade` attribute offers it to every exact pass."""
        k = C.shape[0]
        b = self.buffers(k)
        lab, bst = self._label_buffers(b) if labels else (None, None)
        cm = self.colmax
        flags = _lib.KMC_PASS_GENERIC if generic else 0
        if _check_rule(rule or self.label_rule) == "float32":
            flags |= _lib.KMC_PASS_LABEL32
        if not generic and self.uses_approx(approx):
            flags |= _lib.KMC_PASS_APPROX
        st = _stream()
        want_bounds = bounded and not labels and not generic
        tc = self.tensor_cores and not generic
        bb = self.bounds(k) if want_bounds and not tc else None
        eb = None
        casc = None
        if tc:
            sp, cs = self.split(), self.csplit(k)
            if not (flags & _lib.KMC_PASS_APPROX) and self.cascade_ok(k, forced=cascade):
                casc = self.cascade_state(k)
                casc["used"] = False
                if not self._split_ready:
                    # the cascade prunes against each row's previous label: a plain pass leaves them first
                    # (core.py:2104-2107 bootstraps a forced cascade the same way); the cascade below overwrites
                    # its totals
                    f0 = flags
                    for i, p in enumerate(self.parts):
                        _lib.call("kmc_pass_split", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                                  _ptr(b["totals"]), None, None, f0, _ptr(sp[i][0]), sp[i][1], _ptr(cs[0]), cs[1],
                                  _ptr(b["ws"]), b["wsb"], st)
                        f0 |= _lib.KMC_PASS_ACCUMULATE
                Cm = C.index_select(1, casc["cols"]).contiguous()
            elif want_bounds and self.elkan_ok(k) and not (flags & _lib.KMC_PASS_APPROX):
                eb = self.elkan_state(k)
                eb["used"] = False
                if not eb["valid"] and eb["wait"] > 0:
                    eb["wait"] -= 1
                    eb = None
            bb = None
        for i, p in enumerate(self.parts):
            if tc and casc is not None:
                ebuf, ebytes = casc["bufs"][i]
                ms, mb = casc["msplits"][i]
                _lib.call("kmc_pass_cascade", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                          _ptr(b["totals"]), _ptr(lab[i]) if labels else None, _ptr(bst[i]) if labels else None,
                          flags, _ptr(sp[i][0]), sp[i][1], _ptr(cs[0]), cs[1], _ptr(Cm), casc["m"], _ptr(ms), mb,
                          _ptr(casc["mcsplit"][0]), casc["mcsplit"][1], _ptr(ebuf), ebytes, _ptr(b["ws"]), b["wsb"],
                          st)
            elif tc and eb is not None:
                ebuf, ebytes = eb["bufs"][i]
                _lib.call("kmc_pass_elkan", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                          _ptr(b["totals"]), _ptr(lab[i]) if labels else None, _ptr(bst[i]) if labels else None,
                          flags | (0 if eb["valid"] else _lib.KMC_PASS_ELKAN_BUILD), _ptr(sp[i][0]), sp[i][1],
                          _ptr(cs[0]), cs[1], _ptr(ebuf), ebytes, _ptr(b["ws"]), b["wsb"], st)
            elif tc:
                _lib.call("kmc_pass_split", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                          _ptr(b["totals"]), _ptr(lab[i]) if labels else None, _ptr(bst[i]) if labels else None,
                          flags, _ptr(sp[i][0]), sp[i][1], _ptr(cs[0]), cs[1], _ptr(b["ws"]), b["wsb"], st)
            elif bb is not None:
                _lib.call("kmc_pass_bounded", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                          _ptr(b["totals"]), flags, _ptr(bb[i][0]), bb[i][1], _ptr(b["ws"]), b["wsb"], st)
            else:
                _lib.call("kmc_pass", _ptr(p), p.shape[0], self.d, _ptr(C), k, _ptr(cm), self.n_total,
                          _ptr(b["totals"]), _ptr(lab[i]) if labels else None, _ptr(bst[i]) if labels else None,
                          flags, _ptr(b["ws"]), b["wsb"], st)
            flags = flags | _lib.KMC_PASS_ACCUMULATE
        if eb is not None:
            eb["used"] = eb["valid"]              # this pass used the bounds (a build pass visits nothing)
            eb["valid"] = True
        if casc is not None:
            casc["used"] = True
        if tc:
            self._split_ready = True
        if reduce:
            self.allreduce_totals(b, k)
        return b

    def read_stats(self, b):
        host = np.zeros(8, dtype=np.int64)
        _lib.call("kmc_stats_read", _ptr(b["stats"]), host.ctypes.data, _stream())
        return dict(inertia=float(host[:1].view(np.float64)[0]), n_empty=int(host[1]), n_relocated=int(host[2]),
                    needs_reloc=int(host[3]), flags=int(host[4]), rescored=int(host[5]), screened=int(host[6]))

    def step(self, C, generic=False, bounded=True, rule=None, approx=False, cascade=False):
        """One Lloyd iteration on the device: C (k, d) CUDA -> (C_new CUDA tensor (a buffer reused by the
        next step with the same k; copy it to keep it), stats dict).  bounded: keep per-row bounds between
        steps so rows whose label cannot have changed skip the comparison with every center (the labels are
        those of a full pass; the totals agree to the float32 rounding of the per-lane partial sums).  rule: the
        label rule (None: the Dataset's). approx: exact=False (see run_pass)."""
        k = C.shape[0]
        x = self._exchange(k) if self.group is not None else False
        b = self.run_pass(C, generic=generic, bounded=bounded, reduce=not x, rule=rule, approx=approx,
                          cascade=cascade)
        if x:
            # the all-reduce over peer memory and the finish in one launch
            _lib.call("kmc_exchange_finish", _ptr(b["totals"]), k, self.d, _ptr(x["dev"]), self.world, self.rank,
                      x["step"], _ptr(b["C_new"]), _ptr(b["stats"]), _ptr(b["ws"]), b["wsb"], _stream())
            x["step"] += 1
        else:
            _lib.call("kmc_finish", _ptr(b["totals"]), k, self.d, None, 0, 1, _ptr(b["C_new"]), _ptr(b["stats"]),
                      _ptr(b["ws"]), b["wsb"], _stream())
        s = self.read_stats(b)
        if s["flags"] & 2:
            raise RuntimeError("the all-reduce of the totals timed out waiting for a peer GPU")
        self.elkan_after(k, s)
        self.cascade_after(k, s)
        if s["needs_reloc"]:
            s = self._relocate(C, b, s["n_empty"], generic, rule, approx, cascade)
        return b["C_new"], s

    def device_loop_ok(self, generic=False):
        """Whether a fit can run its Lloyd loop on the device (kmc_lloyd): one GPU, one slice, the CUDA-core
        pass (the tensor-core pass runs step by step)."""
        return self.group is None and len(self.parts) == 1 and (generic or not self.tensor_cores)

    def lloyd_loop(self, C, max_iter, tol, generic=False, bounded=True, rule=None):
        """Up to max_iter Lloyd steps from C (k, d) CUDA, stopping as the reference's estimator does
        (estimator.py:132-150: once |prev - inertia| <= tol * prev), with the loop on the device (kmc_lloyd): the
        host reads the loop's record once at the end, and once per step that empties clusters (that step is
        relocated here, as Dataset.step does, and the loop resumes).  -> (centers (k, d) CUDA tensor, inertia of the
        last step, steps run, flags of the last step)."""
        L = _lib.load()
        k = C.shape[0]
        b = self.buffers(k)
        if "loop" not in b:
            b["loop"] = torch.zeros(64, dtype=torch.uint8, device=self.device)
        loop = b["loop"]
        p = self.parts[0]
        cm = self.colmax
        flags = _lib.KMC_PASS_GENERIC if generic else 0
        if _check_rule(rule or self.label_rule) == "float32":
            flags |= _lib.KMC_PASS_LABEL32
        bb, bbytes = self.bounds(k)[0] if bounded and not generic else (None, 0)
        bufs = [C.clone(), torch.empty_like(C)]
        cur = 0                                        # the buffer holding the current centers
        st = _stream()
        done, prev, have = 0, 0.0, 0
        while True:
            _lib.call("kmc_loop_init", _ptr(loop), float(tol), int(max_iter), done, prev, have, st)
            _lib.call("kmc_lloyd", _ptr(p), p.shape[0], self.d, _ptr(bufs[cur]), _ptr(bufs[1 - cur]), k, _ptr(cm),
                      self.n_total, _ptr(b["totals"]), flags, _ptr(bb), bbytes, _ptr(b["stats"]), _ptr(loop),
                      int(max_iter - done), _ptr(b["ws"]), b["wsb"], st)
            rec = loop.cpu().numpy()                   # the one synchronising read of this segment
            ran = int(rec[16:24].view(np.int64)[0]) - done
            state = int(rec[32:40].view(np.int64)[0])
            cur = (cur + ran) % 2
            done += ran
            prev = float(rec[0:8].view(np.float64)[0])
            have = int(rec[40:48].view(np.int64)[0])
            if state != 2:                             # converged, max_iter, or non-finite: the last step's stats
                stats = self.read_stats(b)
                return bufs[cur], stats["inertia"], done, stats["flags"]
            # a step emptied clusters: relocate it on the host, then apply the stopping rule to it
            s = self._relocate(bufs[cur], b, self.read_stats(b)["n_empty"], generic, rule)
            done += 1
            inertia = s["inertia"]
            bufs[1 - cur].copy_(b["C_new"])
            cur = 1 - cur
            if s["flags"] & 1 or (have and abs(prev - inertia) <= tol * prev) or done >= max_iter:
                return bufs[cur], inertia, done, s["flags"]
            prev, have = inertia, 1

    def _relocate(self, C, b, n_empty, generic, rule=None, approx=False, cascade=False):
        """Empty clusters: recompute the pass with labels and best, gather the farthest rows of every slice
        and rank, and finish again with them (core.py:2224-2236)."""
        k = C.shape[0]
        b = self.run_pass(C, labels=True, generic=generic, rule=rule, approx=approx, cascade=cascade)
        E = int(n_empty)
        R = self.d + 4
        fwb = int(_lib.load().kmc_far_workspace_bytes(E))
        fws = torch.empty(fwb, dtype=torch.uint8, device=self.device)
        lists = []
        for i, p in enumerate(self.parts):
            cand = torch.empty((E, R), dtype=torch.int32, device=self.device)
            row0 = self.row0 + sum(q.shape[0] for q in self.parts[:i])
            _lib.call("kmc_far_rows", _ptr(p), p.shape[0], self.d, _ptr(b["labels"][i]), _ptr(b["best"][i]),
                      row0, E, _ptr(cand), _ptr(fws), fwb, _stream())
            lists.append(cand)
        local = torch.cat(lists, 0) if len(lists) > 1 else lists[0]
        nlists = len(lists)
        if self.group is not None:
            if len(self.parts) != 1:
                raise ValueError("a sharded Dataset holds one slice per rank")
            local = gather_candidates(local, self.group, self.world)
            nlists = self.world
        _lib.call("kmc_finish", _ptr(b["totals"]), k, self.d, _ptr(local), E, nlists, _ptr(b["C_new"]),
                  _ptr(b["stats"]), _ptr(b["ws"]), b["wsb"], _stream())
        return self.read_stats(b)

    def assign(self, C, return_labels=False, generic=False, rule=None, approx=False, cascade=False):
        """One pass -> (sums float64 (k, d), counts int64 (k), inertia float[, labels int64 (n_local)])."""
        k = C.shape[0]
        b = self.run_pass(C, labels=return_labels, generic=generic, rule=rule, approx=approx, cascade=cascade)
        sums = torch.empty((k, self.d), dtype=torch.float64, device=self.device)
        counts = torch.empty(k, dtype=torch.int64, device=self.device)
        inertia = torch.empty(1, dtype=torch.float64, device=self.device)
        _lib.call("kmc_totals_unpack", _ptr(b["totals"]), k, self.d, _ptr(sums), _ptr(counts), _ptr(inertia),
                  _ptr(b["ws"]), b["wsb"], _stream())
        out = (sums.cpu().numpy(), counts.cpu().numpy(), float(inertia.item()))
        if return_labels:
            out += (torch.cat(b["labels"]).to(torch.int64).cpu().numpy(),)
        return out


# (process-group id, k, d) -> (group, exchange): see Dataset._exchange
_exchanges = {}


# ---------------------------------------------------------------- multi-rank host steps (any torch.distributed
# backend: NCCL with CUDA tensors in the product, gloo with CPU tensors in the CPU tests)

def shard_plan(n_local, group, device):
    """(rank, world, row0, n_total) of a rank holding n_local contiguous rows: the rows of lower ranks come first."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    counts = torch.tensor([n_local], dtype=torch.int64, device=device)
    allc = [torch.zeros_like(counts) for _ in range(world)]
    dist.all_gather(allc, counts, group=group)
    allc = [int(c.item()) for c in allc]
    return rank, world, sum(allc[:rank]), sum(allc)


def allreduce_colmax(cm, group):
    """The global per-column max |x| from every rank's (float bits as int32: they order like the values)."""
    import torch.distributed as dist
    dist.all_reduce(cm, op=dist.ReduceOp.MAX, group=group)
    return cm


def gather_candidates(local, group, world):
    """Every rank's far-row candidate list (E records each, kmc_far_rows' layout), concatenated in rank order: the
    layout kmc_finish merges (farthest first, lower global row on ties) with ranks = world."""
    import torch.distributed as dist
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local, group=group)
    return torch.cat(gathered, 0)


def _close_exchange(opened, own):
    L = _lib.load()
    for p in opened:
        L.kmc_exchange_close(ctypes.c_void_p(p), 0)
    if own:
        L.kmc_exchange_close(ctypes.c_void_p(own), 1)


# identity cache, like core.py:548-578: a second array never sees the first one's state
_datasets = {}


def _dataset(parts):
    if isinstance(parts, Dataset):
        return parts
    if isinstance(parts, (torch.Tensor, np.ndarray)) or not isinstance(parts, (list, tuple)):
        parts = [parts]
    if all(isinstance(p, torch.Tensor) and p.is_cuda and p.dtype == torch.float32 and p.is_contiguous()
           and p.ndim == 2 for p in parts):
        key = tuple((id(p), p.data_ptr(), tuple(p.shape), p._version) for p in parts)
        hit = _datasets.get(key)
        if hit is not None:
            ds, refs = hit
            if all(r() is p for r, p in zip(refs, parts)):
                return ds
        ds = Dataset(list(parts))
        refs = [weakref.ref(p) for p in parts]

        def gone(_r, key=key):
            _datasets.pop(key, None)
        for p in parts:
            weakref.finalize(p, gone, None)
        _datasets[key] = (ds, refs)
        return ds
    return Dataset(list(parts))


LABEL_RULES = ("float64", "float32")


def _check_rule(rule):
    """The label rules: "float64" (the float64-optimal center, NumPy-pairwise distance, lowest index on ties: the
    reference's test oracle, tests/accuracy.py:31-51) or "float32" (the reference's exact-mode kernels' own rule,
    core.py:218-219 and 263-274: the float32 direct sum, strict < in index order)."""
    if rule not in LABEL_RULES:
        raise ValueError(f"label_rule must be one of {LABEL_RULES}, got {rule!r}")
    return rule


def _check_method(method, accumulate, k, d):
    if method not in EXACT_METHODS + ("approx",):
        raise ValueError(f"unknown method {method!r}")
    if accumulate not in ACCUMULATE_METHODS:
        raise ValueError(f"unknown accumulate {accumulate!r}")
    if method == "tiles" and (k % 8 or d % 8):
        raise ValueError(f"method='tiles' needs k and dims to be multiples of 8 (got k={k}, dims={d}); 'auto' picks it "
                         f"only where it applies")


def _centers(C, ds):
    C = np.ascontiguousarray(C, dtype=np.float32) if not isinstance(C, torch.Tensor) else C
    if C.ndim != 2:
        raise ValueError(f"centers must be 2-D (k, dims), got {C.ndim}-D")
    if C.shape[1] != ds.d:
        raise ValueError(f"data has {ds.d} columns but the centers have {C.shape[1]}; fit and predict need the "
                         f"same features")
    if isinstance(C, torch.Tensor):
        return C.to(ds.device, torch.float32).contiguous()
    return torch.from_numpy(C).to(ds.device)


# ---------------------------------------------------------------- the reference's entry points

def lloyd_step(parts, C, method="auto", accumulate="auto", label_rule=None):
    """One exact Lloyd iteration on the GPU -> (new centers float32, inertia, number of empty clusters).

    core.py:2209-2242: the inertia belongs to the centers the step started from; empty clusters take the
    farthest rows (farthest first, lower row index on ties), a cluster still empty takes the largest
    cluster's center. Everything but the statistics stays on the device. label_rule: "float64" or "float32"
    (None: the Dataset's, "float64" by default)."""
    ds = _dataset(parts)
    Cd = _centers(C, ds)
    _check_method(method, accumulate, Cd.shape[0], ds.d)
    C_new, s = ds.step(Cd, generic=(method == "generic"), rule=label_rule and _check_rule(label_rule),
                       approx=(method == "approx"), cascade=(method == "cascade"))
    inertia = float("nan") if s["flags"] & 1 else s["inertia"]
    return C_new.cpu().numpy(), inertia, s["n_empty"]


def assign_mlx(parts, C, method="auto", return_labels=False, accumulate="auto", label_rule=None):
    """One pass -> (per-cluster sums float64, counts int64, inertia[, labels int64]) (core.py:2200-2206)."""
    ds = _dataset(parts)
    Cd = _centers(C, ds)
    _check_method(method, accumulate, Cd.shape[0], ds.d)
    out = ds.assign(Cd, return_labels=return_labels, generic=(method == "generic"),
                    rule=label_rule and _check_rule(label_rule), approx=(method == "approx"),
                    cascade=(method == "cascade"))
    return out


assign = assign_mlx


def take_rows(parts, idx):
    """Gather global row indices from a list of slices -> float32 numpy array (core.py:132-143)."""
    ds = _dataset(parts)
    idx = np.asarray(idx, dtype=np.int64)
    out = np.empty((len(idx), ds.d), dtype=np.float32)
    off = 0
    for p in ds.parts:
        m = (idx >= off) & (idx < off + p.shape[0])
        if m.any():
            local = torch.from_numpy(idx[m] - off).to(p.device)
            out[m] = p.index_select(0, local).cpu().numpy()
        off += p.shape[0]
    return out


def kmeans_pp_init(parts, rows, k, rng, sample=None):
    """k-means++ seeding on a random subsample (core.py:153-192).

    The sample rows and the first center come from `rng` exactly as the reference draws them
    (core.py:170-181); the k-1 greedy rounds then run on the device (kmc_pp_init) with no host round trip."""
    ds = _dataset(parts)
    if sample is None:
        sample = min(200_000, max(20_000, 20 * k))
    idx = np.sort(rng.choice(rows, size=min(sample, rows), replace=False))
    S = _gather_rows(ds, idx)
    m, d = S.shape
    first = int(rng.integers(m))
    seeds = rng.integers(2**63 - 1, size=max(k - 1, 0)).astype(np.uint64)
    return pp_init_device(S, k, first, seeds).cpu().numpy()


def _gather_rows(ds, idx):
    """Rows idx (sorted global indices, all on this rank) gathered on the device -> (m, d) tensor."""
    outs = []
    off = 0
    for p in ds.parts:
        lo, hi = np.searchsorted(idx, [off, off + p.shape[0]])
        if hi > lo:
            outs.append(p.index_select(0, torch.from_numpy(idx[lo:hi] - off).to(p.device)))
        off += p.shape[0]
    return torch.cat(outs, 0).contiguous()


def pp_init_device(S, k, first, seeds):
    """kmc_pp_init on a device sample S (m, d) -> (k, d) CUDA tensor."""
    m, d = S.shape
    if k > m:
        raise ValueError(f"k={k} exceeds the {m} sample rows")
    L = _lib.load()
    wsb = int(L.kmc_pp_workspace_bytes(m, d, k))
    ws = torch.empty(max(wsb, 256), dtype=torch.uint8, device=S.device)
    seeds_d = torch.from_numpy(np.asarray(seeds, dtype=np.uint64).view(np.int64)).to(S.device)
    picks = torch.empty(k, dtype=torch.int64, device=S.device)
    C = torch.empty((k, d), dtype=torch.float32, device=S.device)
    _lib.call("kmc_pp_init", _ptr(S), m, d, k, int(first), _ptr(seeds_d) if k > 1 else None, _ptr(picks), _ptr(C),
              _ptr(ws), wsb, _stream())
    pp_init_device.last_picks = picks
    return C


def kmeans(parts, rows, k, max_iter, tol, seed, verbose=True):
    """The reference's synthetic driver (core.py:2247-2273, MLX backend branch) on the device."""
    import time
    ds = _dataset(parts)
    rng = np.random.default_rng(seed)
    C = kmeans_pp_init(ds, rows, k, rng)
    prev = None
    Cd = torch.from_numpy(C).to(ds.device)
    for it in range(1, max_iter + 1):
        t = time.perf_counter()
        newC, s = ds.step(Cd)
        newC = newC.clone()
        shift = float(torch.sqrt(((newC - Cd) ** 2).sum(1)).max())
        Cd = newC
        inertia = s["inertia"]
        if verbose:
            note = f"  ({s['n_empty']} empty clusters relocated)" if s["n_empty"] else ""
            print(f"iter {it:3d}  inertia {inertia:.6e}  max_center_shift {shift:.5f}  "
                  f"{time.perf_counter() - t:.3f}s{note}")
        if prev is not None and abs(prev - inertia) <= tol * prev:
            break
        prev = inertia
    inertia = ds.assign(Cd)[2]
    return Cd.cpu().numpy(), inertia
