/*
 * kmc.h -- C ABI of the B200 Lloyd-pass library (libkmc.so, sm_100a).
 *
 * Drop-in boundary for the hot path of kakollu/mlx-kmeans.  The reference has no C/FFI layer: its
 * boundary is three Python functions in mlx_kmeans/core.py, and each entry point below names the one
 * it replaces.  A ctypes binding (mlx_kmeans_b200/_lib.py) puts the same Python signatures back on top.
 *
 * Conventions
 *   - Every pointer marked (device) is a device pointer on the current CUDA device; (host) pointers are
 *     ordinary host memory.  `stream` is a cudaStream_t passed as void* (0 = legacy default stream).
 *   - Calls only enqueue work on `stream`; none synchronises, except kmc_stats_read which copies the
 *     statistics back and waits for them.
 *   - Every call returns KMC_OK (0) or an error code; nothing is thrown across the ABI.  The message of
 *     the last failure on the calling thread is kmc_last_error().
 *   - The library allocates nothing on its own for these calls: the caller passes device workspaces
 *     (256-byte aligned) of the sizes the *_workspace_bytes functions give.
 *
 * Numeric contract (the reference's float64 test oracle, tests/accuracy.py:31-51):
 *   label = the center with the smallest float64 distance sum_j ((double)x_j - (double)c_j)^2 (NumPy's
 *   pairwise summation order), lowest index on exact ties -- or, with KMC_PASS_LABEL32, the reference's
 *   float32 exact-mode rule (core.py:218-219, 263-274); best = the float32 distance to that center,
 *   each square and add rounded on its own; totals are exact and independent of summation order.
 */
#ifndef KMC_H
#define KMC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum kmc_status {
    KMC_OK = 0,
    KMC_ERR_INVALID = 1,      /* bad shape, null pointer, workspace too small (ValueError in Python) */
    KMC_ERR_CUDA = 2,         /* a CUDA call failed (RuntimeError in Python) */
    KMC_ERR_UNSUPPORTED = 3,  /* shape outside what the library handles (d > KMC_MAX_DIMS) */
};

#define KMC_MAX_DIMS 4096

/* Flags of kmc_pass. */
#define KMC_PASS_ACCUMULATE 1u   /* add into `totals` instead of overwriting them (data held in slices) */
#define KMC_PASS_GENERIC 2u      /* force the any-shape kernel (tests compare the specialised kernels to it) */
/* The float32 label rule of the reference's rows kernel (core.py:263-274, its exact-mode contract at
 * core.py:218-219): label = the center with the smallest float32 direct sum s = s + (x_j - c_j)^2 over j in
 * order, each subtraction, square and add rounded on its own (no fused multiply-add), strict < over centers in
 * index order (lowest index on ties).  Without it the label is the float64-optimal center (the numeric contract
 * below).  The two differ only where the float32 sums of two centers are within their rounding of each other. */
#define KMC_PASS_LABEL32 4u
/* exact=False (the reference's approximate assignment, core.py:859-1088 and 2036-2060), kmc_pass_split only:
 * x.c from one bf16 MMA per product (x and c rounded to bf16, float32 accumulation) and the smallest score's
 * center taken with no error window, so a row whose two best centers are within the bf16 rounding may get the
 * second.  Counts, sums and inertia are still exact for the labels given (read from the float32 rows). */
#define KMC_PASS_APPROX 8u
/* kmc_pass_elkan: (re)build the per-center bounds with a full tensor-core pass instead of using them. */
#define KMC_PASS_ELKAN_BUILD 16u

/* Device statistics of one Lloyd step, as kmc_finish leaves them (layout fixed, 64 bytes). */
typedef struct kmc_stats {
    double inertia;        /* sum of best over all rows, for the centers the pass started from */
    int64_t n_empty;       /* clusters that received no row */
    int64_t n_relocated;   /* clusters given a far row by the relocation rule */
    int64_t needs_reloc;   /* 1: clusters emptied and no candidate rows were given; C_new not written */
    int64_t flags;         /* 1 = non-finite data, centers or distance; 2 = kmc_exchange_sum timed out */
    int64_t rescored;      /* rows whose label was decided in float64 (diagnostic) */
    int64_t screened;      /* rows compared with every center (bounded passes: those whose bound failed) */
    int64_t reserved;
} kmc_stats;

/* ---------------------------------------------------------------- library */

int kmc_version(void);
const char *kmc_last_error(void);
/* Number of streaming multiprocessors of the current device (grid sizing of the caller's own work). */
int kmc_num_sms(void);
/* Row granularity of the pass kernels' fixed blocks for a dataset of n_total rows in all (slices and GPUs):
 * when every shard / slice starts at a global row that is a multiple of this, the totals are bit-identical
 * however the rows are split over slices and GPUs.  8192 below 64M rows, 20480 from there. */
int64_t kmc_row_block(int64_t n_total);

/* ---------------------------------------------------------------- workspace */

/* Bytes of device workspace kmc_pass, kmc_finish and kmc_totals_unpack need for d dims and k centers.
 * kmc_finish and kmc_totals_unpack read the constants kmc_pass left there, so a Lloyd step uses one
 * workspace throughout. */
size_t kmc_workspace_bytes(int d, int k);
/* Bytes of device workspace kmc_far_rows needs for `cand_rows` candidates (a separate buffer). */
size_t kmc_far_workspace_bytes(int64_t cand_rows);

/* ---------------------------------------------------------------- Lloyd step
 * Replaces core.py:2209-2242 `lloyd_step(parts, C)` and core.py:2200-2206 `assign_mlx(parts, C)`:
 *   kmc_colmax      once per dataset (the fixed-point grid of the totals),
 *   kmc_pass        per slice: nearest center + accumulation into totals,
 *   [ranks > 1: the caller sums totals over ranks, int64 sum -- exact, order-free]
 *   kmc_finish      center divide, empty-cluster relocation, still-empty rule, statistics.
 */

/* Per-column max |x| of X (n x d, device) into colmax (d uint32 float bits, device).  Accumulates
 * (atomic max) into colmax; zero it first with KMC_PASS_ACCUMULATE clear (flags & 1 == 0). */
int kmc_colmax(const float *X, int64_t n, int d, uint32_t *colmax, unsigned flags, void *stream);

/* One assignment pass over X (n x d, device) against C (k x d, device).
 * totals (device, k x (d+2) int64): per cluster [count, sum of best, sum of x_j ...] in fixed point.
 * labels (device, n int32) and best (device, n float32) are optional (NULL to skip).
 * colmax: the GLOBAL per-column maxima (all slices, all ranks); n_total: the GLOBAL row count.
 * Replaces core.py:2018-2197 `_gpu_pass`. */
int kmc_pass(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax, int64_t n_total,
             int64_t *totals, int32_t *labels, float *best, unsigned flags, void *workspace, size_t ws_bytes,
             void *stream);

/* Per-row bounds between Lloyd passes (the reference keeps per-centre bounds for high d, core.py:1690-2015;
 * here: Hamerly-style, one 32-bit word per row for the fused low-d kernel).  A caller buffer of
 * kmc_bounds_bytes(n, d, k) bytes per slice holds the drift of the centers, the centers of the last pass and
 * one word per row: a lower bound on the row's distance to every center but its label, with the label in its
 * low bits.  kmc_pass_bounded is kmc_pass (same totals, same labels) that reads and refreshes these words:
 * a row whose distance to its stored label is below its bound less the centers' drift since keeps its label
 * without being compared to the other centers.  The first pass after kmc_bounds_reset (or on a zeroed buffer)
 * compares every row and writes all words.  Centers may change arbitrarily between passes: the drift is
 * measured from the centers themselves.  Shapes outside the fused kernel (d > 8 or k above its limit) run
 * the plain pass and leave the buffer untouched.  No labels/best outputs (use kmc_pass for those). */
size_t kmc_bounds_bytes(int64_t n, int d, int k);
int kmc_bounds_reset(void *bounds, void *stream);
int kmc_pass_bounded(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax,
                     int64_t n_total, int64_t *totals, unsigned flags, void *bounds, size_t bounds_size,
                     void *workspace, size_t ws_bytes, void *stream);

/* Tensor-core pass for high d (the reference's tiles / tiles1 paths, core.py:289-377 and 675-844).  x.c is
 * computed on the tcgen05 tensor cores from bf16 hi/lo splits of x and c (three MMAs per product); a row whose
 * two best centers are closer than the proven error window is decided in float64, so labels, best, counts and
 * sums are those of kmc_pass; the inertia column sums each row's float64 distance (kmc_pass: the float32
 * `best`), the same to about 1e-7.  The rows are then grouped by label and summed per cluster.  The row split
 * is per dataset slice: kmc_split_bytes(n, d) bytes filled once by kmc_split_rows (bf16 copies of X, row
 * norms, and per-row scratch of the pass); the center split, kmc_csplit_bytes(d, k) bytes, is refilled by
 * every pass.  One call takes at most 2^32 - 1 rows.  Any d is accepted; it pays off from d = 32 up.
 * Arguments, outputs and errors otherwise as kmc_pass. */
size_t kmc_split_bytes(int64_t n, int d);
int kmc_split_rows(const float *X, int64_t n, int d, void *split, size_t split_bytes, void *stream);
size_t kmc_csplit_bytes(int d, int k);
int kmc_pass_split(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax,
                   int64_t n_total, int64_t *totals, int32_t *labels, float *best, unsigned flags, void *split,
                   size_t split_bytes, void *csplit, size_t csplit_bytes, void *workspace, size_t ws_bytes,
                   void *stream);

/* Per-center lower bounds between passes for the tensor-core shapes (Elkan): the reference's bounded high-d path
 * (core.py:1690-2015, engaged at core.py:2063-2084).  A caller buffer of kmc_elkan_bytes(n, d, k) bytes per slice
 * holds the centers the bounds refer to, their drift, and one float16 lower bound per (row, center), rounded toward
 * zero.  kmc_pass_elkan is kmc_pass_split (same arguments plus the bounds; the same labels, best and totals, bit for
 * bit) that, with KMC_PASS_ELKAN_BUILD, runs the full tensor-core pass and writes every bound, and without it runs
 * the bounded pass: each row's distance to its previous label is recomputed, every bound is lowered by its center's
 * drift since, and only the centers whose lowered bound does not exceed that distance (plus the decision window)
 * are visited; near ties go to the same float64 (or float32-rule) decision.  The labels of the previous pass on the
 * slice (kept in the split) are the starting guesses -- any labels are correct starting guesses, only the work
 * depends on them.  The number of visited (row, center) pairs is added to the statistics' `screened`; a caller
 * rebuilds (or drops) the bounds when it grows.  The first call on a split must build (any pass on the split leaves
 * the grouped row order the bounded pass walks).  k must be a multiple of 8; not with KMC_PASS_APPROX. */
size_t kmc_elkan_bytes(int64_t n, int d, int k);
int kmc_pass_elkan(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax, int64_t n_total,
                   int64_t *totals, int32_t *labels, float *best, unsigned flags, void *split, size_t split_bytes,
                   void *csplit, size_t csplit_bytes, void *elkan, size_t elkan_bytes, void *workspace,
                   size_t ws_bytes, void *stream);

/* The prefix-pruning cascade: replaces the reference's two-stage exact assignment `_cascade_nearest`
 * (core.py:1212-1260; stage kernels core.py:1107-1196, engaged at core.py:2085-2109).  The squared distance over a
 * subset of the columns is a lower bound on the full one, so a center whose prefix distance already exceeds the
 * row's distance to its previous label (widened by the decision window) cannot be its label.  Each row's threshold
 * comes from its previous label; the tensor-core pass over the prefix (the caller's m columns, highest variance
 * first: msplit = kmc_split_rows of those columns, kmc_split_bytes(n, m) bytes, filled once per slice; Cm = the
 * centers' same columns, k x m float32, device; mcsplit = kmc_csplit_bytes(m, k) bytes, refilled by every pass)
 * marks one bit per (row, center) whose rigorous lower bound is within it; the marked centers are then scored in
 * full and near ties go to the label rule's decision, so labels, best and totals are kmc_pass_split's, bit for
 * bit, whatever the prefix prunes.  cascade: kmc_cascade_bytes(n, k) bytes of caller memory per slice (the
 * thresholds and the survivor bits, rewritten by every call).  The previous pass's labels on the split are the
 * starting guesses, so a kmc_pass_split (or kmc_pass_elkan) must have run on the split first.  The number of
 * survivors is added to the statistics' `screened`; the reference stops offering the cascade once more than 15% of
 * the (row, center) pairs survive (core.py:491, 2155-2156).  k a multiple of 8; exact passes only (no
 * KMC_PASS_APPROX or KMC_PASS_ELKAN_BUILD). */
size_t kmc_cascade_bytes(int64_t n, int k);
int kmc_pass_cascade(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax,
                     int64_t n_total, int64_t *totals, int32_t *labels, float *best, unsigned flags, void *split,
                     size_t split_bytes, void *csplit, size_t csplit_bytes, const float *Cm, int m, void *msplit,
                     size_t msplit_bytes, void *mcsplit, size_t mcsplit_bytes, void *cascade, size_t cascade_bytes,
                     void *workspace, size_t ws_bytes, void *stream);

/* The tensor-core pass's raw scores, for auditing its error window (no counterpart in the reference): out
 * (device, n x k float32) = x.c for every row of the split (kmc_split_rows) and every center, exactly as the
 * tcgen05 MMAs of kmc_pass_split accumulate them (xh.ch + xh.cl + xl.ch in float32), before any decision.
 * error (device, one int) is set to 1 if the kernel gave up on a barrier (out is then incomplete). */
int kmc_tc_dot(const float *C, int64_t n, int d, int k, void *split, size_t split_bytes, void *csplit,
               size_t csplit_bytes, float *out, int *error, void *stream);

/* All-reduce of the totals over the GPUs of one node through peer memory (NVLink), one kernel per step: no
 * counterpart in the reference (single device); it replaces an NCCL all-reduce of the int64 totals.  Set-up once
 * per (process group, k): each rank kmc_exchange_alloc's a kmc_exchange_bytes(k, d) buffer (device memory the
 * library allocates, zeroed) and gets its 64-byte CUDA IPC handle; the handles are exchanged (any host
 * collective); each rank kmc_exchange_open's its peers' buffers.  `peers` is a device array of the world buffer
 * addresses (own included, at index rank).  Per pass, after the pass on every local slice: kmc_exchange_sum with
 * a step number that every rank increments the same way (0, 1, 2, ...); on return (stream order) totals hold the
 * sum over ranks.  A peer that does not arrive within KMC_EXCHANGE_TIMEOUT_MS milliseconds (an environment variable read on
 * every call; 30 s when unset) sets stats flag 2 (read by kmc_finish) and the totals keep this rank's own values.  All ranks
 * must call it the same number of times (kmc_exchange_sum and kmc_exchange_finish share the step count).
 * kmc_exchange_close(ptr, own) unmaps a peer's buffer (own = 0) or frees one's own (own = 1): only once every
 * rank is done with the buffers, since a peer may still be reading one after its owner's call returned. */
size_t kmc_exchange_bytes(int k, int d);
int kmc_exchange_alloc(size_t bytes, void **ptr, void *handle);
int kmc_exchange_open(const void *handle, void **ptr);
int kmc_exchange_close(void *ptr, int own);
int kmc_exchange_sum(int64_t *totals, int k, int d, const uint64_t *peers, int world, int rank, uint64_t step,
                     void *workspace, size_t ws_bytes, void *stream);

/* kmc_exchange_sum then kmc_finish without relocation candidates, in one launch (the step's tail when rows are
 * sharded over GPUs): the same exchange protocol and step count (`step` as for kmc_exchange_sum; a timeout sets
 * stats flag 2 and leaves this rank's own totals), then the divide, empties and statistics of kmc_finish.  Wide
 * totals (k (d + 2) >= 16384 values) are exchanged by a multi-CTA launch of their own first, as kmc_exchange_sum
 * does for them. */
int kmc_exchange_finish(int64_t *totals, int k, int d, const uint64_t *peers, int world, int rank, uint64_t step,
                        float *C_new, kmc_stats *stats, void *workspace, size_t ws_bytes, void *stream);

/* kmc_pass without a caller workspace.  No counterpart in the reference: it exists for callers that cannot
 * allocate device memory -- a host runtime that owns every device allocation through its own pool, or a
 * phase of a program in which calling an allocator is not allowed -- and so cannot provide the workspace
 * kmc_pass asks for.  Its scratch is a file-scope device array of KMC_STATIC_SCRATCH_BYTES, one copy in every
 * CUDA context that loads the library, held until the process exits; shapes needing more
 * (kmc_workspace_bytes(d, k) above it, e.g. k above ~4000 at d = 64) are refused with KMC_ERR_UNSUPPORTED.  It
 * calls no allocator.  The first call in a context looks up that context's copy of the array
 * (cudaGetSymbolAddress) and caches it; make that first call before any stream capture.  All calls in a
 * context share the one array and it keeps the last call's contents: calls whose work overlaps on the GPU
 * race, so issue them in one stream (or order them).  The pass clears what must start at zero itself (totals
 * and counters, unless KMC_PASS_ACCUMULATE).  The array also holds the fixed-point grid of the totals, so
 * finish the step with kmc_finish or kmc_totals_unpack given workspace = NULL: they then read the same array,
 * and must follow the kmc_pass_static that made the totals in stream order, before the next one.
 * Arguments, outputs and errors as kmc_pass. */
#define KMC_STATIC_SCRATCH_BYTES (64 * 1024)
int kmc_pass_static(const float *X, int64_t n, int d, const float *C, int k, const uint32_t *colmax,
                    int64_t n_total, int64_t *totals, int32_t *labels, float *best, unsigned flags, void *stream);

/* Local relocation candidates: the `cand_rows` rows of X with the largest best (lower row index on
 * ties), as records of (d + 4) 32-bit words [best, global row lo, global row hi, label, x_0 .. x_{d-1}],
 * farthest first, padded with best = -1.  row0 = global index of local row 0.
 * Replaces the far-row selection of core.py:2225-2230. */
int kmc_far_rows(const float *X, int64_t n, int d, const int32_t *labels, const float *best, int64_t row0,
                 int64_t cand_rows, uint32_t *cands, void *workspace, size_t ws_bytes, void *stream);

/* Finish a Lloyd step from the (global) totals, on the workspace of the kmc_pass that made them (its
 * fixed-point grid lives there; workspace = NULL: the static scratch of kmc_pass_static, ws_bytes ignored): relocation of empty clusters to the farthest rows (candidate lists of
 * `ranks` ranks, each from kmc_far_rows, concatenated; NULL when none were gathered), then
 * C_new = sums / counts rounded to float32, a still-empty cluster takes the largest cluster's center,
 * and kmc_stats.  totals are updated in place by the relocation.  C_new (device, k x d).
 * Replaces core.py:2223-2241. */
int kmc_finish(int64_t *totals, int k, int d, const uint32_t *cands, int64_t cand_rows, int ranks, float *C_new,
               kmc_stats *stats, void *workspace, size_t ws_bytes, void *stream);

/* ---------------------------------------------------------------- Lloyd loop on the device
 * Replaces the loop of estimator.py:132-150 (`_one_run`: step, then stop once |prev - inertia| <= tol * prev)
 * with no host round trip per step.  The loop's record (kmc_loop, device, 64 bytes) holds the stopping rule's
 * state; kmc_loop_init sets it.  kmc_lloyd enqueues `steps` Lloyd steps (kmc_pass or kmc_pass_bounded when
 * `bounds` is given, then kmc_finish) on one slice, reading the centers from C0 and C1 in turn (step i reads
 * C_{i % 2} and writes C_{(i + 1) % 2}); after each step the finish applies the stopping rule, and once the loop
 * has stopped the kernels of the steps still queued return at once.  One kmc_stats_read-style copy of the record
 * at the end says how it stopped: converged, max_steps reached, non-finite (flags), or a step that emptied
 * clusters (kmc_finish without candidates leaves its centers unwritten): the caller then relocates that step with
 * kmc_far_rows + kmc_finish, continues the record with kmc_loop_init(steps_done + 1, that step's inertia) and
 * calls kmc_lloyd again.  Single GPU, one slice; shapes on the tensor-core pass use the step-by-step calls.
 * The final centers are in C_{steps % 2} of the record's `steps` counted from this call's start. */
typedef struct kmc_loop {
    double prev_inertia;   /* inertia of the last step run */
    double tol;
    int64_t steps;         /* steps completed */
    int64_t max_steps;
    int64_t state;         /* 0 running, 1 converged, 2 a step needs relocation, 3 non-finite, 4 max_steps ran */
    int64_t have_prev;
    int64_t reserved[2];
} kmc_loop;
int kmc_loop_init(kmc_loop *loop, double tol, int64_t max_steps, int64_t steps_done, double prev_inertia,
                  int have_prev, void *stream);
int kmc_lloyd(const float *X, int64_t n, int d, float *C0, float *C1, int k, const uint32_t *colmax, int64_t n_total,
              int64_t *totals, unsigned flags, void *bounds, size_t bounds_size, kmc_stats *stats, kmc_loop *loop,
              int steps, void *workspace, size_t ws_bytes, void *stream);

/* Copy the device statistics to the host and wait for them (the one synchronising call). */
int kmc_stats_read(const kmc_stats *stats_dev, kmc_stats *stats_host, void *stream);

/* Convert totals to float64 sums (k x d), int64 counts (k) and the inertia (all device), as
 * core.py:2200-2206 `assign_mlx` returns them; same workspace as the kmc_pass that made the totals
 * (workspace = NULL: the static scratch of kmc_pass_static, ws_bytes ignored). */
int kmc_totals_unpack(const int64_t *totals, int k, int d, double *sums, int64_t *counts, double *inertia,
                      void *workspace, size_t ws_bytes, void *stream);

/* The float64 distance labels are decided by: out[i] = D64(X[i], C[i]) for m row pairs (X, C: device,
 * m x d float32; out: device, m float64) -- (double)x_j - (double)c_j, squared, summed in NumPy's pairwise
 * order, as the reference's accuracy check computes it (tests/accuracy.py:31-51).  One warp per pair, the
 * same arithmetic the passes re-score near ties with; for auditing labels. */
int kmc_d64(const float *X, const float *C, int d, int64_t m, double *out, void *stream);

/* ---------------------------------------------------------------- k-means++
 * Replaces core.py:153-192 `kmeans_pp_init(parts, rows, k, rng, sample)` after the host has drawn the
 * sample rows and gathered them into S (m x d, device): greedy k-means++ with 2 + floor(ln k) candidates
 * per round by the Gumbel-max trick (Philox4x32-10 with key seeds[r]), the candidate lowering the total
 * d2 the most kept.  first = sample row of the first center; seeds (device, k-1 uint64);
 * picks (device, k int64) = chosen sample rows; C_out (device, k x d). */
size_t kmc_pp_workspace_bytes(int64_t m, int d, int k);
int kmc_pp_init(const float *S, int64_t m, int d, int k, int64_t first, const uint64_t *seeds, int64_t *picks,
                float *C_out, void *workspace, size_t ws_bytes, void *stream);

/* ---------------------------------------------------------------- data generation
 * Synthetic inputs of the benchmark configurations, generated on the device from the global row index
 * (Philox4x32-10, key = seed), so any split of rows over GPUs yields the same rows.  Replaces
 * core.py:111-129 `make_data_mlx` (which draws from a splitmix64 hash instead).
 *   kind 0: uniform [0, 1)                           (params unused)
 *   kind 1: Gaussian mixture: component uniform over `ncomp`, x = means[c] + sds[c] * N(0,1),
 *           means/sds (device, ncomp x d); clipped to [lo, hi] when lo < hi
 *   kind 2: kind 1 then each row scaled to unit L2 norm (float64 norm)
 */
int kmc_gen(int kind, float *X, int64_t n, int d, int64_t row0, uint64_t seed, const float *means,
            const float *sds, int ncomp, float lo, float hi, void *stream);

/* Column sums of X and of X^2 in exact fixed point (grid from colmax, n_total), accumulated into
 * sums (device, 2 x d int64); and the in-place standardisation X = (X - mean) / std with mean/std
 * (device, 2 x d float64) derived from those sums.  Used by the 96M-row configuration (standardised
 * per column in float64, README.md:90 of the reference). */
int kmc_colsums(const float *X, int64_t n, int d, const uint32_t *colmax, int64_t n_total, int64_t *sums,
                void *stream);
int kmc_standardize(float *X, int64_t n, int d, const int64_t *sums, const uint32_t *colmax, int64_t n_total,
                    double *mean_std, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* KMC_H */
