/*
 * kmc_oracle.c -- CPU restatement of the reference's Lloyd-pass arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the CUDA library, the Python package) links,
 * loads or calls this file; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg do,
 * and only as the checker.
 *
 * What it restates (reference = kakollu/mlx-kmeans):
 *   - kmo_d64: the float64 distance of the reference's own test oracle, tests/accuracy.py:31-51
 *     (`((x[rows] - C64[cols]) ** 2).sum(1)`): x and c widened to double, difference and square
 *     rounded separately, then summed in NumPy's pairwise order (0.0 + pairwise(all terms)), the
 *     order NumPy 2.x uses for a reduction over a contiguous last axis.  Pinned bit-for-bit against
 *     NumPy in tests/test_oracle.py.
 *   - kmo_assign: label = argmin of kmo_d64 over centers, lowest index on exact ties
 *     (tests/accuracy.py:48-49, core.py:218-219 "lowest index on ties").
 *   - kmo_assign_rule(rule = 1): the reference's exact-mode label rule itself, its rows kernel
 *     (core.py:263-274, contract at core.py:218-219): for each center in index order the float32 direct
 *     sum s = s + (x_j - c_j)^2 (kmo_best32: each subtraction, square and add rounded on its own), and
 *     the center is taken when s < best (strict: lowest index on ties).  Pinned against a NumPy
 *     restatement of that loop (tests/golden/make_golden.py: rows_kernel_labels).
 *   - kmo_best32: the per-row float32 distance to the assigned center that the reference keeps as
 *     `best` (core.py:248-257: s += (x_j - c_j)^2 in order), here with the square and the add rounded
 *     separately (no fused multiply-add), so the CUDA kernels can reproduce it bit for bit.
 *   - kmo_lloyd_step: core.py:2209-2242 -- float64 sums and counts, inertia = sum of best,
 *     empty-cluster relocation (farthest `best` first, lower row index on ties, core.py:2224-2236),
 *     C_new = sums / counts rounded to float32, a still-empty cluster takes the largest cluster's
 *     center (core.py:2241).
 *   - kmo_pp_init: greedy k-means++ of core.py:153-192 (2 + floor(ln k) candidates per round drawn by
 *     the Gumbel-max trick over d2, the candidate lowering the total d2 the most is kept, ties to the
 *     first row / first trial), with the random numbers drawn from Philox4x32-10 (Salmon et al.,
 *     SC'11) instead of the reference's splitmix64 hash, as the CUDA build does.
 *
 * Compile with -ffp-contract=off: every float operation here is rounded on its own.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ distances */

/* NumPy's pairwise summation (numpy/_core/src/umath/loops_utils.h.src, pairwise_sum): fewer than 8
 * terms are added in order; up to 128 terms use 8 running partials combined as
 * ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) followed by the tail in order; longer runs split at
 * n/2 rounded down to a multiple of 8. */
static double pairwise(const double *a, int64_t n) {
    if (n < 8) {
        double r = 0.0;
        for (int64_t i = 0; i < n; i++) r += a[i];
        return r;
    } else if (n <= 128) {
        double r[8];
        int64_t i;
        for (int j = 0; j < 8; j++) r[j] = a[j];
        for (i = 8; i < n - (n % 8); i += 8)
            for (int j = 0; j < 8; j++) r[j] += a[i + j];
        double res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
        for (; i < n; i++) res += a[i];
        return res;
    } else {
        int64_t n2 = n / 2;
        n2 -= n2 % 8;
        return pairwise(a, n2) + pairwise(a + n2, n - n2);
    }
}

double kmo_d64(const float *x, const float *c, int d) {
    double t[4096];
    double *buf = d <= 4096 ? t : (double *)malloc(sizeof(double) * (size_t)d);
    for (int j = 0; j < d; j++) {
        double q = (double)x[j] - (double)c[j];
        buf[j] = q * q;
    }
    double r = 0.0 + pairwise(buf, d);
    if (buf != t) free(buf);
    return r;
}

float kmo_best32(const float *x, const float *c, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; j++) {
        float q = x[j] - c[j];
        float q2 = q * q;
        s = s + q2;
    }
    return s;
}

/* ------------------------------------------------------------------ assignment */

typedef struct {
    const float *X, *C;
    int64_t r0, r1;
    int d, k;
    int64_t *labels;
    double *d64;
    float *best32;
    int rule;
} assign_job;

static void *assign_worker(void *p) {
    assign_job *j = (assign_job *)p;
    for (int64_t i = j->r0; i < j->r1; i++) {
        const float *x = j->X + i * (int64_t)j->d;
        int64_t bl = 0;
        if (j->rule == 1) {
            float bs = INFINITY;
            for (int c = 0; c < j->k; c++) {
                float s = kmo_best32(x, j->C + (int64_t)c * j->d, j->d);
                if (s < bs) { bs = s; bl = c; }      /* strict <: lowest index on ties */
            }
        } else {
            double bd = INFINITY;
            for (int c = 0; c < j->k; c++) {
                double v = kmo_d64(x, j->C + (int64_t)c * j->d, j->d);
                if (v < bd) { bd = v; bl = c; }      /* strict <: lowest index on ties */
            }
        }
        if (j->labels) j->labels[i] = bl;
        if (j->d64) j->d64[i] = kmo_d64(x, j->C + bl * (int64_t)j->d, j->d);
        if (j->best32) j->best32[i] = kmo_best32(x, j->C + bl * (int64_t)j->d, j->d);
    }
    return NULL;
}

/* rule 0: the float64 distance (tests/accuracy.py:31-51); rule 1: the float32 direct sum (core.py:263-274).
 * d64 (optional) receives each row's float64 distance to its label, best32 (optional) its float32 one. */
void kmo_assign_rule(const float *X, int64_t n, int d, const float *C, int k, int64_t *labels, double *d64,
                     float *best32, int nthreads, int rule) {
    if (nthreads < 1) nthreads = 1;
    if (nthreads > 256) nthreads = 256;
    if (n < 4096) nthreads = 1;
    pthread_t th[256];
    assign_job jobs[256];
    for (int t = 0; t < nthreads; t++) {
        jobs[t] = (assign_job){X, C, n * t / nthreads, n * (t + 1) / nthreads, d, k, labels, d64, best32, rule};
        if (nthreads > 1) pthread_create(&th[t], NULL, assign_worker, &jobs[t]);
        else assign_worker(&jobs[t]);
    }
    if (nthreads > 1)
        for (int t = 0; t < nthreads; t++) pthread_join(th[t], NULL);
}

void kmo_assign(const float *X, int64_t n, int d, const float *C, int k, int64_t *labels, double *d64,
                float *best32, int nthreads) {
    kmo_assign_rule(X, n, d, C, k, labels, d64, best32, nthreads, 0);
}

/* ------------------------------------------------------------------ Lloyd step */

/* Order of far rows: larger best first, lower row index on ties (core.py:2227-2229). */
static const float *g_best;
static int far_cmp(const void *a, const void *b) {
    int64_t i = *(const int64_t *)a, j = *(const int64_t *)b;
    float bi = g_best[i], bj = g_best[j];
    if (bi > bj) return -1;
    if (bi < bj) return 1;
    return i < j ? -1 : (i > j);
}

/* Sums, counts and inertia for given labels and best (core.py:2223; the reference sums in float64 on
 * the host).  sums k*d, counts k. */
void kmo_accumulate(const float *X, int64_t n, int d, int k, const int64_t *labels, const float *best32,
                    double *sums, int64_t *counts, double *inertia) {
    memset(sums, 0, sizeof(double) * (size_t)k * d);
    memset(counts, 0, sizeof(int64_t) * (size_t)k);
    double in = 0.0;
    for (int64_t i = 0; i < n; i++) {
        int64_t l = labels[i];
        counts[l]++;
        for (int j = 0; j < d; j++) sums[l * d + j] += (double)X[i * d + j];
        in += (double)best32[i];
    }
    *inertia = in;
}

/* core.py:2209-2242 for precomputed labels/best.  Returns n_empty; writes C_new (k*d float32) and the
 * relocated (empty cluster, row) pairs into reloc (2*n_empty int64, may be NULL). */
int kmo_finish(const float *X, int64_t n, int d, const float *C, int k, const int64_t *labels,
               const float *best32, float *C_new, double *inertia, int64_t *reloc) {
    double *sums = (double *)malloc(sizeof(double) * (size_t)k * d);
    int64_t *counts = (int64_t *)malloc(sizeof(int64_t) * (size_t)k);
    kmo_accumulate(X, n, d, k, labels, best32, sums, counts, inertia);
    int n_empty = 0;
    for (int c = 0; c < k; c++) n_empty += counts[c] == 0;
    if (n_empty) {
        float mx = 0.0f;
        for (int64_t i = 0; i < n; i++) mx = best32[i] > mx ? best32[i] : mx;
        if (mx > 0.0f) {
            int64_t *order = (int64_t *)malloc(sizeof(int64_t) * (size_t)n);
            for (int64_t i = 0; i < n; i++) order[i] = i;
            g_best = best32;
            qsort(order, (size_t)n, sizeof(int64_t), far_cmp);
            int64_t *empty = (int64_t *)malloc(sizeof(int64_t) * (size_t)n_empty);
            int ne = 0;
            for (int c = 0; c < k; c++) if (counts[c] == 0) empty[ne++] = c;   /* fixed before any move */
            int e = 0;
            for (; e < n_empty && e < n; e++) {
                int64_t c = empty[e];
                int64_t f = order[e];
                int64_t old = labels[f];
                for (int j = 0; j < d; j++) {
                    sums[old * d + j] -= (double)X[f * d + j];
                    sums[c * d + j] = (double)X[f * d + j];
                }
                counts[old] -= 1;
                counts[c] = 1;
                if (reloc) { reloc[2 * e] = c; reloc[2 * e + 1] = f; }
            }
            free(empty);
            free(order);
        }
    }
    int64_t big = 0;
    for (int c = 1; c < k; c++) if (counts[c] > counts[big]) big = c;   /* np.argmax: first maximum */
    for (int c = 0; c < k; c++)
        if (counts[c] > 0)
            for (int j = 0; j < d; j++) C_new[(int64_t)c * d + j] = (float)(sums[(int64_t)c * d + j] / (double)counts[c]);
    for (int c = 0; c < k; c++)
        if (counts[c] <= 0)
            for (int j = 0; j < d; j++) C_new[(int64_t)c * d + j] = C_new[big * d + j];
    (void)C;
    free(sums);
    free(counts);
    return n_empty;
}

/* ------------------------------------------------------------------ Philox4x32-10 */

/* Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11: ten rounds of
 * two 32x32->64 multiplies on a 4-word counter with a Weyl-sequence key schedule. */
#define PHILOX_M0 0xD2511F53u
#define PHILOX_M1 0xCD9E8D57u
#define PHILOX_W0 0x9E3779B9u
#define PHILOX_W1 0xBB67AE85u

void kmo_philox(const uint32_t ctr_in[4], const uint32_t key_in[2], uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)PHILOX_M0 * c0, p1 = (uint64_t)PHILOX_M1 * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        k0 += PHILOX_W0; k1 += PHILOX_W1;
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Natural log of a double in (0, inf) from the definition log(m * 2^e) = e ln2 + 2 atanh(s),
 * s = (m - 1) / (m + 1), m in [sqrt(1/2), sqrt(2)), with the atanh series summed to 1e-17 relative.
 * Written with plain IEEE operations only so the CUDA build (kmc_log in csrc/common.cuh) gets the same
 * bits; accuracy is ~1 ulp, ample for drawing a sample. */
double kmo_log(double v) {
    int e = 0;
    double m = frexp(v, &e);                 /* v = m 2^e, m in [0.5, 1) */
    if (m < 0.70710678118654752440) { m = m * 2.0; e -= 1; }
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double term = s, sum = 0.0;
    for (int i = 0; i < 40; i++) {          /* |s| < 0.1716 -> s^(2i+1)/(2i+1) < 1e-17 by i = 11 */
        sum = sum + term / (double)(2 * i + 1);
        term = term * s2;
    }
    return (double)e * 0.69314718055994530942 + 2.0 * sum;
}

/* Uniform in (0, 1) with 53 random bits from one Philox block (words 0,1). */
static double philox_u01(uint64_t key, uint64_t row, uint32_t trial) {
    uint32_t ctr[4] = {(uint32_t)row, (uint32_t)(row >> 32), trial, 0x6B6D7070u /* "kmpp" */};
    uint32_t kk[2] = {(uint32_t)key, (uint32_t)(key >> 32)};
    uint32_t o[4];
    kmo_philox(ctr, kk, o);
    uint64_t b = ((uint64_t)o[0] << 32 | o[1]) >> 11;
    return ((double)b + 0.5) * (1.0 / 9007199254740992.0);
}

/* Gumbel-max key of core.py:86-88, written as the ratio it orders by:
 *   argmax log(d2) - log(-log u)  ==  argmax d2 / (-log u). */
double kmo_pp_key(float d2, uint64_t key, uint64_t row, uint32_t trial) {
    double u = philox_u01(key, row, trial);
    double ex = -kmo_log(u);
    double dd = (double)(d2 > 1e-30f ? d2 : 1e-30f);
    return dd / ex;
}

static int64_t ceil_log2_u(double v) {   /* smallest e with v <= 2^e, v > 0 */
    int e = 0;
    double m = frexp(v, &e);
    return m == 0.5 ? e - 1 : e;
}

/* The fixed-point scale the k-means++ trial totals use: 2^sh * max_d2 * m < 2^62, so the sum of m
 * quantised values is exact in int64 and independent of summation order. */
int kmo_pp_shift(float max_d2, int64_t m) {
    if (!(max_d2 > 0.0f)) return 0;
    int64_t lm = ceil_log2_u((double)m);
    int64_t lv = ceil_log2_u((double)max_d2);
    int64_t sh = 61 - lm - lv;
    if (sh > 1000) sh = 1000;
    if (sh < -1000) sh = -1000;
    return (int)sh;
}

int64_t kmo_quantize(float v, int sh) {
    return (int64_t)llrint(ldexp((double)v, sh));
}

/* Greedy k-means++ over the sample S (m x d): core.py:153-192 with Philox keys.  `first` is the
 * sample row of the first center (core.py:177), seeds[r] the key of round r+1 (core.py:181).
 * picks (k) receives sample-row indices; C_out (k x d) the centers. */
void kmo_pp_init(const float *S, int64_t m, int d, int k, int64_t first, const uint64_t *seeds, int64_t *picks,
                 float *C_out) {
    int trials = k > 1 ? 2 + (int)floor(log((double)k)) : 1;
    float *d2 = (float *)malloc(sizeof(float) * (size_t)m);
    float *mins = (float *)malloc(sizeof(float) * (size_t)m * trials);
    int64_t *cand = (int64_t *)malloc(sizeof(int64_t) * trials);
    int64_t *tot = (int64_t *)malloc(sizeof(int64_t) * trials);
    picks[0] = first;
    float mx = 0.0f;
    for (int64_t i = 0; i < m; i++) {
        d2[i] = kmo_best32(S + i * d, S + first * d, d);
        mx = d2[i] > mx ? d2[i] : mx;
    }
    int sh = kmo_pp_shift(mx, m);
    for (int r = 1; r < k; r++) {
        for (int t = 0; t < trials; t++) {
            double bk = -1.0;
            int64_t bi = 0;
            for (int64_t i = 0; i < m; i++) {
                double kv = kmo_pp_key(d2[i], seeds[r - 1], (uint64_t)i, (uint32_t)t);
                if (kv > bk) { bk = kv; bi = i; }       /* first row on ties */
            }
            cand[t] = bi;
            tot[t] = 0;
        }
        for (int64_t i = 0; i < m; i++)
            for (int t = 0; t < trials; t++) {
                float s = kmo_best32(S + i * d, S + cand[t] * d, d);
                float v = d2[i] < s ? d2[i] : s;
                mins[i * trials + t] = v;
                tot[t] += kmo_quantize(v, sh);
            }
        int bt = 0;
        for (int t = 1; t < trials; t++) if (tot[t] < tot[bt]) bt = t;   /* argmin: first trial on ties */
        for (int64_t i = 0; i < m; i++) d2[i] = mins[i * trials + bt];
        picks[r] = cand[bt];
    }
    for (int c = 0; c < k; c++) memcpy(C_out + (int64_t)c * d, S + picks[c] * d, sizeof(float) * (size_t)d);
    free(d2); free(mins); free(cand); free(tot);
}
