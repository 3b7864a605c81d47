// common.cuh -- device helpers shared by the kmc kernels (sm_100a).
//
// Numeric contract of every pass (mirrors the reference's, kakollu/mlx-kmeans):
//   label(x)  = argmin_c D64(x, c), lowest index on exact ties, where D64 is the float64 distance of
//               the reference's test oracle (tests/accuracy.py:31-51): (double)x_j - (double)c_j,
//               squared, summed in NumPy's pairwise order.  A float32 screen picks the label and only
//               rows whose two best screen scores lie inside a proven error window are re-scored with
//               D64, so the screen never decides a label it cannot prove.
//   best(x)   = float32 distance to the chosen center, s = s + (x_j - c_j)^2 in order with every
//               operation rounded on its own (core.py:248-257 keeps the same quantity as `best`).
//   totals    = per cluster [count, sum of best, sum of x_j ...] (core.py:236-237 layout), held as
//               exact int64 fixed point: every value is rounded once to a per-column power-of-two grid
//               and the integers are summed, so totals do not depend on summation order, thread
//               schedule, or how rows are split across blocks and GPUs.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace kmc {

// Programmatic dependent launch: a kernel launched with launch_pdl may be scheduled while the kernel before it in
// the stream is still finishing; it runs this first, which returns once that kernel has completed and its memory
// writes are visible (at once when it was launched the ordinary way), so nothing the kernel does changes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel of the stream be scheduled now (its pdl_wait still waits for this kernel to complete).
__device__ __forceinline__ void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

constexpr int kMaxDims = 4096;     // largest d the pass kernels accept

// Per-pass constants, computed on device by k_prepare (no host round trip).
struct Prep {
    double inv_scale_i;     // 2^-si
    double scale_i;         // 2^si: inertia fixed point
    float cmax2;            // max_c |c|^2 (float32, rounded up)
    float win_coef;         // screen window = win_coef * (|x|^2 + cmax2) + win_abs
    float win_abs;
    int si;
    int flags;              // kFlag* below
    int bvalid;             // bounded passes: the per-row bounds were written by an earlier pass
    float bcum_lo, bcum_up; // bounded passes: total center drift so far, rounded down / up
    int rule;               // label rule: 0 = float64 distance (NumPy pairwise), 1 = float32 direct sum
    int skip;               // a device Lloyd loop has stopped: the pass and the finish of this step do nothing
};

// State of a Lloyd loop run on the device (kmc_lloyd; the public kmc_loop, 64 bytes).  k_prepare reads `state` to
// skip the steps after the loop stopped; k_finish applies the reference's stopping rule after every step
// (estimator.py:132-150: stop once |prev - inertia| <= tol * prev) and updates the record.
struct LoopState {
    double prev_inertia;    // inertia of the last step run (the tol test compares the next one with it)
    double tol;
    long long steps;        // steps completed (this loop record)
    long long max_steps;
    long long state;        // kLoop* below
    long long have_prev;    // prev_inertia is set
    long long reserved[2];
};
enum : long long {
    kLoopRunning = 0,
    kLoopConverged = 1,     // the tol test held after the last step
    kLoopRelocate = 2,      // the last step emptied clusters: its centers were not written (the host relocates)
    kLoopNonFinite = 3,     // non-finite data, centers or distance
    kLoopMaxSteps = 4,      // max_steps steps ran
};

enum : int {
    kFlagNonFinite = 1,     // data or centers hold NaN / inf, or a distance overflowed float32
    kFlagExchange = 2,      // the peer-memory all-reduce of the totals timed out waiting for a peer
};

// Device statistics written by the finish kernel; read by the host once per pass.
struct Stats {
    double inertia;         // sum of best over all rows (of the centers the pass started from)
    int64_t n_empty;        // clusters with no rows after the pass (before relocation)
    int64_t n_relocated;    // clusters given a far row by the relocation rule
    int64_t needs_reloc;    // 1: empties exist and the finish had no candidate rows -> centers not written
    int64_t flags;          // kFlag*
    int64_t rescored;       // rows re-scored in float64 by the pass kernels (diagnostic)
    int64_t screened;       // rows compared with every center (bounded passes: the rows whose bound failed)
    int64_t pad;
};

// ---------------------------------------------------------------- fixed point

// smallest e with |v| <= 2^e (v finite, > 0)
__host__ __device__ inline int ceil_log2(double v) {
    int e;
    double m = frexp(v, &e);
    return m == 0.5 ? e - 1 : e;
}

// The grid a column is summed on: |v| <= absmax and n rows -> sum of n quantised values < 2^61.
__host__ __device__ inline int column_shift(float absmax, int64_t n_total) {
    double m = absmax > 0.0f ? (double)absmax : 1.1754943508222875e-38;   // FLT_MIN
    int L = ceil_log2((double)(n_total > 0 ? n_total : 1));
    int s = 61 - L - ceil_log2(m);
    return s > 1000 ? 1000 : (s < -1000 ? -1000 : s);
}

__device__ __forceinline__ long long quantize(float v, double scale) {
    return __double2ll_rn(__dmul_rn((double)v, scale));
}

// ---------------------------------------------------------------- distances

// float32 distance with every operation rounded separately (no contraction): the `best` value.
__device__ __forceinline__ float best32_term(float s, float x, float c) {
    float q = __fsub_rn(x, c);
    return __fadd_rn(s, __fmul_rn(q, q));
}

// The float32 direct sum of the reference's rows kernel (core.py:263-274): s = s + (x_j - c_j)^2 over j in
// order, each operation rounded on its own -- the distance the float32 label rule takes the argmin of.
__device__ __forceinline__ float best32(const float* x, const float* c, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; j++) s = best32_term(s, x[j], c[j]);
    return s;
}

// Extra width of a screen window under the float32 label rule.  The direct sum of d terms is B = D (1 + theta),
// |theta| <= gamma_{d+2} (a subtraction, a square and at most d - 1 additions of nonnegative terms per term), so a
// center c beats the exact nearest l under that rule only if D_c - D_l <= theta (D_c + D_l), i.e. its half
// distance exceeds l's by at most theta / (1 - theta) D_l.  With D_l <= 2 (|x|^2 + max|c|^2) (the low-d and
// CUDA-core screens' unit) or D_l <= (|x| + max|c|)^2 (the tensor-core window's), a coefficient of 2.5 (d + 3) u
// covers 2 theta / (1 - theta) for every d <= 4096 (u = 2^-24).
__host__ __device__ inline double rule32_coef(int d) { return 2.5 * (d + 3) / 16777216.0; }

// NumPy's pairwise sum of the float64 terms t_j = ((double)x_j - (double)c_j)^2, j in [lo, lo + n).
// Fewer than 8 terms: in order; up to 128: eight running partials + tail; longer: split at n/2 rounded
// down to a multiple of 8 (the same tree NumPy builds for a reduction over a contiguous axis).
__device__ __forceinline__ double d64_term(const float* x, const float* c, int j) {
    double q = __dsub_rn((double)x[j], (double)c[j]);
    return __dmul_rn(q, q);
}

__device__ inline double d64_leaf(const float* x, const float* c, int lo, int n) {
    if (n < 8) {
        double r = 0.0;
        for (int i = 0; i < n; i++) r = __dadd_rn(r, d64_term(x, c, lo + i));
        return r;
    }
    double r0 = d64_term(x, c, lo + 0), r1 = d64_term(x, c, lo + 1), r2 = d64_term(x, c, lo + 2),
           r3 = d64_term(x, c, lo + 3), r4 = d64_term(x, c, lo + 4), r5 = d64_term(x, c, lo + 5),
           r6 = d64_term(x, c, lo + 6), r7 = d64_term(x, c, lo + 7);
    int i = 8;
    for (; i < n - (n % 8); i += 8) {
        r0 = __dadd_rn(r0, d64_term(x, c, lo + i + 0));
        r1 = __dadd_rn(r1, d64_term(x, c, lo + i + 1));
        r2 = __dadd_rn(r2, d64_term(x, c, lo + i + 2));
        r3 = __dadd_rn(r3, d64_term(x, c, lo + i + 3));
        r4 = __dadd_rn(r4, d64_term(x, c, lo + i + 4));
        r5 = __dadd_rn(r5, d64_term(x, c, lo + i + 5));
        r6 = __dadd_rn(r6, d64_term(x, c, lo + i + 6));
        r7 = __dadd_rn(r7, d64_term(x, c, lo + i + 7));
    }
    double res = __dadd_rn(__dadd_rn(__dadd_rn(r0, r1), __dadd_rn(r2, r3)),
                           __dadd_rn(__dadd_rn(r4, r5), __dadd_rn(r6, r7)));
    for (; i < n; i++) res = __dadd_rn(res, d64_term(x, c, lo + i));
    return res;
}

// Iterative form of the recursive split (no device recursion): a post-order walk with an explicit
// stack; depth <= log2(kMaxDims / 128) + 2.
__device__ inline double d64_pairwise(const float* x, const float* c, int d) {
    if (d <= 128) return __dadd_rn(0.0, d64_leaf(x, c, 0, d));
    struct Frame { int lo, n, state; double left; };
    Frame st[16];
    int sp = 0;
    st[0] = {0, d, 0, 0.0};
    double ret = 0.0;
    while (true) {
        Frame& f = st[sp];
        if (f.n <= 128) {
            ret = d64_leaf(x, c, f.lo, f.n);
            if (sp == 0) break;
            sp--;
            continue;
        }
        int n2 = f.n / 2;
        n2 -= n2 % 8;
        if (f.state == 0) {            // descend left
            f.state = 1;
            st[++sp] = {f.lo, n2, 0, 0.0};
        } else if (f.state == 1) {     // left done -> descend right
            f.left = ret;
            f.state = 2;
            st[++sp] = {f.lo + n2, f.n - n2, 0, 0.0};
        } else {                       // right done
            ret = __dadd_rn(f.left, ret);
            if (sp == 0) break;
            sp--;
        }
    }
    return __dadd_rn(0.0, ret);
}

// D64 by one warp, bit-identical to d64_pairwise (every lane returns the value).  The leaves of the split tree
// (left to right) are listed by lane 0; leaf L's eight running partials are chains 8 L + r, spread over the
// lanes 32 at a time; a leaf's partials meet in the reference's order ((r0 + r1) + (r2 + r3)) + ((r4 + r5) +
// (r6 + r7)) through xor shuffles inside eight-lane groups (float64 addition commutes exactly), its tail terms
// follow in order, and lane 0 joins the leaves by the tree's post-order walk.  Scratch: kD64WarpScratch bytes of
// shared memory per warp, 8-byte aligned.
constexpr int kD64MaxLeaves = 64;                               // d <= kMaxDims: leaves of more than 64 terms
constexpr int kD64WarpScratch = kD64MaxLeaves * (8 + 8);
__device__ inline double d64_warp(const float* x, const float* c, int d, void* scratch) {
    const int lane = threadIdx.x & 31;
    if (d < 8) {
        double v = 0.0;
        if (lane == 0) v = d64_pairwise(x, c, d);
        return __shfl_sync(0xffffffffu, v, 0);
    }
    double* leafv = static_cast<double*>(scratch);
    int2* leaf = reinterpret_cast<int2*>(leafv + kD64MaxLeaves);     // (lo, n)
    int nleaf = 0;
    if (lane == 0) {
        int2 st[16];
        int sp = 0;
        st[0] = make_int2(0, d);
        while (sp >= 0) {
            const int2 f = st[sp--];
            if (f.y <= 128) {
                leaf[nleaf++] = f;
                continue;
            }
            int n2 = f.y / 2;
            n2 -= n2 % 8;
            st[++sp] = make_int2(f.x + n2, f.y - n2);               // right after left
            st[++sp] = make_int2(f.x, n2);
        }
    }
    nleaf = __shfl_sync(0xffffffffu, nleaf, 0);
    __syncwarp();
    for (int base = 0; base < 8 * nleaf; base += 32) {
        const int q = base + lane;
        const bool live = q < 8 * nleaf;
        const int L = live ? q >> 3 : 0, r = q & 7;
        const int2 lf = leaf[L];
        double p = 0.0;
        if (live) {
            // a chain has at most 16 terms (leaves of at most 128): its values are loaded before any is used
            const int nfull = lf.y - (lf.y % 8);
            float xv[16], cv[16];
#pragma unroll
            for (int m = 0; m < 16; m++) {
                const int i = r + 8 * m;
                xv[m] = i < nfull ? x[lf.x + i] : 0.0f;
                cv[m] = i < nfull ? c[lf.x + i] : 0.0f;
            }
            double q = __dsub_rn((double)xv[0], (double)cv[0]);
            p = __dmul_rn(q, q);
#pragma unroll
            for (int m = 1; m < 16; m++) {
                if (r + 8 * m >= nfull) break;
                q = __dsub_rn((double)xv[m], (double)cv[m]);
                p = __dadd_rn(p, __dmul_rn(q, q));
            }
        }
        p = __dadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 1));
        p = __dadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 2));
        p = __dadd_rn(p, __shfl_xor_sync(0xffffffffu, p, 4));
        if (live && r == 0) {
            for (int i = lf.y - (lf.y % 8); i < lf.y; i++) p = __dadd_rn(p, d64_term(x, c, lf.x + i));
            leafv[L] = p;
        }
    }
    __syncwarp();
    double ret = 0.0;
    if (lane == 0) {
        if (d <= 128) {
            ret = leafv[0];
        } else {
            struct Frame { int n, state; double left; };
            Frame st[16];
            int sp = 0, next = 0;
            st[0] = {d, 0, 0.0};
            while (true) {
                Frame& f = st[sp];
                if (f.n <= 128) {
                    ret = leafv[next++];
                    if (sp == 0) break;
                    sp--;
                    continue;
                }
                int n2 = f.n / 2;
                n2 -= n2 % 8;
                if (f.state == 0) {
                    f.state = 1;
                    st[++sp] = {n2, 0, 0.0};
                } else if (f.state == 1) {
                    f.left = ret;
                    f.state = 2;
                    st[++sp] = {f.n - n2, 0, 0.0};
                } else {
                    ret = __dadd_rn(f.left, ret);
                    if (sp == 0) break;
                    sp--;
                }
            }
        }
        ret = __dadd_rn(0.0, ret);
    }
    __syncwarp();
    return __shfl_sync(0xffffffffu, ret, 0);
}

// ---------------------------------------------------------------- Philox4x32-10

// Salmon, Moraes, Dror, Shaw, SC'11: ten rounds of two 32x32->64 multiplies with a Weyl key schedule.
__host__ __device__ inline void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
    for (int r = 0; r < 10; r++) {
        uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c[0] = n0; c[1] = n1; c[2] = n2; c[3] = n3;
        k0 += 0x9E3779B9u;
        k1 += 0xBB67AE85u;
    }
}

// Natural log in (0, inf) from log(m 2^e) = e ln2 + 2 atanh((m-1)/(m+1)), m in [sqrt(1/2), sqrt(2)),
// every operation an IEEE double op rounded on its own, so host and device agree bit for bit.
__host__ __device__ inline double kmc_log(double v) {
    int e = 0;
    double m = frexp(v, &e);
    if (m < 0.70710678118654752440) { m = m * 2.0; e -= 1; }
#ifdef __CUDA_ARCH__
    double s = __ddiv_rn(__dsub_rn(m, 1.0), __dadd_rn(m, 1.0));
    double s2 = __dmul_rn(s, s);
    double term = s, sum = 0.0;
    for (int i = 0; i < 40; i++) {
        sum = __dadd_rn(sum, __ddiv_rn(term, (double)(2 * i + 1)));
        term = __dmul_rn(term, s2);
    }
    return __dadd_rn(__dmul_rn((double)e, 0.69314718055994530942), __dmul_rn(2.0, sum));
#else
    double s = (m - 1.0) / (m + 1.0);
    double s2 = s * s;
    double term = s, sum = 0.0;
    for (int i = 0; i < 40; i++) {
        sum = sum + term / (double)(2 * i + 1);
        term = term * s2;
    }
    return (double)e * 0.69314718055994530942 + 2.0 * sum;
#endif
}

}  // namespace kmc
