// pass_lowd.cu -- the fused low-dimensional pass (d <= 8, k <= 32): one read of X, nearest center and
// per-cluster totals in one kernel, on CUDA cores.
//
// Reference: the one-hot fused kernel of core.py:1537-1675 (configs with d <= 16: rows assigned and summed
// per cluster in one read of X) and the rows kernel's label rule (core.py:263-274); built here for B200.
//
// Per thread, one row at a time (rows streamed into shared memory by cp.async, kStages - 1 rows ahead):
//   screen   score_c = |c|^2/2 - x.c for all k centers with packed fma.rn.f32x2 (two centers per
//            instruction, centers held in registers); each score carries its center index in the low
//            mantissa bits, and a tournament over the keys yields the smallest key (value and index) and the
//            second smallest.
//   window   when the two best keys are closer than the proven error bound (screen rounding + index bits +
//            the float64 rounding of D64), the whole warp re-scores that row in float64 -- one center per
//            lane, NumPy-pairwise D64, lowest index on ties -- so a label is never decided by rounding.
//   totals   residual t = x - c_label (the float32 `best` is built from it, square and add rounded on their
//            own); lane-private float32 sums per (cluster, column) and 8-bit counts in shared memory; every
//            block of kRowsPerLane rows per lane the warp folds the 32 lanes in float64 in a fixed order,
//            adds count * c back (sum x = sum t + n c), rounds once to the fixed-point grid and adds the
//            integers into the CTA's int64 totals.  Inertia: float64 per lane, folded per block likewise.
// A block is a fixed range of kBlockRows local rows, so results are bit-reproducible; with shard starts that
// are multiples of kBlockRows they are also identical for any split of the rows over GPUs.
#include <type_traits>

#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kThreads = 128;          // 4 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 8;             // ring slots per thread (power of two)
constexpr int kRowsPerLane = 128;      // rows per lane between folds (a multiple of kStages, < 256)
constexpr int kBlockRows = kThreads * kRowsPerLane;   // 16384 rows per block
static_assert(kRowsPerLane % kStages == 0 && kRowsPerLane < 256, "block layout");

__device__ __forceinline__ unsigned long long pack2(float lo, float hi) {
    return ((unsigned long long)__float_as_uint(hi) << 32) | __float_as_uint(lo);
}
__device__ __forceinline__ float lo_of(unsigned long long v) { return __uint_as_float((unsigned)v); }
__device__ __forceinline__ float hi_of(unsigned long long v) { return __uint_as_float((unsigned)(v >> 32)); }

__device__ __forceinline__ unsigned long long fma2(unsigned long long a, unsigned long long b, unsigned long long c) {
    unsigned long long d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ unsigned long long add2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long sub2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ unsigned long long mul2(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float min3(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// key = distance with its low mantissa bits replaced by the center index: (s & keep) | IDX in one lop3, the
// index an immediate and keep (~index mask) a register
template <unsigned IDX>
__device__ __forceinline__ float keyed_imm(float s, unsigned keep) {
    unsigned d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEC;" : "=r"(d) : "r"(__float_as_uint(s)), "n"(IDX), "r"(keep));
    return __uint_as_float(d);
}

__host__ __device__ constexpr unsigned idx_bits(int k) { return k <= 2 ? 1 : k <= 4 ? 2 : k <= 8 ? 3 : k <= 16 ? 4 : 5; }

// s[0..D) += t in shared memory (a slot only this thread touches, so a plain read-modify-write), in
// 16- / 8-byte pieces where D allows
template <int D>
__device__ __forceinline__ void add_row(unsigned saddr, const float (&t)[D]) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++) {
            float a0, a1, a2, a3;
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(a0), "=f"(a1), "=f"(a2), "=f"(a3) : "r"(saddr + 16 * q));
            unsigned long long lo = add2(pack2(a0, a1), pack2(t[4 * q], t[4 * q + 1]));
            unsigned long long hi = add2(pack2(a2, a3), pack2(t[4 * q + 2], t[4 * q + 3]));
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(saddr + 16 * q), "f"(lo_of(lo)), "f"(hi_of(lo)),
                         "f"(lo_of(hi)), "f"(hi_of(hi)) : "memory");
        }
    } else if constexpr (D % 2 == 0) {
#pragma unroll
        for (int q = 0; q < D / 2; q++) {
            float a0, a1;
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(a0), "=f"(a1) : "r"(saddr + 8 * q));
            unsigned long long s = add2(pack2(a0, a1), pack2(t[2 * q], t[2 * q + 1]));
            asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(saddr + 8 * q), "f"(lo_of(s)), "f"(hi_of(s)) : "memory");
        }
    } else {
#pragma unroll
        for (int j = 0; j < D; j++) {
            float a;
            asm volatile("ld.shared.f32 %0, [%1];" : "=f"(a) : "r"(saddr + 4 * j));
            asm volatile("st.shared.f32 [%0], %1;" ::"r"(saddr + 4 * j), "f"(__fadd_rn(a, t[j])) : "memory");
        }
    }
}

__device__ __forceinline__ void add_u32(unsigned saddr, unsigned v) {
    unsigned a;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(a) : "r"(saddr));
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(saddr), "r"(a + v) : "memory");
}

template <int BYTES>
__device__ __forceinline__ void cp_async(void* smem, const void* gmem) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    if constexpr (BYTES == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], %2;" ::"r"(s), "l"(gmem), "n"(BYTES) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// float64 distance in NumPy's pairwise order (D <= 16)
template <int D>
__device__ __forceinline__ double d64_regs(const float* x, const float* c) {
    double t[D];
#pragma unroll
    for (int j = 0; j < D; j++) {
        double q = __dsub_rn((double)x[j], (double)c[j]);
        t[j] = __dmul_rn(q, q);
    }
    if constexpr (D < 8) {
        double r = 0.0;
#pragma unroll
        for (int j = 0; j < D; j++) r = __dadd_rn(r, t[j]);
        return __dadd_rn(0.0, r);
    } else {
        double r[8];
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] = t[j];
        constexpr int full = D - (D % 8);
#pragma unroll
        for (int i = 8; i < full; i += 8)
#pragma unroll
            for (int j = 0; j < 8; j++) r[j] = __dadd_rn(r[j], t[i + j]);
        double res = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                               __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
#pragma unroll
        for (int i = full; i < D; i++) res = __dadd_rn(res, t[i]);
        return __dadd_rn(0.0, res);
    }
}

// D floats from shared memory (32-bit shared-window address), in 16- or 8-byte pieces where D allows;
// the caller guarantees the alignment (rows and centers start at multiples of D floats, the buffers at 16 B)
template <int D>
__device__ __forceinline__ void load_row(float (&x)[D], unsigned saddr) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(x[4 * q]), "=f"(x[4 * q + 1]), "=f"(x[4 * q + 2]), "=f"(x[4 * q + 3])
                         : "r"(saddr + 16 * q));
    } else if constexpr (D % 2 == 0) {
#pragma unroll
        for (int q = 0; q < D / 2; q++)
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(x[2 * q]), "=f"(x[2 * q + 1]) : "r"(saddr + 8 * q));
    } else {
#pragma unroll
        for (int j = 0; j < D; j++) asm volatile("ld.shared.f32 %0, [%1];" : "=f"(x[j]) : "r"(saddr + 4 * j));
    }
}

template <int D>
struct RowVec {
    float v[D];
};

// Decide the warp's rows flagged in `fm` in float64, one center per lane, lowest index on exact ties; returns
// the label of the calling lane's row (`l` when its row is not flagged).  Out of line: it runs for a few rows
// per million and would otherwise take registers from the row loop.
template <int D>
__device__ __noinline__ int rescore_rows(unsigned fm, RowVec<D> x, const float* cs, int k, int lane, int l) {
    while (fm) {
        const int src = __ffs(fm) - 1;
        fm &= fm - 1;
        float xs[D];
#pragma unroll
        for (int j = 0; j < D; j++) xs[j] = __shfl_sync(0xffffffffu, x.v[j], src);
        double v = lane < k ? d64_regs<D>(xs, cs + lane * D) : INFINITY;
        int vi = lane;
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            double ov = __shfl_xor_sync(0xffffffffu, v, o);
            int oi = __shfl_xor_sync(0xffffffffu, vi, o);
            if (ov < v || (ov == v && oi < vi)) { v = ov; vi = oi; }
        }
        if (lane == src) l = vi;
    }
    return l;
}

}  // namespace

template <int D, int K, bool BND>
struct LowdSmem {
    static constexpr int kSums = K * D * 32;                       // floats per warp
    static constexpr int kCnts = ((K + 3) / 4) * 32;               // packed 8-bit counts per warp (words)
    static constexpr int kQueue = 64;                              // queued rows per warp (power of two)
    static constexpr size_t ring = (size_t)kStages * kThreads * D * 4;
    static constexpr size_t sums = (size_t)kWarps * kSums * 4;
    static constexpr size_t cnts = (size_t)kWarps * kCnts * 4;
    static constexpr size_t fold = (size_t)kWarps * K * (D + 1) * 8;
    static constexpr size_t centers = (size_t)32 * D * 4;
    static constexpr size_t acc = (size_t)K * (D + 2) * 8;
    static constexpr size_t wring = BND ? (size_t)kStages * kThreads * 4 : 0;
    static constexpr size_t queue = BND ? (size_t)kWarps * kQueue * 4 : 0;
    static constexpr size_t total = ring + sums + cnts + fold + centers + acc + wring + queue;
};

// Per-thread state of the row loop.
template <int D, int K>
struct LowdRow {
    static constexpr unsigned IDXBITS = idx_bits(K);
    static constexpr unsigned MASK = (1u << IDXBITS) - 1u;
    unsigned long long cp2[K / 2][D];   // -c, two centers per register pair
    unsigned long long hp2[K / 2];      // |c|^2 / 2
    float coef, slack, cmax2, wabs;
    float cum_lo, cum_up;               // drift of the centers since the bounds were started (bounds mode)
    unsigned keep;                      // ~(index mask), a launch argument so it stays in a register
    const float* cs;                    // shared copy of the centers (zero padded to 32 rows)
    unsigned cs_s;                      // its shared-window address
    float* sums;                        // this warp's sums slots: [cluster][lane][D]
    unsigned* cnts;                     // this warp's packed 8-bit counts: [cluster / 4][lane]
    unsigned sums_s, cnts_s;            // their shared-window addresses
    int lane, k;
    double inert;
    float ichunk;
    long long rescored, screened;
    int bad;

    struct Scr {
        int l;          // label
        float m2, x2;   // second smallest key, |x|^2
        bool exact;     // decided in float64
    };

    // keys of centers 2P and 2P+1: one packed distance chain, then one lop3 each inserting the index
    template <int P>
    __device__ __forceinline__ void pair(const unsigned long long (&xx)[D], unsigned long long xh2, float (&t1)[K / 2],
                                         float (&t2)[K / 2]) {
        unsigned long long s = add2(xh2, hp2[P]);
#pragma unroll
        for (int j = 0; j < D; j++) s = fma2(xx[j], cp2[P][j], s);
        const float ka = keyed_imm<2 * P>(lo_of(s), keep), kb = keyed_imm<2 * P + 1>(hi_of(s), keep);
        t1[P] = fminf(ka, kb);
        t2[P] = fmaxf(ka, kb);
    }
    template <int... P>
    __device__ __forceinline__ void pairs(std::integer_sequence<int, P...>, const unsigned long long (&xx)[D],
                                          unsigned long long xh2, float (&t1)[K / 2], float (&t2)[K / 2]) {
        (pair<P>(xx, xh2, t1, t2), ...);
    }

    // Nearest center of x over all k centers.  Warp-collective (every lane calls it; `valid` marks real rows).
    __device__ __forceinline__ Scr screen(const float (&x)[D], bool valid) {
        unsigned long long xx[D];
        float x2 = 0.0f;
#pragma unroll
        for (int j = 0; j < D; j++) {
            xx[j] = pack2(x[j], x[j]);
            x2 = __fmaf_rn(x[j], x[j], x2);
        }
        // half squared distance |x|^2/2 + |c|^2/2 - x.c: near the winner it is small, so are the index
        // bits' perturbations of the keys
        const float xh = 0.5f * x2;
        const unsigned long long xh2 = pack2(xh, xh);
        float t1[K / 2], t2[K / 2];
        pairs(std::make_integer_sequence<int, K / 2>{}, xx, xh2, t1, t2);
#pragma unroll
        for (int w = K / 4; w >= 1; w >>= 1) {
#pragma unroll
            for (int p = 0; p < w; p++) {
                const float a1 = t1[p], a2 = t2[p], b1 = t1[p + w], b2 = t2[p + w];
                t1[p] = fminf(a1, b1);
                t2[p] = min3(fmaxf(a1, b1), a2, b2);
            }
        }
        const float m1 = t1[0], m2 = t2[0];
        Scr s;
        s.l = (int)(__float_as_uint(m1) & MASK);
        s.m2 = m2;
        s.x2 = x2;
        const float win = __fmaf_rn(coef, x2 + cmax2, wabs) + slack * (fabsf(m1) + fabsf(m2));
        const bool flag = valid && !(m2 - m1 > win);
        s.exact = flag;
        // rows inside the window: float64, one center per lane, lowest index on ties
        unsigned fm = __ballot_sync(0xffffffffu, flag);
        if (fm) {
            rescored += flag ? 1 : 0;
            RowVec<D> xv;
#pragma unroll
            for (int j = 0; j < D; j++) xv.v[j] = x[j];
            s.l = rescore_rows<D>(fm, xv, cs, k, lane, s.l);
        }
        return s;
    }

    // residual t = x - c_l and best = sum t^2 (each op rounded on its own, in column order)
    __device__ __forceinline__ float residual(const float (&x)[D], int l, float (&t)[D]) {
        float c[D];
        load_row<D>(c, cs_s + (unsigned)(l * D * 4));
        float q[D];
        if constexpr (D % 2 == 0) {
#pragma unroll
            for (int j = 0; j < D; j += 2) {
                unsigned long long tp = sub2(pack2(x[j], x[j + 1]), pack2(c[j], c[j + 1]));
                unsigned long long qp = mul2(tp, tp);
                t[j] = lo_of(tp); t[j + 1] = hi_of(tp);
                q[j] = lo_of(qp); q[j + 1] = hi_of(qp);
            }
        } else {
#pragma unroll
            for (int j = 0; j < D; j++) {
                t[j] = __fsub_rn(x[j], c[j]);
                q[j] = __fmul_rn(t[j], t[j]);
            }
        }
        float b = q[0];                    // 0 + q0 == q0 exactly
#pragma unroll
        for (int j = 1; j < D; j++) b = __fadd_rn(b, q[j]);
        return b;
    }

    // this lane's slot of cluster l (plain read-modify-write: nobody else touches it)
    __device__ __forceinline__ void accumulate(int l, const float (&t)[D], float b) {
        add_row<D>(sums_s + (unsigned)((l * 32 + lane) * D * 4), t);
        add_u32(cnts_s + (unsigned)(((l >> 2) * 32 + lane) * 4), 1u << ((l & 3) * 8));
        ichunk = __fadd_rn(ichunk, b);     // float32 over at most kStages rows, then float64
    }

    // Bound word of a screened row: a lower bound on its distance to every center but its label, plus the
    // drift so far, rounded down, with the label in the low mantissa bits.  Keys of the other centers are at
    // least m2 less the index bits' share; the float32 error of a half distance is at most half of
    // coef (|x|^2 + max|c|^2).  A row decided in float64 gets no bound (0).
    __device__ __forceinline__ unsigned bound_word(const Scr& s) {
        float h = s.m2 - slack * fabsf(s.m2) - coef * (s.x2 + cmax2);
        float lb = (h > 0.0f && !s.exact) ? __fsqrt_rn(2.0f * h) : 0.0f;
        float adj = __fmul_rn(__fadd_rn(lb, cum_lo), 1.0f - 1.0f / (float)(1u << (20 - IDXBITS)));
        return (__float_as_uint(adj) & keep) | (unsigned)s.l;
    }

    // plain row: screen, residual, totals (and optionally the bound word, labels, best)
    template <bool CHECK, bool OUT, bool BW>
    __device__ __forceinline__ void row(const float (&x)[D], int64_t row, int64_t n, const PassArgs& a) {
        const bool valid = !CHECK || row < n;
        const Scr s = screen(x, valid);
        if (!valid) return;
        float t[D];
        const float b = residual(x, s.l, t);
        accumulate(s.l, t, b);
        if (BW) a.brows[row] = bound_word(s);
        if (OUT) {
            if (a.labels) a.labels[row] = s.l;
            if (a.best) a.best[row] = b;
        }
    }

    // end of a chunk of kStages rows: the float32 partial of the inertia joins the float64 one
    __device__ __forceinline__ void chunk_done() {
        inert = __dadd_rn(inert, (double)ichunk);
        ichunk = 0.0f;
    }
};

#ifndef KMC_LOWD_MIN_BLOCKS
#define KMC_LOWD_MIN_BLOCKS 4
#endif

// BND: the pass keeps per-row bounds (a.brows, one word per row; a.bmeta holds validity and drift).  On the
// first pass (bounds not valid yet) every row is screened and its word written; afterwards a row whose
// distance to its stored label is below its stored bound less the drift keeps its label without a screen,
// and the others queue per warp and are screened 32 at a time (one per lane) so the warp does not diverge.
template <int D, int K, bool OUT, bool BND>
__global__ void __launch_bounds__(kThreads, KMC_LOWD_MIN_BLOCKS) k_pass_lowd(PassArgs a) {
    static_assert(K % 2 == 0 && K <= 32, "K even, at most 32");
    constexpr int CPB = (D % 4 == 0) ? 16 : ((D % 2 == 0) ? 8 : 4);   // bytes per cp.async
    constexpr int NCP = D * 4 / CPB;
    constexpr unsigned IDXBITS = idx_bits(K);
    constexpr unsigned MASK = (1u << IDXBITS) - 1u;
    using L = LowdSmem<D, K, BND>;
    extern __shared__ __align__(16) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    float* sums_all = reinterpret_cast<float*>(smem + L::ring);
    unsigned* cnts_all = reinterpret_cast<unsigned*>(smem + L::ring + L::sums);
    double* fold_all = reinterpret_cast<double*>(smem + L::ring + L::sums + L::cnts);
    float* cs = reinterpret_cast<float*>(smem + L::ring + L::sums + L::cnts + L::fold);
    long long* acc = reinterpret_cast<long long*>(smem + L::ring + L::sums + L::cnts + L::fold + L::centers);
    unsigned* wring = reinterpret_cast<unsigned*>(smem + L::ring + L::sums + L::cnts + L::fold + L::centers + L::acc);
    int* queue_all = reinterpret_cast<int*>(smem + L::ring + L::sums + L::cnts + L::fold + L::centers + L::acc + L::wring);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = a.k;
    const int64_t n = a.n;
    double* fold = fold_all + (size_t)warp * K * (D + 1);

    for (int e = tid; e < 32 * D; e += kThreads) cs[e] = (e / D) < k ? a.C[e] : 0.0f;
    for (int e = tid; e < K * (D + 2); e += kThreads) acc[e] = 0;
    for (int e = tid; e < kWarps * L::kSums; e += kThreads) sums_all[e] = 0.0f;
    for (int e = tid; e < kWarps * L::kCnts; e += kThreads) cnts_all[e] = 0u;
    __syncthreads();

    LowdRow<D, K> st;
#pragma unroll
    for (int p = 0; p < K / 2; p++) {
        const int c0 = 2 * p, c1 = 2 * p + 1;
        // padding centers score 2^126: finite, never below a real score of representable data
        st.hp2[p] = pack2(c0 < k ? a.hc[c0] : 8.5070591730234616e37f, c1 < k ? a.hc[c1] : 8.5070591730234616e37f);
#pragma unroll
        for (int j = 0; j < D; j++) st.cp2[p][j] = pack2(-cs[c0 * D + j], -cs[c1 * D + j]);
    }
    const Prep prep = *a.prep;
    // Window of the screen.  With u = 2^-24 and g = D u / (1 - D u), the computed half distance of every
    // center is within (2 g + u / 2)(|x|^2 + |c|^2) of the exact one (|x|^2 and |c|^2 each carry g, the add
    // that joins them u, the fma chain g on |x|^2/2 + |c|^2/2 + |x||c|), so two centers within
    // (4 g + u)(|x|^2 + max|c|^2) -- taken with a 2^-10 margin plus D 2^-48 for the float64 rounding of
    // D64 -- may be misordered.  The index bits move a key by less than 2^(IDXBITS-23) of itself; every key
    // above the second smallest is at least that key less that share, hence slack = 2^(IDXBITS-22) on
    // |m1| + |m2| (a factor two to spare).
    st.coef = (float)(((4.0 * D + 2.0) / 16777216.0) * (1.0 + 1.0 / 1024.0) + (double)D / 281474976710656.0);
    st.slack = 1.0f / (float)(1u << (22 - IDXBITS));
    st.keep = a.key_keep;
    st.cmax2 = prep.cmax2;
    st.wabs = prep.win_abs;
    st.cum_lo = prep.bcum_lo;
    st.cum_up = prep.bcum_up;
    st.cs = cs;
    st.cs_s = (unsigned)__cvta_generic_to_shared(cs);
    st.sums = sums_all + (size_t)warp * L::kSums;
    st.cnts = cnts_all + (size_t)warp * L::kCnts;
    st.sums_s = (unsigned)__cvta_generic_to_shared(st.sums);
    st.cnts_s = (unsigned)__cvta_generic_to_shared(st.cnts);
    st.lane = lane;
    st.k = k;
    st.inert = 0.0;
    st.ichunk = 0.0f;
    st.rescored = 0;
    st.screened = 0;
    st.bad = 0;
    // bounded steps only once the bounds exist (the first pass writes them)
    const bool bounded = BND && prep.bvalid != 0;

    // Row of thread tid at step r of block b: b * kBlockRows + r * kThreads + tid.  Ring slot r % kStages
    // holds step r; the prefetch of step r + kStages - 1 is issued at step r into the slot read at step
    // r - 1, so this thread's reads of that slot have completed.  The prefetch walks a pointer (and, near
    // the end of the rows, a row index) kStages - 1 steps ahead of the reads, jumping to the CTA's next
    // block when it leaves the current one.  Bounded passes stream the rows' bound words the same way.
    const int64_t nblk = (n + kBlockRows - 1) / kBlockRows;
    float* myring = ring + (size_t)tid * D;
    const unsigned myring_s = (unsigned)__cvta_generic_to_shared(myring);
    unsigned* mywring = wring + tid;
    constexpr int SLOT = kThreads * D;
    constexpr int STEP = kThreads * D;                 // floats between a thread's consecutive rows
    const float* pf = a.X + ((int64_t)blockIdx.x * kBlockRows + tid) * D;
    int64_t pf_row = (int64_t)blockIdx.x * kBlockRows + tid;
    auto fetch = [&](int slot, bool ok) {
        if (ok) {
            float* dst = myring + slot * SLOT;
#pragma unroll
            for (int q = 0; q < NCP; q++) cp_async<CPB>(dst + q * (CPB / 4), pf + q * (CPB / 4));
            if (BND && bounded) cp_async<4>(mywring + slot * kThreads, a.brows + pf_row);
        }
        cp_commit();
        pf += STEP;
        pf_row += kThreads;
    };
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) fetch(s, pf_row < n);

    // per-warp queue of rows that failed their bound (offsets within the block), screened 32 at a time
    int* queue = queue_all + warp * L::kQueue;
    int qhead = 0, qcount = 0;

    for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        const int64_t base = blk * kBlockRows + tid;
        const int64_t blk0 = blk * kBlockRows;
        const int64_t next = (blk + gridDim.x) * kBlockRows + tid;
        // checks are needed only while this block or the prefetched part of the next one is ragged
        const bool clean = (blk + gridDim.x + 1) * kBlockRows <= n;

        // screen `cnt` queued rows, one per lane
        auto flush = [&](int cnt) {
            const bool v = lane < cnt;
            const int off = v ? queue[(qhead + lane) & (L::kQueue - 1)] : 0;
            const int64_t row = blk0 + off;
            float x[D];
#pragma unroll
            for (int j = 0; j < D; j++) x[j] = v ? __ldg(a.X + row * D + j) : 0.0f;
            const auto s = st.screen(x, v);
            if (v) {
                float t[D];
                const float b = st.residual(x, s.l, t);
                st.accumulate(s.l, t, b);
                a.brows[row] = st.bound_word(s);
            }
            st.screened += v ? 1 : 0;
            qhead = (qhead + cnt) & (L::kQueue - 1);
            qcount -= cnt;
        };

        auto steps = [&](auto check) {
            constexpr bool CHECK = decltype(check)::value;
            for (int ch = 0; ch < kRowsPerLane / kStages; ch++) {
#pragma unroll
                for (int s = 0; s < kStages; s++) {
                    const int r = ch * kStages + s;
                    if (s == 1 && ch == kRowsPerLane / kStages - 1) {   // step r + kStages - 1 == kRowsPerLane
                        pf = a.X + next * D;
                        pf_row = next;
                    }
                    fetch((s + kStages - 1) & (kStages - 1), !CHECK || pf_row < n);
                    cp_wait<kStages - 1>();
                    float x[D];
                    load_row<D>(x, myring_s + (unsigned)(s * SLOT * 4));
                    const int64_t row = base + (int64_t)r * kThreads;
                    if constexpr (BND) {
                        if (bounded) {
                            const bool valid = !CHECK || row < n;
                            const unsigned w = mywring[s * kThreads];
                            const int l = (int)(w & MASK);
                            float t[D];
                            const float b = st.residual(x, l, t);
                            // stored bound less the drift since it was stored (both rounded against the row)
                            const float lbn = __fmul_rn(__fsub_rn(__uint_as_float(w & st.keep), st.cum_up),
                                                        1.0f - 1.0f / 4194304.0f);
                            const bool keep_label = valid && lbn > 0.0f &&
                                                    __fmul_rn(b, 1.0f + (float)(D + 4) / 8388608.0f) <
                                                        __fmul_rn(__fmul_rn(lbn, lbn), 1.0f - 1.0f / 4194304.0f);
                            if (keep_label) st.accumulate(l, t, b);
                            const unsigned fm = __ballot_sync(0xffffffffu, valid && !keep_label);
                            if (fm) {
                                const int pos = __popc(fm & ((1u << lane) - 1u));
                                if ((fm >> lane) & 1u)
                                    queue[(qhead + qcount + pos) & (L::kQueue - 1)] = (int)(row - blk0);
                                qcount += __popc(fm);
                                if (qcount >= 32) flush(32);
                            }
                            continue;
                        }
                        st.template row<CHECK, OUT, true>(x, row, n, a);
                        st.screened += (!CHECK || row < n) ? 1 : 0;
                    } else {
                        st.template row<CHECK, OUT, false>(x, row, n, a);
                    }
                }
                st.chunk_done();
            }
        };
        if (clean) steps(std::integral_constant<bool, false>{});
        else steps(std::integral_constant<bool, true>{});
        if (BND && qcount > 0) flush(qcount);
        st.chunk_done();

        // ---- fold the lanes' slots into the CTA's int64 totals (fixed order => deterministic)
        __syncwarp();
        float* sums = st.sums;
        unsigned* cnts = st.cnts;
        // slot (c, lane) holds D floats at sums[(c * 32 + lane) * D]; lane L folds columns s = c * D + j
        for (int s = lane; s < K * D; s += 32) {
            float* col = sums + (size_t)(s / D) * 32 * D + (s % D);
            double sum = 0.0;
#pragma unroll 8
            for (int i = 0; i < 32; i++) {
                const int li = (i + lane) & 31;
                sum = __dadd_rn(sum, (double)col[li * D]);
            }
            fold[(s / D) * (D + 1) + (s % D)] = sum;
        }
        if (lane < K) {
            const unsigned* col = cnts + (lane >> 2) * 32;
            const int sh = (lane & 3) * 8;
            unsigned c = 0;
#pragma unroll 8
            for (int i = 0; i < 32; i++) c += (col[(i + lane) & 31] >> sh) & 255u;
            fold[lane * (D + 1) + D] = (double)c;
        }
        __syncwarp();
        for (int e = lane; e < L::kCnts; e += 32) cnts[e] = 0u;
        for (int e = lane; e < L::kSums; e += 32) sums[e] = 0.0f;
        for (int s = lane; s < K * (D + 1); s += 32) {
            const int c = s / (D + 1), j = s % (D + 1);
            if (c >= k) continue;
            const double cnt = fold[c * (D + 1) + D];
            if (cnt == 0.0) continue;
            if (j == D) {
                atomicAdd(reinterpret_cast<unsigned long long*>(&acc[c * (D + 2)]), (unsigned long long)(long long)cnt);
            } else {
                const double sxv = __fma_rn(cnt, (double)cs[c * D + j], fold[s]);
                atomicAdd(reinterpret_cast<unsigned long long*>(&acc[c * (D + 2) + 2 + j]),
                          (unsigned long long)__double2ll_rn(__dmul_rn(sxv, a.scale_x[j])));
            }
        }
        // inertia of the block: fixed xor-tree over the warp, one quantised add
        double inert = st.inert;
#pragma unroll
        for (int o = 16; o; o >>= 1) inert = __dadd_rn(inert, __shfl_xor_sync(0xffffffffu, inert, o));
        if (!(inert <= 1.0e300)) st.bad = 1;            // a non-finite distance anywhere in the block
        else if (lane == 0 && inert != 0.0)
            atomicAdd(reinterpret_cast<unsigned long long*>(&acc[1]),
                      (unsigned long long)__double2ll_rn(__dmul_rn(inert, prep.scale_i)));
        st.inert = 0.0;
        __syncwarp();
    }
    cp_wait<0>();
    __syncthreads();
    for (int e = tid; e < k * (D + 2); e += kThreads) {
        long long v = acc[e];
        if (v) atomicAdd(reinterpret_cast<unsigned long long*>(a.totals + e), (unsigned long long)v);
    }
    long long rescored = st.rescored, screened = st.screened;
    for (int o = 16; o; o >>= 1) {
        rescored += __shfl_xor_sync(0xffffffffu, rescored, o);
        screened += __shfl_xor_sync(0xffffffffu, screened, o);
    }
    if (lane == 0 && rescored) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)rescored);
    if (BND && lane == 0 && screened)
        atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[2]), (unsigned long long)screened);
    if (st.bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
}

namespace {

template <int D, int K, bool OUT, bool BND>
cudaError_t run(PassArgs a, cudaStream_t st) {
    using L = LowdSmem<D, K, BND>;
    const size_t smem = L::total;
    static unsigned long long configured = 0;   // one bit per device: the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_pass_lowd<D, K, OUT, BND>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        configured |= 1ull << (dev & 63);
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pass_lowd<D, K, OUT, BND>, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const int64_t nblk = (a.n + kBlockRows - 1) / kBlockRows;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > nblk) grid = nblk;
    if (grid < 1) grid = 1;
    a.key_keep = ~((1u << idx_bits(K)) - 1u);
    k_pass_lowd<D, K, OUT, BND><<<(int)grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

// bounded passes write no labels; plain passes optionally do
template <int D, int K>
cudaError_t run_out(PassArgs a, cudaStream_t st) {
    if (a.brows) return run<D, K, false, true>(a, st);
    return (a.labels || a.best) ? run<D, K, true, false>(a, st) : run<D, K, false, false>(a, st);
}

template <int D>
cudaError_t run_k(PassArgs a, cudaStream_t st) {
    const int k = a.k;
    // register budget: K * (D + 1) packed center floats
    if (k <= 2) return run_out<D, 2>(a, st);
    if (k <= 4) return run_out<D, 4>(a, st);
    if (k <= 8) return run_out<D, 8>(a, st);
    if constexpr (D <= 5) {
        if (k <= 16) return run_out<D, 16>(a, st);
    }
    if constexpr (D <= 2) {
        if (k <= 32) return run_out<D, 32>(a, st);
    }
    return cudaErrorNotSupported;
}

}  // namespace

int64_t lowd_block_rows() { return kBlockRows; }

bool lowd_supports(int d, int k) { return d >= 1 && d <= 8 && k >= 1 && k <= (d <= 2 ? 32 : d <= 5 ? 16 : 8); }

cudaError_t launch_pass_lowd(PassArgs a, cudaStream_t st) {
    if (!lowd_supports(a.d, a.k)) return cudaErrorNotSupported;
    switch (a.d) {
        case 1: return run_k<1>(a, st);
        case 2: return run_k<2>(a, st);
        case 3: return run_k<3>(a, st);
        case 4: return run_k<4>(a, st);
        case 5: return run_k<5>(a, st);
        case 6: return run_k<6>(a, st);
        case 7: return run_k<7>(a, st);
        case 8: return run_k<8>(a, st);
        default: return cudaErrorNotSupported;
    }
}

}  // namespace kmc
