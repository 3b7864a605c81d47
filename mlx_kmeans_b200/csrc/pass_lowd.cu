// pass_lowd.cu -- the fused low-dimensional pass (d <= 8, k <= 32): one read of X, nearest center and
// per-cluster totals in one kernel, on CUDA cores.
//
// Reference: the one-hot fused kernel of core.py:1537-1675 (configs with d <= 16: rows assigned and summed
// per cluster in one read of X) and the rows kernel's label rule (core.py:263-274); built here for B200.
//
// Per thread, one row at a time (rows streamed into shared memory by cp.async, several rows ahead):
//   screen   score_c = |c|^2/2 - x.c for all k centers with packed fma.rn.f32x2 (two centers per
//            instruction, centers held in registers); each score carries its center index in the low
//            mantissa bits, and a tournament over the keys yields the smallest key (value and index) and the
//            second smallest.
//   window   when the two best keys are closer than the proven error bound (screen rounding + index bits +
//            the float64 rounding of D64), the whole warp re-scores that row in float64 -- one center per
//            lane, NumPy-pairwise D64, lowest index on ties -- so a label is never decided by rounding.
//   totals   residual t = x - c_label (the float32 `best` is built from it, square and add rounded on their
//            own); lane-private float32 sums per (cluster, column) and 8-bit counts in shared memory; every
//            block of rpl rows per lane the warp folds the 32 lanes in a fixed order (fold_block),
//            adds count * c back (sum x = sum t + n c), rounds once to the fixed-point grid and adds the
//            integers into the CTA's int64 totals.  Inertia: float64 per lane, folded per block likewise.
// A block is a fixed range of 128 rpl local rows, so results are bit-reproducible; with shard starts that are
// multiples of the block (kmc_row_block(n_total)) they are also identical for any split of the rows over GPUs.
//
// Two kernels:
//   k_pass_lowd     every row is screened (optionally writing labels and `best`).
//   k_pass_bounded  per-row bounds: each row carries one 32-bit word, a lower bound on its distance to every
//                   center but its label (plus the drift at the time it was stored) with the label in the low
//                   bits.  A row whose distance to its stored label's center is below the stored bound less
//                   the drift since keeps that label without a screen -- the same label the screen would give,
//                   so totals, labels and inertia are those of a full pass.  Failing rows queue per warp and
//                   are screened 32 at a time, one per lane.  The first pass after a reset screens every row.
#include <type_traits>

#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kThreads = 128;          // 4 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 8;             // ring slots per thread of the screening kernel (power of two)
#ifndef KMC_BOUNDED_AHEAD
#define KMC_BOUNDED_AHEAD 0
#endif
#ifndef KMC_BOUNDED_MAX_CTAS
#define KMC_BOUNDED_MAX_CTAS 0
#endif
// rows per thread in flight in the bounded kernel, held in registers: about 128 bytes of rows
constexpr int bounded_ahead(int d) { return KMC_BOUNDED_AHEAD ? KMC_BOUNDED_AHEAD : d <= 4 ? 8 : 4; }
// Rows per lane between folds (PassArgs::rpl), set by the dataset's global row count so that every split of the
// rows over slices and GPUs uses the same blocks: 64 (8192-row blocks) up to kLargeRows rows, 160 (20480-row
// blocks) from there -- the per-block fold of the lane sums and each round's start are paid 2.5x less often
// (96M x 4, k = 16: 0.520 -> 0.492 ms per pass), and a 12M-row shard of eight GPUs is 586 blocks, one round of
// the 592 CTA slots, where 8192-row blocks needed three rounds for 2.47 blocks per slot (0.092 -> 0.082 ms).
// Small datasets keep the smaller blocks so that more CTAs share the rows.
constexpr int kRowsSmall = 64, kRowsLarge = 160;
constexpr int64_t kLargeRows = 64000000;
constexpr int rows_per_lane(int64_t n_total) { return n_total >= kLargeRows ? kRowsLarge : kRowsSmall; }
constexpr int kQueue = 64;             // queued rows per warp in the bounded kernel (power of two, >= 64)
static_assert(kRowsSmall % kStages == 0 && kRowsSmall % 8 == 0 && kRowsLarge % kStages == 0 &&
              kRowsLarge % 8 == 0 && kRowsLarge < 256, "block layout: 8-bit counts per lane between folds");

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

// store D floats (same pieces as load_row)
template <int D>
__device__ __forceinline__ void store_row(unsigned saddr, const float (&v)[D]) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(saddr + 16 * q), "f"(v[4 * q]),
                         "f"(v[4 * q + 1]), "f"(v[4 * q + 2]), "f"(v[4 * q + 3]) : "memory");
    } else if constexpr (D % 2 == 0) {
#pragma unroll
        for (int q = 0; q < D / 2; q++)
            asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(saddr + 8 * q), "f"(v[2 * q]), "f"(v[2 * q + 1])
                         : "memory");
    } else {
#pragma unroll
        for (int j = 0; j < D; j++) asm volatile("st.shared.f32 [%0], %1;" ::"r"(saddr + 4 * j), "f"(v[j]) : "memory");
    }
}

// s += t elementwise, in packed pairs where D allows
template <int D>
__device__ __forceinline__ void add_into(float (&s)[D], const float (&t)[D]) {
#pragma unroll
    for (int j = 0; j + 1 < D; j += 2) {
        const unsigned long long r = add2(pack2(s[j], s[j + 1]), pack2(t[j], t[j + 1]));
        s[j] = lo_of(r);
        s[j + 1] = hi_of(r);
    }
    if constexpr (D % 2 == 1) s[D - 1] = __fadd_rn(s[D - 1], t[D - 1]);
}

// s[0..D) += t in shared memory (a slot only this thread touches, so a plain read-modify-write)
template <int D>
__device__ __forceinline__ void add_row(unsigned saddr, const float (&t)[D]) {
    float s[D];
    load_row<D>(s, saddr);
    add_into<D>(s, t);
    store_row<D>(saddr, s);
}

__device__ __forceinline__ unsigned long long ld_u64(unsigned saddr) {
    unsigned long long a;
    asm volatile("ld.shared.u64 %0, [%1];" : "=l"(a) : "r"(saddr));
    return a;
}

__device__ __forceinline__ void red_u32(unsigned saddr, unsigned v) {
    asm volatile("red.shared.add.u32 [%0], %1;" ::"r"(saddr), "r"(v) : "memory");
}

// global loads for data read once in a pass (read-only path, no L1 allocation), kept in program order
template <int D>
__device__ __forceinline__ void ldg_row(float (&x)[D], const float* p) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
                         : "=f"(x[4 * q]), "=f"(x[4 * q + 1]), "=f"(x[4 * q + 2]), "=f"(x[4 * q + 3])
                         : "l"(p + 4 * q));
    } else if constexpr (D % 2 == 0) {
#pragma unroll
        for (int q = 0; q < D / 2; q++)
            asm volatile("ld.global.nc.L1::no_allocate.v2.f32 {%0, %1}, [%2];" : "=f"(x[2 * q]), "=f"(x[2 * q + 1])
                         : "l"(p + 2 * q));
    } else {
#pragma unroll
        for (int j = 0; j < D; j++)
            asm volatile("ld.global.nc.L1::no_allocate.f32 %0, [%1];" : "=f"(x[j]) : "l"(p + j));
    }
}
// Rows of an even number of columns as D/2 packed pairs (one 64-bit register pair each), so the packed float32
// arithmetic of the bounded kernel needs no register moves: 16-byte pieces where the row is 16-byte aligned
// (D % 4 == 0), else 8-byte pieces.
template <int D>
__device__ __forceinline__ void ldg_row2(unsigned long long (&x)[D / 2], const float* p) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("ld.global.nc.L1::no_allocate.v2.u64 {%0, %1}, [%2];" : "=l"(x[2 * q]), "=l"(x[2 * q + 1])
                         : "l"(p + 4 * q));
    } else {
#pragma unroll
        for (int q = 0; q < D / 2; q++)
            asm volatile("ld.global.nc.L1::no_allocate.u64 %0, [%1];" : "=l"(x[q]) : "l"(p + 2 * q));
    }
}
template <int D>
__device__ __forceinline__ void lds_row2(unsigned long long (&x)[D / 2], unsigned saddr) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(x[2 * q]), "=l"(x[2 * q + 1]) : "r"(saddr + 16 * q));
    } else {
#pragma unroll
        for (int q = 0; q < D / 2; q++) asm volatile("ld.shared.u64 %0, [%1];" : "=l"(x[q]) : "r"(saddr + 8 * q));
    }
}
template <int D>
__device__ __forceinline__ void sts_row2(unsigned saddr, const unsigned long long (&x)[D / 2]) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++)
            asm volatile("st.shared.v2.u64 [%0], {%1, %2};" ::"r"(saddr + 16 * q), "l"(x[2 * q]), "l"(x[2 * q + 1])
                         : "memory");
    } else {
#pragma unroll
        for (int q = 0; q < D / 2; q++)
            asm volatile("st.shared.u64 [%0], %1;" ::"r"(saddr + 8 * q), "l"(x[q]) : "memory");
    }
}

__device__ __forceinline__ unsigned ldg_u32(const uint32_t* p) {
    unsigned v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// cp.async of BYTES (4, 8 or 16) from global memory to a shared-window address
template <int BYTES>
__device__ __forceinline__ void cp_async(unsigned s, const void* gmem) {
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

template <int D>
struct RowVec {
    float v[D];
};

// The float32 direct sum of the reference's rows kernel on registers (core.py:263-274), as best32
template <int D>
__device__ __forceinline__ float best32_regs(const float* x, const float* c) {
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < D; j++) s = best32_term(s, x[j], c[j]);
    return s;
}

// Decide the warp's rows flagged in `fm` by the label rule (rule 0: the float64 distance, rule 1: the float32
// direct sum), one center per lane, lowest index on exact ties; returns the label of the calling lane's row
// (`l` when its row is not flagged).  Out of line: it runs for a few rows per million and would otherwise take
// registers from the row loop.
template <int D>
__device__ __noinline__ int rescore_rows(unsigned fm, RowVec<D> x, const float* cs, int k, int lane, int l,
                                         int rule) {
    while (fm) {
        const int src = __ffs(fm) - 1;
        fm &= fm - 1;
        float xs[D];
#pragma unroll
        for (int j = 0; j < D; j++) xs[j] = __shfl_sync(0xffffffffu, x.v[j], src);
        double v = lane >= k ? INFINITY
                   : rule ? (double)best32_regs<D>(xs, cs + lane * D) : d64_regs<D>(xs, cs + lane * D);
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

// Centers packed two per 64-bit register pair for the screen: hp2[P] = (|c_2P|^2/2, |c_2P+1|^2/2) and
// cp2[P][j] = (-c_2P[j], -c_2P+1[j]).  Padding centers (index >= k) score 2^126: finite, never below a real
// score of representable data.
template <int D, int K>
struct Packed {
    unsigned long long cp2[K / 2][D];
    unsigned long long hp2[K / 2];

    static constexpr int kWords = K / 2 * (D + 1);   // shared layout: per pair, hp2 then cp2[0..D)

    __device__ __forceinline__ static unsigned long long word(const float* C, const float* hc, int k, int e) {
        const int P = e / (D + 1), j = e % (D + 1), c0 = 2 * P, c1 = 2 * P + 1;
        if (j == 0) return pack2(c0 < k ? hc[c0] : 8.5070591730234616e37f, c1 < k ? hc[c1] : 8.5070591730234616e37f);
        return pack2(c0 < k ? -C[c0 * D + j - 1] : -0.0f, c1 < k ? -C[c1 * D + j - 1] : -0.0f);
    }
    // from the shared layout (volatile loads: the compiler keeps them where they are written)
    __device__ __forceinline__ void load(unsigned saddr) {
#pragma unroll
        for (int P = 0; P < K / 2; P++) {
            hp2[P] = ld_u64(saddr + (unsigned)(P * (D + 1)) * 8u);
#pragma unroll
            for (int j = 0; j < D; j++) cp2[P][j] = ld_u64(saddr + (unsigned)(P * (D + 1) + 1 + j) * 8u);
        }
    }
    __device__ __forceinline__ unsigned long long hp(int P) const { return hp2[P]; }
    __device__ __forceinline__ unsigned long long cp(int P, int j) const { return cp2[P][j]; }
    __device__ __forceinline__ void load(const float* C, const float* hc, int k) {
#pragma unroll
        for (int P = 0; P < K / 2; P++) {
            hp2[P] = word(C, hc, k, P * (D + 1));
#pragma unroll
            for (int j = 0; j < D; j++) cp2[P][j] = word(C, hc, k, P * (D + 1) + 1 + j);
        }
    }
};


// The same packed centers read from their shared layout at the point of use (volatile loads, so they are not
// hoisted into registers held across a loop): for screens that are rare enough not to need registers.
template <int D, int K>
struct PackedShared {
    unsigned s;
    __device__ __forceinline__ unsigned long long hp(int P) const { return ld_u64(s + (unsigned)(P * (D + 1)) * 8u); }
    __device__ __forceinline__ unsigned long long cp(int P, int j) const {
        return ld_u64(s + (unsigned)(P * (D + 1) + 1 + j) * 8u);
    }
};

template <int D, int K>
struct PlainSmem {
    static constexpr int kSums = K * D * 32;                       // floats per warp
    static constexpr int kCnts = ((K + 3) / 4) * 32;               // packed 8-bit counts per warp (words)
    static constexpr size_t ring = (size_t)kStages * kThreads * D * 4;
    static constexpr size_t sums = (size_t)kWarps * kSums * 4;
    static constexpr size_t cnts = (size_t)kWarps * kCnts * 4;
    static constexpr size_t centers = (size_t)32 * D * 4;
    static constexpr size_t acc = (size_t)K * (D + 2) * 8;
    static constexpr size_t total = ring + sums + cnts + centers + acc;
};

template <int D, int K>
struct BoundSmem {
    static constexpr int kSums = K * D * 32;
    static constexpr int kCnts = ((K + 3) / 4) * 32;
    static constexpr size_t sums = (size_t)kWarps * kSums * 4;
    static constexpr size_t cnts = (size_t)kWarps * kCnts * 4;
    static constexpr size_t centers = (size_t)32 * D * 4;
    static constexpr size_t packed = (size_t)Packed<D, K>::kWords * 8;
    static constexpr size_t acc = (size_t)K * (D + 2) * 8;
    static constexpr size_t queue = (size_t)kWarps * kQueue * 4;
    static constexpr size_t qrows = (size_t)kWarps * kQueue * D * 4;   // the queued rows' values
    static constexpr size_t total = sums + cnts + centers + packed + acc + queue + qrows;
    static_assert(sums % 16 == 0 && cnts % 16 == 0 && centers % 16 == 0 && packed % 8 == 0 && acc % 8 == 0 &&
                  queue % 16 == 0, "shared carve alignment");
};

// Per-thread state of the row loop.  Counts are packed four 8-bit fields to a word: a lane adds at most
// rpl < 256 rows to one cluster between folds.
template <int D, int K>
struct LowdRow {
    static constexpr unsigned IDXBITS = idx_bits(K);
    static constexpr unsigned MASK = (1u << IDXBITS) - 1u;
    float coef, slack, cmax2, wabs;
    float cum_lo, cum_up;               // drift of the centers since the bounds were started (bounds mode)
    float hold_f;                       // factor of the bound test (holds), wider under the float32 rule
    int rule;                           // label rule (Prep::rule)
    unsigned keep;                      // ~(index mask), a launch argument so it stays in a register
    const float* cs;                    // shared copy of the centers (zero padded to 32 rows)
    unsigned cs_s;                      // its shared-window address
    float* sums;                        // this warp's sums slots: [cluster][lane][D]
    unsigned* cnts;                     // this warp's packed counts: [cluster / 4][lane]
    unsigned slot0_s, cnt0_s;           // shared-window addresses of this lane's slot / count word of cluster 0
    int lane, k;
    double inert;
    float ichunk;
    int rescored, screened;
    int bad;

    struct Scr {
        int l;          // label
        float m2, x2;   // second smallest key, |x|^2
        bool exact;     // decided in float64
    };

    // keys of centers 2P and 2P+1: one packed distance chain, then one lop3 each inserting the index
    template <int P, class PK>
    __device__ __forceinline__ void pair(const PK& pk, const unsigned long long (&xx)[D], unsigned long long xh2,
                                         float (&t1)[K / 2], float (&t2)[K / 2]) {
        unsigned long long s = add2(xh2, pk.hp(P));
#pragma unroll
        for (int j = 0; j < D; j++) s = fma2(xx[j], pk.cp(P, j), s);
        const float ka = keyed_imm<2 * P>(lo_of(s), keep), kb = keyed_imm<2 * P + 1>(hi_of(s), keep);
        t1[P] = fminf(ka, kb);
        t2[P] = fmaxf(ka, kb);
    }
    template <class PK, int... P>
    __device__ __forceinline__ void pairs(std::integer_sequence<int, P...>, const PK& pk,
                                          const unsigned long long (&xx)[D], unsigned long long xh2,
                                          float (&t1)[K / 2], float (&t2)[K / 2]) {
        (pair<P>(pk, xx, xh2, t1, t2), ...);
    }

    // Nearest center of x over all k centers.  Warp-collective (every lane calls it; `valid` marks real rows).
    template <class PK>
    __device__ __forceinline__ Scr screen(const float (&x)[D], bool valid, const PK& pk) {
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
        pairs(std::make_integer_sequence<int, K / 2>{}, pk, xx, xh2, t1, t2);
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
            s.l = rescore_rows<D>(fm, xv, cs, k, lane, s.l, rule);
        }
        return s;
    }

    // residual t = x - c and best = sum t^2 (each op rounded on its own, in column order)
    __device__ __forceinline__ float residual(const float (&x)[D], const float (&c)[D], float (&t)[D]) {
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
    __device__ __forceinline__ float residual(const float (&x)[D], int l, float (&t)[D]) {
        float c[D];
        load_row<D>(c, cs_s + (unsigned)(l * D * 4));
        return residual(x, c, t);
    }

    __device__ __forceinline__ unsigned slot_addr(int l) const { return slot0_s + (unsigned)l * (32u * D * 4u); }
    __device__ __forceinline__ unsigned cnt_addr(int l) const { return cnt0_s + (unsigned)(l >> 2) * 128u; }
    __device__ __forceinline__ static unsigned cnt_one(int l) { return 1u << ((l & 3) * 8); }

    // this lane's slot of cluster l (plain read-modify-write: nobody else touches it)
    __device__ __forceinline__ void accumulate(int l, const float (&t)[D], float b) {
        add_row<D>(slot_addr(l), t);
        red_u32(cnt_addr(l), cnt_one(l));
        ichunk = __fadd_rn(ichunk, b);     // float32 over at most 8 rows, then float64
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

    // Does the stored label still hold?  w: the row's bound word, b: its float32 distance to the stored label's
    // center.  With Y = stored bound - drift since (cum_up rounds the drift up), the row keeps its label when
    // the exact distance is below Y^2: b carries at most (D + 4) 2^-23 of relative error, and the computed
    // y = fl(Y) and fl(y y) exceed Y and Y^2 by at most 2^-24 and 3 2^-24 relative, fl(b F) falls short of
    // b F by at most 2^-24 -- all inside F's extra factor 1 + 2^-20.
    // Under the float32 label rule the stored label must also be the only center the direct sum can pick: every
    // other center's exact distance must exceed the label's by the direct sum's relative error on both sides,
    // (1 + theta) / (1 - theta) with theta <= gamma_{D+2}, folded into the factor as 1 + rule32_coef(D).
    static constexpr double kHoldD = (1.0 + (D + 4) / 8388608.0) * (1.0 + 1.0 / 1048576.0) * (1.0 + 1.0 / 8388608.0);
    static constexpr float kHoldF = (float)kHoldD;
    __device__ __forceinline__ bool holds(unsigned w, float b) const {
        const float y = __fsub_rn(__uint_as_float(w & keep), cum_up);
        return y > 0.0f && __fmul_rn(b, hold_f) < __fmul_rn(y, y);
    }

    // screened row: screen, residual, totals (and optionally labels and best)
    template <bool CHECK, bool OUT>
    __device__ __forceinline__ void row(const float (&x)[D], int64_t row, int64_t n, const PassArgs& a,
                                        const Packed<D, K>& pk) {
        const bool valid = !CHECK || row < n;
        const Scr s = screen(x, valid, pk);
        if (!valid) return;
        float t[D];
        const float b = residual(x, s.l, t);
        accumulate(s.l, t, b);
        if (OUT) {
            if (a.labels) a.labels[row] = s.l;
            if (a.best) a.best[row] = b;
        }
    }

    // end of a chunk of 8 rows: the float32 partial of the inertia joins the float64 one
    __device__ __forceinline__ void chunk_done() {
        inert = __dadd_rn(inert, (double)ichunk);
        ichunk = 0.0f;
    }

    __device__ __forceinline__ void init(const PassArgs& a, const Prep& prep, const float* cs_, float* sums_all,
                                         unsigned* cnts_all, int kSums, int kCnts, int warp, int lane_) {
        // Window of the screen.  With u = 2^-24 and g = D u / (1 - D u), the computed half distance of every
        // center is within (2 g + u / 2)(|x|^2 + |c|^2) of the exact one (|x|^2 and |c|^2 each carry g, the
        // add that joins them u, the fma chain g on |x|^2/2 + |c|^2/2 + |x||c|), so two centers within
        // (4 g + u)(|x|^2 + max|c|^2) -- taken with a 2^-10 margin plus D 2^-48 for the float64 rounding of
        // D64 -- may be misordered.  The index bits move a key by less than 2^(IDXBITS-23) of itself; every
        // key above the second smallest is at least that key less that share, hence slack = 2^(IDXBITS-22)
        // on |m1| + |m2| (a factor two to spare).
        // (The float32 label rule widens the window by rule32_coef(D): see common.cuh.)
        rule = prep.rule;
        coef = (float)(((4.0 * D + 2.0) / 16777216.0) * (1.0 + 1.0 / 1024.0) + (double)D / 281474976710656.0 +
                       (rule ? rule32_coef(D) : 0.0));
        hold_f = rule ? __double2float_ru(kHoldD * (1.0 + rule32_coef(D))) : kHoldF;
        slack = 1.0f / (float)(1u << (22 - IDXBITS));
        keep = a.key_keep;
        cmax2 = prep.cmax2;
        wabs = prep.win_abs;
        cum_lo = prep.bcum_lo;
        cum_up = prep.bcum_up;
        cs = cs_;
        cs_s = (unsigned)__cvta_generic_to_shared(cs_);
        sums = sums_all + (size_t)warp * kSums;
        cnts = cnts_all + (size_t)warp * kCnts;
        slot0_s = (unsigned)__cvta_generic_to_shared(sums) + (unsigned)(lane_ * D * 4);
        cnt0_s = (unsigned)__cvta_generic_to_shared(cnts) + (unsigned)(lane_ * 4);
        lane = lane_;
        k = a.k;
        inert = 0.0;
        ichunk = 0.0f;
        rescored = 0;
        screened = 0;
        bad = 0;
    }

    // End of a block: fold the lanes' slots into the CTA's int64 totals (fixed order => deterministic) and
    // the block's inertia into acc[1].  Counts first: the even and the odd 8-bit fields of each word are summed
    // over the warp as 16-bit fields (at most 32 * rpl < 2^16 each), and lane j < 4 parks the count of
    // cluster 4 w + j in its own word.  Then the columns: the 32 lanes' partial sums of a column in a fixed
    // order (even D: columns j, j + 1 of a cluster as one packed float32 pair, a five-level tree; odd D: one
    // column in float64), then sum x = sum t + count * c in float64, rounded once to the fixed-point grid.  (The
    // lanes' partials are sequential float32 sums of rpl residuals already; five more levels of float32
    // addition keep the error of the same order.)
    __device__ __forceinline__ void fold_block(long long* acc, const double* scale_x, double scale_i) {
        static_assert(32 * kRowsLarge < 65536, "16-bit count fields");
        __syncwarp();
#pragma unroll
        for (int w = 0; w < (K + 3) / 4; w++) {
            const unsigned v = cnts[w * 32 + lane];
            const unsigned ev = __reduce_add_sync(0xffffffffu, v & 0x00ff00ffu);          // fields 0 and 2
            const unsigned od = __reduce_add_sync(0xffffffffu, (v >> 8) & 0x00ff00ffu);   // fields 1 and 3
            const unsigned f = (lane & 1) ? od : ev;
            cnts[w * 32 + lane] = lane < 2 ? (f & 0xffffu) : lane < 4 ? (f >> 16) : 0u;
        }
        __syncwarp();
        auto put = [&](int c, int j, double sum) {
            const unsigned cnt = cnts[(c >> 2) * 32 + (c & 3)];
            if (c < k && cnt) {
                const double sxv = __fma_rn((double)cnt, (double)cs[c * D + j], sum);
                atomicAdd(reinterpret_cast<unsigned long long*>(&acc[c * (D + 2) + 2 + j]),
                          (unsigned long long)__double2ll_rn(__dmul_rn(sxv, scale_x[j])));
                if (j == 0) atomicAdd(reinterpret_cast<unsigned long long*>(&acc[c * (D + 2)]), (unsigned long long)cnt);
            }
        };
        if constexpr (D % 2 == 0) {
            // columns j, j + 1 of a cluster side by side: the 32 lanes' pairs summed in packed float32 by a
            // fixed five-level tree (four eight-leaf trees, then their pairs)
            for (int p = lane; p < K * D / 2; p += 32) {
                const int c = (2 * p) / D, j = (2 * p) % D;
                const float* col = sums + (size_t)c * 32 * D + j;
                unsigned long long part[4];
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    unsigned long long v[8];
#pragma unroll
                    for (int e = 0; e < 8; e++)
                        v[e] = *reinterpret_cast<const unsigned long long*>(col + ((8 * q + e + lane) & 31) * D);
                    part[q] = add2(add2(add2(v[0], v[1]), add2(v[2], v[3])), add2(add2(v[4], v[5]), add2(v[6], v[7])));
                }
                const unsigned long long s2 = add2(add2(part[0], part[1]), add2(part[2], part[3]));
                put(c, j, (double)lo_of(s2));
                put(c, j + 1, (double)hi_of(s2));
            }
        } else {
            for (int s = lane; s < K * D; s += 32) {
                const int c = s / D, j = s % D;
                const float* col = sums + (size_t)c * 32 * D + j;
                double sum = 0.0;
#pragma unroll 8
                for (int i = 0; i < 32; i++) {
                    const int li = (i + lane) & 31;
                    sum = __dadd_rn(sum, (double)col[li * D]);
                }
                put(c, j, sum);
            }
        }
        __syncwarp();
        if (lane < 4)
            for (int w = 0; w < (K + 3) / 4; w++) cnts[w * 32 + lane] = 0u;
        static_assert((K * D * 32) % 64 == 0, "sums slots zeroed as float2");
        for (int e = lane; e < K * D * 16; e += 32) reinterpret_cast<float2*>(sums)[e] = make_float2(0.0f, 0.0f);
        // inertia of the block: fixed xor-tree over the warp, one quantised add
        double in = inert;
#pragma unroll
        for (int o = 16; o; o >>= 1) in = __dadd_rn(in, __shfl_xor_sync(0xffffffffu, in, o));
        if (!(in <= 1.0e300)) bad = 1;            // a non-finite distance anywhere in the block
        else if (lane == 0 && in != 0.0)
            atomicAdd(reinterpret_cast<unsigned long long*>(&acc[1]),
                      (unsigned long long)__double2ll_rn(__dmul_rn(in, scale_i)));
        inert = 0.0;
        __syncwarp();
    }

    // End of the kernel (after a __syncthreads): the CTA's totals and counters into global memory.
    __device__ __forceinline__ void finish(const long long* acc, const PassArgs& a, int tid) {
        for (int e = tid; e < k * (D + 2); e += kThreads) {
            long long v = acc[e];
            if (v) atomicAdd(reinterpret_cast<unsigned long long*>(a.totals + e), (unsigned long long)v);
        }
        int r = rescored, s = screened;
        for (int o = 16; o; o >>= 1) {
            r += __shfl_xor_sync(0xffffffffu, r, o);
            s += __shfl_xor_sync(0xffffffffu, s, o);
        }
        if (lane == 0 && r) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)r);
        if (lane == 0 && s) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[2]), (unsigned long long)s);
        if (bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
    }
};

// CTAs per SM that the shared memory of one CTA allows (228 KB per SM, 1 KB of it reserved per CTA), at most
// eight.  The register cap of __launch_bounds__ follows from it (128 registers at four CTAs of 128 threads,
// 168 at three), so an instance is not squeezed below what its shared memory lets run anyway; the screening
// kernel, which holds the packed centers in registers, asks for at most four.
constexpr int ctas_per_sm(size_t smem) {
    int c = 8;
    while (c > 1 && (smem + 1024) * c > 233472) c--;
    return c;
}

// Every row screened; OUT: labels and best written too.
template <int D, int K, bool OUT>
__global__ void __launch_bounds__(kThreads, ctas_per_sm(PlainSmem<D, K>::total) < 4 ? ctas_per_sm(PlainSmem<D, K>::total)
                                                                                 : 4) k_pass_lowd(PassArgs a) {
    static_assert(K % 2 == 0 && K <= 32, "K even, at most 32");
    constexpr int CPB = (D % 4 == 0) ? 16 : ((D % 2 == 0) ? 8 : 4);   // bytes per cp.async
    constexpr int NCP = D * 4 / CPB;
    using L = PlainSmem<D, K>;
    extern __shared__ __align__(16) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    float* sums_all = reinterpret_cast<float*>(smem + L::ring);
    unsigned* cnts_all = reinterpret_cast<unsigned*>(smem + L::ring + L::sums);
    float* cs = reinterpret_cast<float*>(smem + L::ring + L::sums + L::cnts);
    long long* acc = reinterpret_cast<long long*>(smem + L::ring + L::sums + L::cnts + L::centers);

    pdl_wait();                                        // k_prepare's constants
    if (a.prep->skip) return;                          // a device Lloyd loop has stopped
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = a.k;
    const int64_t n = a.n;
    const Prep prep = *a.prep;

    for (int e = tid; e < 32 * D; e += kThreads) cs[e] = (e / D) < k ? a.C[e] : 0.0f;
    for (int e = tid; e < K * (D + 2); e += kThreads) acc[e] = 0;
    for (int e = tid; e < kWarps * L::kSums; e += kThreads) sums_all[e] = 0.0f;
    for (int e = tid; e < kWarps * L::kCnts; e += kThreads) cnts_all[e] = 0u;
    __syncthreads();

    Packed<D, K> pk;
    pk.load(cs, a.hc, k);
    LowdRow<D, K> st;
    st.init(a, prep, cs, sums_all, cnts_all, L::kSums, L::kCnts, warp, lane);

    // Row of thread tid at step r of block b: b * BR + r * kThreads + tid (BR = kThreads * rpl rows per block).
    // Ring slot r % kStages
    // holds step r; the prefetch of step r + kStages - 1 is issued at step r into the slot read at step
    // r - 1, so this thread's reads of that slot have completed.  The prefetch walks a pointer (and, near
    // the end of the rows, a row index) kStages - 1 steps ahead of the reads, jumping to the CTA's next
    // block when it leaves the current one.
    const int64_t BR = (int64_t)kThreads * a.rpl;
    const int nch = a.rpl / kStages;
    const int64_t nblk = (n + BR - 1) / BR;
    const unsigned myring_s = (unsigned)__cvta_generic_to_shared(ring + (size_t)tid * D);
    constexpr int SLOT = kThreads * D;
    constexpr int STEP = kThreads * D;                 // floats between a thread's consecutive rows
    const float* pf = a.X + ((int64_t)blockIdx.x * BR + tid) * D;
    int64_t pf_row = (int64_t)blockIdx.x * BR + tid;
    auto fetch = [&](int slot, bool ok) {
        if (ok) {
            const unsigned dst = myring_s + (unsigned)(slot * SLOT * 4);
#pragma unroll
            for (int q = 0; q < NCP; q++) cp_async<CPB>(dst + q * CPB, pf + q * (CPB / 4));
        }
        cp_commit();
        pf += STEP;
        pf_row += kThreads;
    };
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) fetch(s, pf_row < n);

    for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        const int64_t base = blk * BR + tid;
        const int64_t next = (blk + gridDim.x) * BR + tid;
        // checks are needed only while this block or the prefetched part of the next one is ragged
        const bool clean = (blk + gridDim.x + 1) * BR <= n;

        auto steps = [&](auto check) {
            constexpr bool CHECK = decltype(check)::value;
            for (int ch = 0; ch < nch; ch++) {
#pragma unroll
                for (int s = 0; s < kStages; s++) {
                    const int r = ch * kStages + s;
                    if (s == 1 && ch == nch - 1) {   // step r + kStages - 1 == rpl: the next block
                        pf = a.X + next * D;
                        pf_row = next;
                    }
                    fetch((s + kStages - 1) & (kStages - 1), !CHECK || pf_row < n);
                    cp_wait<kStages - 1>();
                    float x[D];
                    load_row<D>(x, myring_s + (unsigned)(s * SLOT * 4));
                    st.template row<CHECK, OUT>(x, base + (int64_t)r * kThreads, n, a, pk);
                    if (s % 8 == 7) st.chunk_done();
                }
            }
        };
        if (clean) steps(std::integral_constant<bool, false>{});
        else steps(std::integral_constant<bool, true>{});
        st.chunk_done();
        st.fold_block(acc, a.scale_x, prep.scale_i);
    }
    cp_wait<0>();
    pdl_launch_next();                                 // k_finish may be scheduled now
    __syncthreads();
    st.finish(acc, a, tid);
}

// The bounded pass.  A row keeps its stored label without a screen when either test proves it the nearest center:
// Hamerly's bound (its distance to the label's center below the stored lower bound less the drift since) or his
// half-separation test (that distance below half the label center's distance to its nearest other center,
// hsep, which needs no history).  Each thread streams its rows and their bound words straight into registers, P rows ahead
// (global loads that skip L1: every byte is read once), so neither passes through shared memory; the center
// of the next row's stored label is read one row ahead.  A row whose bound holds adds its residual to its
// lane's slot of the stored label.  Rows whose bound fails queue per warp (offsets within the block) and are
// screened 32 at a time, one per lane, reading the row again (from L2) and the packed centers from shared
// memory at the point of use, so the screen holds no registers across the row loop.  Before the bounds exist
// (the first pass after a reset) every row takes that route and gets its word.
// CTAs per SM of the bounded kernel: four (128 registers) up to four columns, three (168) above, where the
// rows in flight and the screen's operands need more registers
constexpr int bounded_ctas(int d, size_t smem) {
    const int cap = KMC_BOUNDED_MAX_CTAS ? KMC_BOUNDED_MAX_CTAS : d <= 4 ? 4 : 3;
    return ctas_per_sm(smem) < cap ? ctas_per_sm(smem) : cap;
}

template <int D, int K, int P>
__global__ void __launch_bounds__(kThreads, bounded_ctas(D, BoundSmem<D, K>::total)) k_pass_bounded(PassArgs a) {
    static_assert(K % 2 == 0 && K <= 32, "K even, at most 32");
    static_assert(P == 4 || P == 8 || P == 16, "prefetch depth");
    constexpr int U = P > 8 ? P : 8;                    // steps per unrolled chunk
    constexpr unsigned MASK = LowdRow<D, K>::MASK;
    using L = BoundSmem<D, K>;
    extern __shared__ __align__(16) unsigned char smem[];
    size_t off = 0;
    float* sums_all = reinterpret_cast<float*>(smem + off);        off += L::sums;
    unsigned* cnts_all = reinterpret_cast<unsigned*>(smem + off);  off += L::cnts;
    float* cs = reinterpret_cast<float*>(smem + off);              off += L::centers;
    unsigned long long* pks = reinterpret_cast<unsigned long long*>(smem + off);   off += L::packed;
    long long* acc = reinterpret_cast<long long*>(smem + off);     off += L::acc;
    int* queue_all = reinterpret_cast<int*>(smem + off);           off += L::queue;
    float* qrows_all = reinterpret_cast<float*>(smem + off);

    pdl_wait();                                        // k_prepare's constants
    if (a.prep->skip) return;                          // a device Lloyd loop has stopped
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = a.k;
    const int64_t n = a.n;
    __shared__ float sh_hsep[32];                        // Hamerly's s(c)/2 test, squared (0 past k: never holds)

    for (int e = tid; e < 32 * D; e += kThreads) cs[e] = (e / D) < k ? a.C[e] : 0.0f;
    for (int e = tid; e < 32; e += kThreads) sh_hsep[e] = e < k ? a.hsep[e] : 0.0f;
    for (int e = tid; e < Packed<D, K>::kWords; e += kThreads) pks[e] = Packed<D, K>::word(a.C, a.hc, k, e);
    for (int e = tid; e < K * (D + 2); e += kThreads) acc[e] = 0;
    for (int e = tid; e < kWarps * L::kSums; e += kThreads) sums_all[e] = 0.0f;
    for (int e = tid; e < kWarps * L::kCnts; e += kThreads) cnts_all[e] = 0u;
    __syncthreads();

    const Prep prep = *a.prep;
    LowdRow<D, K> st;
    st.init(a, prep, cs, sums_all, cnts_all, L::kSums, L::kCnts, warp, lane);
    const PackedShared<D, K> pk_s{(unsigned)__cvta_generic_to_shared(pks)};
    const bool bounded = prep.bvalid != 0;

    // Row of thread tid at step r of block b: b * BR + r * kThreads + tid, as in the screening kernel.
    // Register slot r % P holds row r; it is refilled with row r + P once row r is done.  Steps run in chunks
    // of U; a refill reads from this chunk's or the next chunk's base (the next block's first chunk after the
    // last one) at a constant offset, so the loads carry immediate offsets and no per-row pointer arithmetic.
    const int64_t BR = (int64_t)kThreads * a.rpl;
    const int64_t nblk = (n + BR - 1) / BR;
    constexpr int XSTEP = kThreads * D;                 // floats between a thread's consecutive rows
    const int nch = a.rpl / U;
    // rows in flight; an even number of columns is kept as packed pairs end to end (PK), so the packed float32
    // arithmetic needs no register moves
    constexpr bool PK = D % 2 == 0;
    constexpr int DH = (D + 1) / 2;
    float xq[P][D];
    unsigned long long xq2[P][DH];
    unsigned wq[P];
    auto fetch = [&](float (&x)[D], unsigned long long (&x2)[DH], unsigned& w, const float* px, const uint32_t* pw,
                     bool ok) {
        if (ok) {
            if constexpr (PK) ldg_row2<D>(x2, px);
            else ldg_row<D>(x, px);
            w = ldg_u32(pw);
        } else {
            if constexpr (PK) {
#pragma unroll
                for (int j = 0; j < DH; j++) x2[j] = 0ull;
            } else {
#pragma unroll
                for (int j = 0; j < D; j++) x[j] = 0.0f;
            }
            w = 0u;
        }
    };
    {
        const int64_t r0 = (int64_t)blockIdx.x * BR + tid;
#pragma unroll
        for (int q = 0; q < P; q++)
            fetch(xq[q], xq2[q], wq[q], a.X + (r0 + q * kThreads) * D, a.brows + r0 + q * kThreads,
                  r0 + q * kThreads < n);
    }
    // the center of the row in flight's stored label (a label past the end is masked: inside the 32-row table)
    float cr[D];
    unsigned long long cr2[DH];
    if constexpr (PK) lds_row2<D>(cr2, st.cs_s + (wq[0] & MASK) * (unsigned)(D * 4));
    else load_row<D>(cr, st.cs_s + (wq[0] & MASK) * (unsigned)(D * 4));

    // failing rows queue per warp: the row's offset in the block and its values (taken from the registers it was
    // streamed into, so a flush reads shared memory only)
    int* queue = queue_all + warp * kQueue;
    const unsigned qrows_s = (unsigned)__cvta_generic_to_shared(qrows_all + (size_t)warp * kQueue * D);
    int qhead = 0, qcount = 0;

    for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        const int64_t base = blk * BR + tid;
        const int64_t blk0 = blk * BR;
        const int64_t next = (blk + gridDim.x) * BR + tid;
        const bool clean = (blk + gridDim.x + 1) * BR <= n;

        // screen `cnt` queued rows, one per lane
        auto flush = [&](int cnt) {
            __syncwarp();                          // the queue entries other lanes stored are visible
            const bool v = lane < cnt;
            const int slot = (qhead + lane) & (kQueue - 1);
            const int qoff = v ? queue[slot] : 0;
            const int64_t row = blk0 + qoff;
            float x[D];
            if (v) load_row<D>(x, qrows_s + (unsigned)(slot * D * 4));
            else {
#pragma unroll
                for (int j = 0; j < D; j++) x[j] = 0.0f;
            }
            const auto s = st.screen(x, v, pk_s);
            if (v) {
                float t[D];
                const float b = st.residual(x, s.l, t);
                st.accumulate(s.l, t, b);
                a.brows[row] = st.bound_word(s);
            }
            st.screened += v ? 1 : 0;
            qhead = (qhead + cnt) & (kQueue - 1);
            qcount -= cnt;
            __syncwarp();                          // every lane has read its entry before the slots are reused
        };

        const float* xblk = a.X + base * D;
        const uint32_t* wblk = a.brows + base;
        auto steps = [&](auto check) {
            constexpr bool CHECK = decltype(check)::value;
            for (int ch = 0; ch < nch; ch++) {
                // this chunk's rows and the next chunk's (the next block's first chunk after the last)
                const bool last = ch == nch - 1;
                const float* xc = xblk + (int64_t)ch * U * XSTEP;
                const uint32_t* wc = wblk + ch * U * kThreads;
                const float* xn = last ? a.X + next * D : xc + U * XSTEP;
                const uint32_t* wn = last ? a.brows + next : wc + U * kThreads;
                const int64_t nrow = last ? next : base + (int64_t)(ch + 1) * U * kThreads;
#pragma unroll
                for (int s = 0; s < U; s++) {
                    const int r = ch * U + s;
                    const int q = s % P;
                    const int rofs = r * kThreads + tid;             // row within the block
                    const bool valid = !CHECK || blk0 + rofs < n;
                    const unsigned w = wq[q];
                    const int l = (int)(w & MASK);
                    // this lane's slot of the stored label first: its latency overlaps the arithmetic
                    const unsigned sa = st.slot_addr(l);
                    const float hl = sh_hsep[l];
                    bool keep;
                    float b;
                    if constexpr (PK) {
                        // residual t = x - c and best = sum t^2 in column order, as LowdRow::residual, on pairs
                        unsigned long long sl2[DH], t2[DH];
                        lds_row2<D>(sl2, sa);
                        b = 0.0f;
#pragma unroll
                        for (int i = 0; i < DH; i++) {
                            t2[i] = sub2(xq2[q][i], cr2[i]);
                            const unsigned long long q2 = mul2(t2[i], t2[i]);
                            b = i == 0 ? lo_of(q2) : __fadd_rn(b, lo_of(q2));
                            b = __fadd_rn(b, hi_of(q2));
                        }
                        // both tests evaluated (no branch per row)
                        keep = bounded & valid & (st.holds(w, b) | (__fmul_rn(b, st.hold_f) < hl));
                        lds_row2<D>(cr2, st.cs_s + (wq[(s + 1) % P] & MASK) * (unsigned)(D * 4));   // row r + 1's
                        if (keep) {
#pragma unroll
                            for (int i = 0; i < DH; i++) sl2[i] = add2(sl2[i], t2[i]);
                            sts_row2<D>(sa, sl2);
                        }
                    } else {
                        float sl[D], t[D];
                        load_row<D>(sl, sa);
                        b = st.residual(xq[q], cr, t);
                        // both tests evaluated (no branch per row)
                        keep = bounded & valid & (st.holds(w, b) | (__fmul_rn(b, st.hold_f) < hl));
                        load_row<D>(cr, st.cs_s + (wq[(s + 1) % P] & MASK) * (unsigned)(D * 4));   // row r + 1's
                        if (keep) {
                            add_into<D>(sl, t);
                            store_row<D>(sa, sl);
                        }
                    }
                    if (keep) {
                        red_u32(st.cnt_addr(l), LowdRow<D, K>::cnt_one(l));
                        st.ichunk = __fadd_rn(st.ichunk, b);
                    }
                    const unsigned fm = __ballot_sync(0xffffffffu, valid && !keep);
                    if (fm) {
                        const int pos = __popc(fm & ((1u << lane) - 1u));
                        if ((fm >> lane) & 1u) {
                            const int slot = (qhead + qcount + pos) & (kQueue - 1);
                            queue[slot] = rofs;
                            const unsigned qa = qrows_s + (unsigned)(slot * D * 4);
                            if constexpr (PK) sts_row2<D>(qa, xq2[q]);
                            else store_row<D>(qa, xq[q]);
                        }
                        qcount += __popc(fm);
                        if (qcount >= 32) flush(32);
                    }
                    // the refill: row r + P, in this chunk or the next
                    if (s + P < U)                       // resolved at compile time: the loop is unrolled
                        fetch(xq[q], xq2[q], wq[q], xc + (s + P) * XSTEP, wc + (s + P) * kThreads,
                              !CHECK || base + (int64_t)(r + P) * kThreads < n);
                    else
                        fetch(xq[q], xq2[q], wq[q], xn + (s + P - U) * XSTEP, wn + (s + P - U) * kThreads,
                              !CHECK || nrow + (int64_t)(s + P - U) * kThreads < n);
                    if (s % 8 == 7) st.chunk_done();
                }
            }
        };
        if (clean) steps(std::integral_constant<bool, false>{});
        else steps(std::integral_constant<bool, true>{});
        if (qcount > 0) flush(qcount);
        st.chunk_done();
        st.fold_block(acc, a.scale_x, prep.scale_i);
    }
    pdl_launch_next();                                 // k_finish may be scheduled now
    __syncthreads();
    st.finish(acc, a, tid);
}

namespace {

template <typename Kern>
cudaError_t launch_grid(Kern kern, size_t smem, unsigned long long& configured, PassArgs a, cudaStream_t st) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1ull)) {   // one bit per device: the attributes are per device
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        // Shared memory and L1 split one 256 KB array per SM.  Left to itself the driver may give shared memory
        // all of it (room for more CTAs than the registers allow), which leaves L1 too small to hold the global
        // loads in flight and caps a streaming kernel well below HBM bandwidth.  Ask for the smallest carveout
        // that still fits the CTAs the kernel can run, and give the rest to L1.
        int want = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&want, kern, kThreads, smem);
        if (e != cudaSuccess) return e;
        if (want >= 1) {
            int pct = (int)((100 * (size_t)want * (smem + 1024) + 233471) / 233472);
            for (; pct <= 100; pct++) {
                e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, pct);
                if (e != cudaSuccess) return e;
                int got = 0;
                e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&got, kern, kThreads, smem);
                if (e != cudaSuccess) return e;
                if (got >= want) break;
            }
        }
        configured |= 1ull << (dev & 63);
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    // as many CTAs as fit, but no more than it takes to give every CTA the same number of blocks: with few
    // blocks per CTA (a shard of a multi-GPU run) an uneven last round would otherwise set the pass time
    const int64_t nblk = (a.n + (int64_t)kThreads * a.rpl - 1) / ((int64_t)kThreads * a.rpl);
    const int64_t max_grid = (int64_t)num_sms() * per_sm;
    const int64_t rounds = (nblk + max_grid - 1) / max_grid;
    int64_t grid = rounds > 0 ? (nblk + rounds - 1) / rounds : 1;
    if (grid < 1) grid = 1;
    return launch_pdl(kern, dim3((unsigned)grid), dim3(kThreads), smem, st, a);
}

template <int D, int K, bool OUT>
cudaError_t run(PassArgs a, cudaStream_t st) {
    static unsigned long long configured = 0;
    a.key_keep = ~((1u << idx_bits(K)) - 1u);
    return launch_grid(k_pass_lowd<D, K, OUT>, PlainSmem<D, K>::total, configured, a, st);
}

template <int D, int K>
cudaError_t run_bounded(PassArgs a, cudaStream_t st) {
    static unsigned long long configured = 0;
    a.key_keep = ~((1u << idx_bits(K)) - 1u);
    return launch_grid(k_pass_bounded<D, K, bounded_ahead(D)>, BoundSmem<D, K>::total, configured, a, st);
}

// bounded passes write no labels; plain passes optionally write labels and best
template <int D, int K>
cudaError_t run_out(PassArgs a, cudaStream_t st) {
    if (a.brows) return run_bounded<D, K>(a, st);
    return (a.labels || a.best) ? run<D, K, true>(a, st) : run<D, K, false>(a, st);
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

int64_t lowd_block_rows(int64_t n_total) { return (int64_t)kThreads * rows_per_lane(n_total); }

bool lowd_supports(int d, int k) { return d >= 1 && d <= 8 && k >= 1 && k <= (d <= 2 ? 32 : d <= 5 ? 16 : 8); }

cudaError_t launch_pass_lowd(PassArgs a, cudaStream_t st) {
    if (!lowd_supports(a.d, a.k)) return cudaErrorNotSupported;
    a.rpl = rows_per_lane(a.n_total);
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
