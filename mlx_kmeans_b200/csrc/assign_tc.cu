// assign_tc.cu -- nearest center for d >= 32 on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Reference: the high-d exact assign of core.py:289-377 / 675-844 (a distance GEMM tile by tile with an online
// per-row argmin, x.c computed in float32) and the rows kernel's label rule (core.py:263-274); built here for
// B200 with split-precision operands and a proven error window, so the label is the float64-optimal one.
//
// Operands: x = xh + xl + ex and c = ch + cl + ec with xh = bf16(x), xl = bf16(x - xh), |ex| <= 2^-16 |x|
// (elementwise; the same for c).  One pass of three bf16 MMAs, xh.ch + xh.cl + xl.ch, accumulated in float32
// in TMEM, gives x.c to within E |x| |c| with E = 3.1 2^-16 (the dropped terms, Cauchy-Schwarz) plus the
// float32 accumulation, bounded by 3 dp 2^-24 (a sequential float32 sum of 3 dp terms each at most |x| |c|
// in total).  The score of center c is s_c = |c|^2/2 - x.c (half the distance less |x|^2/2).  A row whose two
// best scores are closer than the window (both scores' errors plus the float64 rounding of D64) is flagged
// (exact ties included); the accumulation kernel decides it in float64 (NumPy-pairwise D64, lowest index on
// ties).
//
// Kernel layout (one CTA per SM, persistent over 128-row tiles):
//   warp 0   TMA producer: per (row tile, center tile, 64-column chunk) one stage = xh, xl (128 x 64 bf16)
//            and ch, cl (BN x 64 bf16), 128-byte swizzled, 2 to 6 stages in flight (as many as fit).
//   warp 1   MMA issuer: 3 x 4 tcgen05.mma (M=128, N=BN, K=16) per stage into one of two TMEM accumulators;
//            tcgen05.commit frees the stage and, after the last chunk, hands the accumulator to the epilogue.
//   warps 2-9  epilogue: two warps per TMEM lane quarter, one per half of the accumulator's columns; a thread
//            owns one row (TMEM lane), reads its scores 32 columns at a time (tcgen05.ld) and keeps the two
//            best scores with their centers (lowest index first on ties) and the third best score (or a
//            lower bound on it), score by score in two interleaved chains (Top3) or, with many centers, a
//            chunk at a time (TopC); at the end of the row tile the pair merges its halves through shared
//            memory and writes label | flag << 31 and, for a flagged row, its candidates.
// Every wait on an mbarrier is bounded; on a timeout the CTA records an error, stops its loops and frees TMEM.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cuda_fp16.h>

#include <type_traits>

#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int BM = 128;                  // rows per tile (UMMA M)
constexpr int BK = 64;                   // bf16 columns per chunk: one 128-byte swizzle row
constexpr int kTcThreads = 320;          // producer warp, MMA warp, eight epilogue warps
constexpr int kEpiWarps = 8;
constexpr uint32_t kSpinLimit = 1u << 22;

// Shared memory.  AR (rows resident, dp <= 128): the row tile's xh / xl chunks stay for all center tiles and the
// stages carry only ch / cl; otherwise every stage carries a chunk of each.
constexpr int kResidentChunks = 2;       // dp <= 128
// APPROX (exact=False): the hi parts only, one MMA per product.
template <int BN, bool AR, bool APPROX>
struct TcSmem {
    static constexpr int A = BM * BK * 2;             // one 128 x 64 bf16 operand chunk (16 KB)
    static constexpr int B = BN * BK * 2;             // one BN x 64 bf16 chunk
    static constexpr int PARTS = APPROX ? 1 : 2;      // hi and lo, or hi alone
    static constexpr int AREG = AR ? kResidentChunks * PARTS * A : 0;
    static constexpr int STAGE = AR ? PARTS * B : PARTS * (A + B);   // the parts of each operand it carries
    static constexpr int BAR = 256;                   // barriers, TMEM address, abort flag
    static constexpr int EPI = 2 * 4 * 32 * 5 * 4;    // the column halves' trackers: [tile parity][quarter][lane]
    // as many stages as the shared memory holds, 2 to 6: the small stages of few centers (BN = 64: 48 KB) or of
    // exact=False keep more loads in flight (a streaming shape: the operands are read once), the 96 KB stages
    // of 256 centers get two
    static constexpr int FREE = 227 * 1024 - AREG - BAR - EPI - 1024;
    static constexpr int NS = FREE / STAGE < 2 ? 2 : FREE / STAGE > 6 ? 6 : FREE / STAGE;
    static constexpr int total = AREG + NS * STAGE + BAR + EPI + 1024;   // + slack to align to 1 KB
    static_assert(A % 1024 == 0 && B % 1024 == 0, "swizzle atoms are 1024-byte aligned");
    static_assert(total <= 227 * 1024, "shared memory per CTA");
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of parity `parity` to complete, at most kSpinLimit polls; false (and the abort flag set)
// on a timeout or when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
    for (uint32_t i = 0; i < kSpinLimit; i++) {
        if (mbar_try(bar, parity)) return true;
        if (*abort_flag) return false;
    }
    *abort_flag = 1;
    return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(dst), "l"(map), "r"(x), "r"(y), "r"(bar)
        : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand in the 128-byte swizzle layout TMA writes: rows of 128 B, 8-row atoms of 1024 B.  Fields:
// start address >> 4 [0,14), leading byte offset >> 4 [16,30) (1, unused by swizzled K-major), stride byte
// offset >> 4 [32,46) (1024 B between 8-row groups), descriptor version 1 [46,48), swizzle mode 2 [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: f32 accumulator [4,6), bf16 A [7,10) and B [10,13), both K-major,
// N >> 3 at [17,23), M >> 4 at [24,29)
template <int BN>
constexpr uint32_t idesc_bf16() {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_tmem), "l"(a), "l"(b), "r"(idesc), "r"(acc)
        : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive float32 columns of this thread's TMEM lane (the load and its wait in one statement, so no
// use of the registers can be scheduled between them)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
}

// The two smallest scores with their centers and the third smallest score.  push() takes centers in increasing
// index order (a strict less keeps the lower index first on ties); merge() takes another tracker's entries,
// ordered by (score, index).
struct Top3 {
    float m0, m1, m2;
    int l0, l1;
    __device__ __forceinline__ void init() {
        m0 = m1 = m2 = INFINITY;
        l0 = l1 = 0;
    }
    // values by a min / max insertion network (equal values keep their order), centers by two selects; a NaN
    // score leaves the centers alone and can only pull m1 and m2 down to m0 (a wider window: the row goes to
    // the float64 decision)
    __device__ __forceinline__ void push(float s, int c) {
        const bool a0 = s < m0, a1 = s < m1;
        l1 = a0 ? l0 : (a1 ? c : l1);
        l0 = a0 ? c : l0;
        m2 = fminf(m2, fmaxf(m1, s));
        m1 = fminf(m1, fmaxf(m0, s));
        m0 = fminf(m0, s);
    }
    __device__ __forceinline__ void push_ordered(float s, int c) {
        const bool a0 = s < m0 || (s == m0 && c < l0), a1 = s < m1 || (s == m1 && c < l1), a2 = s < m2;
        m2 = a1 ? m1 : (a2 ? s : m2);
        m1 = a0 ? m0 : (a1 ? s : m1);
        l1 = a0 ? l0 : (a1 ? c : l1);
        m0 = a0 ? s : m0;
        l0 = a0 ? c : l0;
    }
    __device__ __forceinline__ void merge(float n0, int k0, float n1, int k1, float n2) {
        push_ordered(n0, k0);
        push_ordered(n1, k1);
        if (n2 < m2) m2 = n2;      // a third best of the other set is at best third here
    }
};

// two float32 values as one packed pair (low = a), the packed subtraction rounded down, a three-way minimum
__device__ __forceinline__ unsigned long long pack2f(float a, float b) {
    return ((unsigned long long)__float_as_uint(b) << 32) | __float_as_uint(a);
}
__device__ __forceinline__ unsigned long long sub2_rd(unsigned long long a, unsigned long long b) {
    unsigned long long d;
    asm("sub.rm.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float fmin3f(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

struct TcArgs {
    int64_t n;
    int dp;                  // padded dims (multiple of 64)
    int kp;                  // padded centers (multiple of BN)
    int k;
    const float* hs;         // kp: |c|^2 / 2 (padding centers: 2^126)
    const float* xn;         // n: |x| rounded up
    const float* cmax;       // max |c| rounded up (one value)
    int32_t* lab;            // n: label | flag << 31 (flag: decide the row in float64)
    int4* cands;             // n: a flagged row's candidate centers (-1: none, w = -2: more than two)
    int* error;              // set on a barrier timeout
    float* dump;             // (kmc_tc_dot) n x k: every accumulated x.c as read from TMEM, or nullptr
    float wr;                // window term per (|x| + max|c|)^2: the rounding of the label rule's distance
    __half* lb;              // (Elkan bounds, built here) n x k: a lower bound on every row-center distance, or nullptr
    const float* xsq_lo;     // n: |x|^2 rounded down (with lb or mask)
    uint32_t* mask;          // (cascade, built here) n x kw: bit c set where c's lower bound is <= ub[row], or nullptr
    const float* ub;         // n: the cascade's threshold on the squared distance (with mask)
    int kw;                  // 32-bit words per row of mask
    const int32_t* plab;     // n: (with mask) each row's previous label
    uint32_t* srows;         // (with mask) the rows with a survivor besides that label, in any order ...
    unsigned int* nsrows;    // ... and their count (zero before the pass)
};

// 1 if x != 0 (or infinite), 0 if x == 0: x * 2^127 is at least 2^-22 for any nonzero float, and the second
// product saturates to 1 (the FMA pipe's .sat clamp; a NaN gives 0, which only a row flagged for the full
// decision can hold).
__device__ __forceinline__ float nonzero01(float x) {
    float r;
    asm("mul.rn.sat.f32 %0, %1, 0f7F000000;" : "=f"(r) : "f"(__fmul_rn(x, 0x1p127f)));
    return r;
}

// Position of the first s[j] equal to m among 32 scores, as a float (32 if none), in FMA-pipe arithmetic only:
// with ne_j = [s_j != m], the number of leading unequal scores is ne_0 (1 + ne_1 (1 + ne_2 (...))), one fused
// multiply-add per score, over four segments of 8 joined by [segment all unequal] = sat(h - 7).  ABS compares
// |s_j - m| (scores below m present); without it every s_j >= m.
template <bool ABS>
__device__ __forceinline__ float first_equal(const float (&s)[32], float m) {
    float h[4];
#pragma unroll
    for (int g = 0; g < 4; g++) {
        float acc = 0.0f;
#pragma unroll
        for (int j = 7; j >= 0; j--) {
            const float d = s[8 * g + j] - m;
            const float ne = nonzero01(ABS ? fabsf(d) : d);
            acc = fmaf(ne, acc, ne);
        }
        h[g] = acc;
    }
    float p = fmaf(__saturatef(h[2] - 7.0f), h[3], h[2]);
    p = fmaf(__saturatef(h[1] - 7.0f), p, h[1]);
    return fmaf(__saturatef(h[0] - 7.0f), p, h[0]);
}

// The two smallest scores with their centers and a lower bound on the third smallest, fed a 32-column chunk at
// a time.  A tournament gives the chunk's two smallest values (pairs by min / max, then min(max(a0, b0),
// min(a1, b1)) for the second; equal values are kept), 92 compare operations for 32 scores; the chunk's
// smallest is located (first occurrence) only when it enters the top two, by first_equal on the FMA pipe, and
// its second only when both enter.  Ties keep the lower index: earlier chunks hold lower indices, a chunk value
// equal to a kept one does not displace it, and within a chunk the first occurrence comes first.  The third
// smallest of the union is min(m2, max(m1, mc), t) with t the chunk's third; t >= sc is not computed and sc
// stands for it, so m2 is exact unless the chunk holds the row's three smallest, and never above the true third
// (a row inside the window then goes to the full decision rather than the two-candidate one).  Scores must be
// finite for the positions to be exact; a row with a non-finite score has a non-finite window and goes to the
// full decision, and positions are clamped to the chunk so a label stays in range.
struct TopC {
    float m0, m1, m2;
    int l0, l1;
    __device__ __forceinline__ void init() {
        m0 = m1 = m2 = INFINITY;
        l0 = l1 = 0;
    }
    __device__ __forceinline__ void chunk(const float (&s)[32], int cb) {
        float a[16], b[16];
#pragma unroll
        for (int i = 0; i < 16; i++) {
            a[i] = fminf(s[2 * i], s[2 * i + 1]);
            b[i] = fmaxf(s[2 * i], s[2 * i + 1]);
        }
#pragma unroll
        for (int w = 8; w >= 1; w >>= 1) {
#pragma unroll
            for (int i = 0; i < w; i++) {
                const float lo = fminf(a[i], a[i + w]);
                b[i] = fminf(fmaxf(a[i], a[i + w]), fminf(b[i], b[i + w]));
                a[i] = lo;
            }
        }
        const float mc = a[0], sc = b[0];
        m2 = fminf(fminf(m2, sc), fmaxf(m1, mc));
        if (mc < m1) {                                   // the chunk's smallest enters the top two
            const int pm = (int)fminf(first_equal<false>(s, mc), 31.0f);
            if (mc < m0) {
                if (m0 <= sc) {                          // second: the previous smallest
                    m1 = m0;
                    l1 = l0;
                } else {                                 // second: the chunk's second smallest
                    int ps;
                    if (sc != mc) {
                        ps = (int)fminf(first_equal<true>(s, sc), 31.0f);
                    } else {                             // a tie inside the chunk: its second occurrence
                        ps = 32;
#pragma unroll
                        for (int j = 31; j >= 0; j--) ps = (j > pm && s[j] == mc) ? j : ps;
                        ps = min(ps, 31);
                    }
                    m1 = sc;
                    l1 = cb + ps;
                }
                m0 = mc;
                l0 = cb + pm;
            } else {                                     // m0 <= mc < m1
                m1 = mc;
                l1 = cb + pm;
            }
        }
    }
    __device__ __forceinline__ void push_ordered(float s, int c) {
        const bool a0 = s < m0 || (s == m0 && c < l0), a1 = s < m1 || (s == m1 && c < l1), a2 = s < m2;
        m2 = a1 ? m1 : (a2 ? s : m2);
        m1 = a0 ? m0 : (a1 ? s : m1);
        l1 = a0 ? l0 : (a1 ? c : l1);
        m0 = a0 ? s : m0;
        l0 = a0 ? c : l0;
    }
    __device__ __forceinline__ void merge(float n0, int k0, float n1, int k1, float n2) {
        push_ordered(n0, k0);
        push_ordered(n1, k1);
        if (n2 < m2) m2 = n2;
    }
};

// The smallest score and its center (exact=False: no window, so the rest of the order is not needed); the same
// interface as Top3 with m1 = m2 = +inf.
struct Top1 {
    float m0, m1, m2;
    int l0, l1;
    __device__ __forceinline__ void init() {
        m0 = m1 = m2 = INFINITY;
        l0 = l1 = 0;
    }
    __device__ __forceinline__ void push(float s, int c) {      // increasing c: strict less keeps the lower index
        const bool a0 = s < m0;
        l0 = a0 ? c : l0;
        m0 = a0 ? s : m0;
    }
    __device__ __forceinline__ void merge(float n0, int k0, float, int, float) {
        if (n0 < m0 || (n0 == m0 && k0 < l0)) {
            m0 = n0;
            l0 = k0;
        }
    }
};

template <int BN, bool AR, bool APPROX, bool CHUNK>
__global__ void __launch_bounds__(kTcThreads, 1)
    k_assign_tc(const __grid_constant__ CUtensorMap mxh, const __grid_constant__ CUtensorMap mxl,
                const __grid_constant__ CUtensorMap mch, const __grid_constant__ CUtensorMap mcl, TcArgs a) {
    using S = TcSmem<BN, AR, APPROX>;
    constexpr int PARTS = S::PARTS;
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // (resident rows,) stages at the first 1024-byte boundary, then the barrier block
    const uint32_t raw = smem_u32(smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const uint32_t sbase = base + S::AREG;
    unsigned char* gbase = smem_raw + (base - raw);
    constexpr int NS = S::NS;
    const uint32_t bars = sbase + NS * S::STAGE;
    unsigned char* gbars = gbase + S::AREG + NS * S::STAGE;
    // barrier block (8 B each): full[NS] empty[NS] accf[2] acce[2], for resident rows afull, aempty; then the TMEM
    // base (4 B) and the abort flag (4 B)
    static_assert(8 * (2 * NS + 6) + 8 <= S::BAR, "barrier block");
    auto full = [&](int s) { return bars + 8u * s; };
    auto empty = [&](int s) { return bars + 8u * (NS + s); };
    auto accf = [&](int b) { return bars + 8u * (2 * NS + b); };
    auto acce = [&](int b) { return bars + 8u * (2 * NS + 2 + b); };
    const uint32_t afull = bars + 8u * (2 * NS + 4), aempty = bars + 8u * (2 * NS + 5);
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbars + 8 * (2 * NS + 6));
    volatile int* abort_flag = reinterpret_cast<volatile int*>(gbars + 8 * (2 * NS + 6) + 4);
    float* epi = reinterpret_cast<float*>(gbars + S::BAR);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t tiles = (a.n + BM - 1) / BM;
    const int ntiles = a.kp / BN, kchunks = a.dp / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(full(s), 1);
            mbar_init(empty(s), 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(accf(b), 1);
            mbar_init(acce(b), kEpiWarps * 32);
        }
        if (AR) {
            mbar_init(afull, 1);
            mbar_init(aempty, 1);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {   // two accumulators of BN float32 columns each
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ---- TMA producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0, tph = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                if constexpr (AR) {
                    // the row tile, once: after the previous tile's last MMA has read the resident chunks
                    ok = mbar_wait(aempty, tph ^ 1u, abort_flag);
                    if (!ok) break;
                    mbar_expect_tx(afull, (uint32_t)(kchunks * PARTS * S::A));
                    for (int kc = 0; kc < kchunks; kc++) {
                        tma_load_2d(base + kc * PARTS * S::A, &mxh, kc * BK, (int)(t * BM), afull);
                        if constexpr (!APPROX)
                            tma_load_2d(base + kc * 2 * S::A + S::A, &mxl, kc * BK, (int)(t * BM), afull);
                    }
                    tph ^= 1u;
                }
                for (int nt = 0; nt < ntiles && ok; nt++)
                    for (int kc = 0; kc < kchunks && ok; kc++) {
                        ok = mbar_wait(empty(stage), phase ^ 1u, abort_flag);
                        if (!ok) break;
                        const uint32_t st = sbase + stage * S::STAGE;
                        mbar_expect_tx(full(stage), S::STAGE);
                        if constexpr (AR) {
                            tma_load_2d(st, &mch, kc * BK, nt * BN, full(stage));
                            if constexpr (!APPROX) tma_load_2d(st + S::B, &mcl, kc * BK, nt * BN, full(stage));
                        } else {
                            tma_load_2d(st, &mxh, kc * BK, (int)(t * BM), full(stage));
                            if constexpr (APPROX) {
                                tma_load_2d(st + S::A, &mch, kc * BK, nt * BN, full(stage));
                            } else {
                                tma_load_2d(st + S::A, &mxl, kc * BK, (int)(t * BM), full(stage));
                                tma_load_2d(st + 2 * S::A, &mch, kc * BK, nt * BN, full(stage));
                                tma_load_2d(st + 2 * S::A + S::B, &mcl, kc * BK, nt * BN, full(stage));
                            }
                        }
                        if (++stage == NS) { stage = 0; phase ^= 1u; }
                    }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16<BN>();
            int stage = 0;
            uint32_t phase = 0, abuf = 0, aphase = 0, tph = 0;
            bool ok = true;
            for (int64_t t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                if constexpr (AR) {
                    ok = mbar_wait(afull, tph, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                }
                for (int nt = 0; nt < ntiles && ok; nt++) {
                    ok = mbar_wait(acce(abuf), aphase ^ 1u, abort_flag);
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t d_tmem = tmem + abuf * BN;
                    for (int kc = 0; kc < kchunks && ok; kc++) {
                        ok = mbar_wait(full(stage), phase, abort_flag);
                        if (!ok) break;
                        tc_fence_after();
                        const uint32_t st = sbase + stage * S::STAGE;
                        const uint32_t sa = AR ? base + kc * PARTS * S::A : st;
                        const uint32_t sb = AR ? st : st + PARTS * S::A;
                        const uint64_t ah = sw128_desc(sa), al = sw128_desc(sa + S::A);
                        const uint64_t bh = sw128_desc(sb), bl = sw128_desc(sb + S::B);
#pragma unroll
                        for (int kk = 0; kk < BK / 16; kk++) {
                            const uint64_t off = (uint64_t)((kk * 32) >> 4);   // 16 bf16 = 32 B along K
                            mma_bf16(d_tmem, ah + off, bh + off, idesc, (kc | kk) != 0);
                            if constexpr (!APPROX) {
                                mma_bf16(d_tmem, ah + off, bl + off, idesc, 1u);
                                mma_bf16(d_tmem, al + off, bh + off, idesc, 1u);
                            }
                        }
                        mma_commit(empty(stage));          // the stage is free once these MMAs are done
                        if (++stage == NS) { stage = 0; phase ^= 1u; }
                    }
                    if (!ok) break;
                    mma_commit(accf(abuf));                // the accumulator is ready for the epilogue
                    abuf ^= 1u;
                    if (abuf == 0) aphase ^= 1u;
                }
                if constexpr (AR) {
                    if (!ok) break;
                    mma_commit(aempty);                    // the resident rows are free once these MMAs are done
                    tph ^= 1u;
                }
            }
        }
    } else {
        // ---- epilogue: warp w reads TMEM lane quarter q = w % 4 (its rows 32 q + lane of the tile) and column
        // half h of every accumulator; the h = 1 warp hands its tracker to the h = 0 warp of the same quarter
        // through shared memory (named barrier 1 + q, 64 threads, once per tile on both warps, abort or not)
        const int q = warp & 3, h = (warp - 2) >> 2;
        const uint32_t lane_base = tmem + ((uint32_t)(32 * q) << 16);
        const float cmax = *a.cmax;
        // Window on the gap between the two best scores: each score is off by at most E |x| |c| (the dropped
        // split terms and the float32 accumulation) plus 2^-24 (|c|^2 + |x| |c|) (rounding of |c|^2/2 and of
        // the subtraction); two of them, with |c| <= cmax, and a 2^-10 margin for the float32 evaluation of the
        // window itself.  The distance that defines the label adds wr (|x| + cmax)^2: 2^-40 for the float64
        // rounding of D64, rule32_coef(d) more under the float32 label rule (its direct sum's error).
        const float E2 = (float)(2.0 * (3.1 / 65536.0 + 3.0 * a.dp / 16777216.0));
        constexpr int HALF = BN / 2;
        uint32_t abuf = 0, aphase = 0;
        bool ok = true;
        int it = 0;                                       // tiles done: the hand-over slot alternates with it
        for (int64_t t = blockIdx.x; t < tiles; t += gridDim.x, it++) {
            const int64_t row = t * BM + 32 * q + lane;
            const bool lbm = a.lb != nullptr || a.mask != nullptr;
            const float xr = ((h == 0 || lbm) && row < a.n) ? __ldg(a.xn + row) : 0.0f;   // in flight meanwhile
            // Elkan bounds of this row (a.lb): |x - c|^2 = |x|^2 + 2 (|c|^2/2 - x.c) >= xsq_lo + 2 (score - err), err
            // the score's error bound of the window below (E |x| max|c| + 2^-24 max|c|^2, with a margin), every
            // step rounded down, then the square root rounded down and stored as half rounded toward zero
            // The cascade's survivor bits (a.mask) come from the same lower bound, squared, against the row's
            // threshold: bit c set unless the bound exceeds ub[row].
            float lb_x = 0.0f, lb_err = 0.0f, ubr = 0.0f;
            int plab = -1;                                // (mask) the row's previous label: its own bit
            uint32_t others = 0u;                         // (mask) any surviving center but the previous label
            if (a.mask && row < a.n) {
                ubr = __ldg(a.ub + row);
                plab = __ldg(a.plab + row);
                if (plab < 0 || plab >= a.k) {            // not a final label of this k: listed for the full scoring
                    plab = 0;
                    others = 1u;
                }
            }
            if (lbm && row < a.n) {
                const float cm = *a.cmax;
                lb_x = __ldg(a.xsq_lo + row);
                lb_err = __fmul_ru(__fadd_ru(__fmul_ru(__fmul_ru((float)(3.1 / 65536.0 + 3.0 * a.dp / 16777216.0), xr), cm),
                                             __fmul_ru(__fmul_ru(cm, cm), 1.0f / 16777216.0f)),
                                   1.0f + 1.0f / 1024.0f);
            }
            using Trk = std::conditional_t<APPROX, Top1, std::conditional_t<CHUNK, TopC, Top3>>;
            Trk ev, od;                                   // per score: even and odd columns in two chains
            ev.init();
            od.init();
            for (int nt = 0; nt < ntiles && ok; nt++) {
                ok = mbar_wait(accf(abuf), aphase, abort_flag);
                if (!ok) break;
                tc_fence_after();
#pragma unroll 1
                for (int cc = h * HALF; cc < (h + 1) * HALF; cc += 32) {
                    float v[32];
                    tmem_ld32(lane_base + abuf * BN + cc, v);
                    const int c0 = nt * BN + cc;
                    if (a.lb != nullptr && row < a.n) {            // the Elkan bounds of these 32 centers
                        __half hv[32];
#pragma unroll
                        for (int j = 0; j < 32; j++) {
                            const float sc = __fsub_rd(__fsub_rd(__ldg(a.hs + c0 + j), v[j]), lb_err);
                            const float d2 = __fmaf_rd(2.0f, sc, lb_x);
                            hv[j] = __float2half_rz(d2 > 0.0f ? __fsqrt_rd(d2) : 0.0f);
                        }
                        __half* dst = a.lb + row * a.k + c0;
                        if (c0 + 32 <= a.k) {                      // k % 8 == 0: 16-byte aligned pieces
#pragma unroll
                            for (int g = 0; g < 4; g++)
                                reinterpret_cast<uint4*>(dst)[g] = reinterpret_cast<const uint4*>(hv)[g];
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; j++)
                                if (c0 + j < a.k) dst[j] = hv[j];
                        }
                    }
                    if (a.mask != nullptr && row < a.n && c0 < a.k) {   // the cascade's survivors of these 32 centers
                        // hs - x.c rounded down, two at a time, and its minimum over the chunk: the bound of that
                        // minimum (every step rounded down, so no bound of the chunk is below it) rules out the
                        // whole chunk at once, as it does for almost every chunk of a row; the others are tested
                        // center by center, from the same values
                        float sv[32];
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            const float4 hq = __ldg(reinterpret_cast<const float4*>(a.hs + c0) + g);
                            const unsigned long long d01 = sub2_rd(pack2f(hq.x, hq.y), pack2f(v[4 * g], v[4 * g + 1]));
                            const unsigned long long d23 = sub2_rd(pack2f(hq.z, hq.w), pack2f(v[4 * g + 2], v[4 * g + 3]));
                            sv[4 * g] = __uint_as_float((unsigned)d01);
                            sv[4 * g + 1] = __uint_as_float((unsigned)(d01 >> 32));
                            sv[4 * g + 2] = __uint_as_float((unsigned)d23);
                            sv[4 * g + 3] = __uint_as_float((unsigned)(d23 >> 32));
                        }
                        float mn[11];
#pragma unroll
                        for (int j = 0; j < 10; j++) mn[j] = fmin3f(sv[3 * j], sv[3 * j + 1], sv[3 * j + 2]);
                        mn[10] = fminf(sv[30], sv[31]);
                        const float m4 = fmin3f(fmin3f(mn[0], mn[1], mn[2]), fmin3f(mn[3], mn[4], mn[5]),
                                                fmin3f(fmin3f(mn[6], mn[7], mn[8]), mn[9], mn[10]));
                        uint32_t bits = 0u;
                        if (!(__fmaf_rd(2.0f, __fsub_rd(m4, lb_err), lb_x) > ubr)) {
#pragma unroll
                            for (int j = 0; j < 32; j++) {
                                const float d2 = __fmaf_rd(2.0f, __fsub_rd(sv[j], lb_err), lb_x);
                                bits |= (!(d2 > ubr) && c0 + j < a.k) ? (1u << j) : 0u;
                            }
                        }
                        a.mask[row * a.kw + (c0 >> 5)] = bits;
                        others |= (plab >> 5) == (c0 >> 5) ? bits & ~(1u << (plab & 31)) : bits;
                    }
                    if (a.mask != nullptr) continue;               // the cascade's prefix pass needs no label
                    if (a.dump != nullptr && row < a.n) {          // diagnostic copy of the raw scores
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (c0 + j < a.k) a.dump[row * a.k + c0 + j] = v[j];
                    }
                    // scores |c|^2/2 - x.c (hs 16-byte aligned: its base is, and c0 is a multiple of 32)
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        const float4 hq = __ldg(reinterpret_cast<const float4*>(a.hs + c0) + g);
                        v[4 * g] = hq.x - v[4 * g];
                        v[4 * g + 1] = hq.y - v[4 * g + 1];
                        v[4 * g + 2] = hq.z - v[4 * g + 2];
                        v[4 * g + 3] = hq.w - v[4 * g + 3];
                    }
                    if constexpr (!CHUNK) {
#pragma unroll
                        for (int j = 0; j < 32; j += 2) {
                            ev.push(v[j], c0 + j);
                            od.push(v[j + 1], c0 + j + 1);
                        }
                    } else {
                        ev.chunk(v, c0);
                    }
                }
                tc_fence_before();
                mbar_arrive(acce(abuf));
                abuf ^= 1u;
                if (abuf == 0) aphase ^= 1u;
            }
            if constexpr (!CHUNK) ev.merge(od.m0, od.l0, od.m1, od.l1, od.m2);
            float* slot = epi + ((((it & 1) * 4 + q) * 32 + lane) * 5);
            if (a.mask != nullptr) {
                // the cascade: a row with a surviving center besides its previous label is listed for the full
                // scoring (the two halves' columns combined through the hand-over slot); the others keep it
                if (h == 1) slot[0] = __uint_as_float(others);
                asm volatile("bar.sync %0, %1;" ::"r"(1 + q), "r"(64) : "memory");
                if (h == 0 && ok && row < a.n && (others | __float_as_uint(slot[0])) != 0u)
                    a.srows[atomicAdd(a.nsrows, 1u)] = (uint32_t)row;
                continue;
            }
            if (h == 1) {
                slot[0] = ev.m0;
                slot[1] = ev.m1;
                slot[2] = ev.m2;
                slot[3] = __int_as_float(ev.l0);
                slot[4] = __int_as_float(ev.l1);
            }
            asm volatile("bar.sync %0, %1;" ::"r"(1 + q), "r"(64) : "memory");
            if (h == 1 || !ok) continue;
            ev.merge(slot[0], __float_as_int(slot[3]), slot[1], __float_as_int(slot[4]), slot[2]);
            const float m0 = ev.m0, m1 = ev.m1, m2 = ev.m2;
            const int l0 = ev.l0, l1 = ev.l1;
            if (row < a.n && a.mask == nullptr) {
                const float r = xr + cmax;
                const float win = (E2 * xr * cmax + cmax * (cmax + xr) * (1.0f / 8388608.0f)) * (1.0f + 1.0f / 1024.0f) +
                                  r * r * a.wr;
                // exact=False: no window (only a row whose best is a padding center -- non-finite scores -- goes to
                // the float64 decision)
                const bool flag = APPROX ? l0 >= a.k : (!(m1 - m0 > win) || l0 >= a.k);
                a.lab[row] = (int32_t)((uint32_t)l0 | (flag ? 0x80000000u : 0u));
                // candidates: the centers whose score is within the window of the smallest; when the third is
                // too (or a score is not finite), there may be more than two: -2 sends the row to the full decision
                if (flag) {
                    int4 cand = make_int4(l0, -1, -1, -1);
                    if (!(m1 - m0 > win)) cand.y = l1;
                    if (!(m2 - m0 > win) || !(m0 <= 3.0e38f) || l0 >= a.k) cand.w = -2;
                    a.cands[row] = cand;
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
    }
    if (threadIdx.x == 0 && *abort_flag) atomicExch(a.error, 1);
}

// ---------------------------------------------------------------- host side: tensor maps and launch

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// rows x dp bf16, row-major; box of `box_rows` rows x 64 columns, 128-byte swizzle, zero fill past the end
bool make_map(CUtensorMap* m, const void* base, int64_t rows, int dp, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)dp, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)dp * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int BN, bool AR, bool APPROX, bool CHUNK = false>
cudaError_t run_tc(const TcSplit& s, cudaStream_t st) {
    CUtensorMap mxh, mxl, mch, mcl;
    if (!make_map(&mxh, s.xh, s.n, s.dp, BM) || !make_map(&mxl, s.xl, s.n, s.dp, BM) ||
        !make_map(&mch, s.ch, s.kp, s.dp, BN) || !make_map(&mcl, s.cl, s.kp, s.dp, BN))
        return cudaErrorInvalidValue;
    static unsigned long long configured = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    const size_t smem = TcSmem<BN, AR, APPROX>::total;
    if (!(configured >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_assign_tc<BN, AR, APPROX, CHUNK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return e;
        configured |= 1ull << (dev & 63);
    }
    TcArgs a;
    a.n = s.n;
    a.dp = s.dp;
    a.kp = s.kp;
    a.k = s.k;
    a.hs = s.hs;
    a.xn = s.xn;
    a.cmax = s.cmax;
    a.lab = s.lab;
    a.cands = s.cands;
    a.error = s.error;
    a.dump = s.dump;
    a.wr = (float)(1.0 / 1099511627776.0 + (s.rule ? rule32_coef(s.dp) : 0.0));
    a.lb = static_cast<__half*>(s.lb);
    a.xsq_lo = s.xsq_lo;
    a.mask = static_cast<uint32_t*>(s.mask);
    a.ub = s.ub;
    a.plab = s.plab;
    a.srows = s.srows;
    a.nsrows = s.nsrows;
    a.kw = (s.k + 31) / 32;
    const int64_t tiles = (s.n + BM - 1) / BM;
    int64_t grid = num_sms();
    if (grid > tiles) grid = tiles;
    if (grid < 1) grid = 1;
    k_assign_tc<BN, AR, APPROX, CHUNK><<<(int)grid, kTcThreads, smem, st>>>(mxh, mxl, mch, mcl, a);
    return cudaGetLastError();
}

// The per-chunk tracker (TopC) pays off with many chunks per row, used from 32 chunks of 32 columns per epilogue
// thread (2048 centers): against the per-score one it measured 25% faster at 50M x 128, k = 4096, level at
// 1M x 768, k = 1024, and 40% slower at 10M x 32, k = 64 (one chunk per thread, where the tournament and its
// lookups outweigh 32 pushes).
constexpr int kChunkTrackerMinK = 2048;

template <int BN>
cudaError_t run_tc_ar(const TcSplit& s, bool ar, cudaStream_t st) {
    if (s.approx) return ar ? run_tc<BN, true, true>(s, st) : run_tc<BN, false, true>(s, st);
    if constexpr (BN == 256) {
        if (s.kp >= kChunkTrackerMinK)
            return ar ? run_tc<BN, true, false, true>(s, st) : run_tc<BN, false, false, true>(s, st);
    }
    return ar ? run_tc<BN, true, false>(s, st) : run_tc<BN, false, false>(s, st);
}

}  // namespace

int tc_block_n(int k) { return k <= 64 ? 64 : k <= 128 ? 128 : 256; }

cudaError_t launch_assign_tc(const TcSplit& s, cudaStream_t st) {
    // the row tile stays resident when it fits (dp <= 128) and is used for more than one center tile
    const bool ar = s.dp <= kResidentChunks * BK && s.kp / tc_block_n(s.k) > 1;
    switch (tc_block_n(s.k)) {
        case 64: return run_tc_ar<64>(s, ar, st);
        case 128: return run_tc_ar<128>(s, ar, st);
        default: return run_tc_ar<256>(s, ar, st);
    }
}

}  // namespace kmc
