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
constexpr int kRowsPerLane = 64;       // rows per lane between folds (a multiple of kStages, < 256)
constexpr int kBlockRows = kThreads * kRowsPerLane;   // 8192 rows per block
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

// key = score with its low mantissa bits replaced by the center index
template <unsigned MASK>
__device__ __forceinline__ float keyed(float s, unsigned idx) {
    return __uint_as_float((__float_as_uint(s) & ~MASK) | idx);
}

// add to a shared-memory word only this thread touches (program order => deterministic)
__device__ __forceinline__ void red_add(float* p, float v) {
    asm volatile("red.shared.add.f32 [%0], %1;" ::"r"((unsigned)__cvta_generic_to_shared(p)), "f"(v) : "memory");
}
__device__ __forceinline__ void red_add(unsigned* p, unsigned v) {
    asm volatile("red.shared.add.u32 [%0], %1;" ::"r"((unsigned)__cvta_generic_to_shared(p)), "r"(v) : "memory");
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

template <int D>
__device__ __forceinline__ void load_row(float (&x)[D], const float* src) {
    if constexpr (D % 4 == 0) {
#pragma unroll
        for (int q = 0; q < D / 4; q++) {
            float4 v = reinterpret_cast<const float4*>(src)[q];
            x[4 * q] = v.x; x[4 * q + 1] = v.y; x[4 * q + 2] = v.z; x[4 * q + 3] = v.w;
        }
    } else if constexpr (D % 2 == 0) {
#pragma unroll
        for (int q = 0; q < D / 2; q++) {
            float2 v = reinterpret_cast<const float2*>(src)[q];
            x[2 * q] = v.x; x[2 * q + 1] = v.y;
        }
    } else {
#pragma unroll
        for (int j = 0; j < D; j++) x[j] = src[j];
    }
}

}  // namespace

template <int D, int K>
struct LowdSmem {
    static constexpr int kSums = K * D * 32;                       // floats per warp
    static constexpr int kCnts = ((K + 3) / 4) * 32;               // packed 8-bit counts per warp (words)
    static constexpr size_t ring = (size_t)kStages * kThreads * D * 4;
    static constexpr size_t sums = (size_t)kWarps * kSums * 4;
    static constexpr size_t cnts = (size_t)kWarps * kCnts * 4;
    static constexpr size_t fold = (size_t)kWarps * K * (D + 1) * 8;
    static constexpr size_t centers = (size_t)32 * D * 4;
    static constexpr size_t acc = (size_t)K * (D + 2) * 8;
    static constexpr size_t total = ring + sums + cnts + fold + centers + acc;
};

// Per-thread state of the row loop.
template <int D, int K>
struct LowdRow {
    unsigned long long cp2[K / 2][D];   // -c, two centers per register pair
    unsigned long long hp2[K / 2];      // |c|^2 / 2
    float coef, cmax2, wabs;
    const float* cs;                    // shared copy of the centers (zero padded to 32 rows)
    float* sums;                        // this warp's sums slots
    unsigned* cnts;                     // this warp's packed counts
    int lane, k;
    double inert;
    long long rescored;
    int bad;

    template <bool CHECK, bool OUT>
    __device__ __forceinline__ void row(const float (&x)[D], int64_t row, int64_t n, int32_t* labels, float* best) {
        constexpr unsigned IDXBITS = K <= 2 ? 1 : K <= 4 ? 2 : K <= 8 ? 3 : K <= 16 ? 4 : 5;
        constexpr unsigned MASK = (1u << IDXBITS) - 1u;
        const bool valid = !CHECK || row < n;
        // ---- screen
        unsigned long long xx[D];
        float x2 = 0.0f;
#pragma unroll
        for (int j = 0; j < D; j++) {
            xx[j] = pack2(x[j], x[j]);
            x2 = __fmaf_rn(x[j], x[j], x2);
        }
        float t1[K / 2], t2[K / 2];
#pragma unroll
        for (int p = 0; p < K / 2; p++) {
            unsigned long long s = hp2[p];
#pragma unroll
            for (int j = 0; j < D; j++) s = fma2(xx[j], cp2[p][j], s);
            const float ka = keyed<MASK>(lo_of(s), 2u * p), kb = keyed<MASK>(hi_of(s), 2u * p + 1u);
            t1[p] = fminf(ka, kb);
            t2[p] = fmaxf(ka, kb);
        }
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
        int l = (int)(__float_as_uint(m1) & MASK);
        const float win = __fmaf_rn(coef, x2 + cmax2, wabs);
        const bool flag = valid && !(m2 - m1 > win);

        // ---- rows inside the window: float64, one center per lane, lowest index on ties
        unsigned fm = __ballot_sync(0xffffffffu, flag);
        if (fm) {
            rescored += flag ? 1 : 0;
            while (fm) {
                const int src = __ffs(fm) - 1;
                fm &= fm - 1;
                float xs[D];
#pragma unroll
                for (int j = 0; j < D; j++) xs[j] = __shfl_sync(0xffffffffu, x[j], src);
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
        }
        if (!valid) return;

        // ---- residual t = x - c_l and best = sum t^2 (each op rounded on its own, in column order)
        float c[D];
        load_row<D>(c, cs + l * D);
        float t[D], q[D];
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
        float* sl = sums + l * (D * 32) + lane;
#pragma unroll
        for (int j = 0; j < D; j++) red_add(sl + j * 32, t[j]);
        red_add(cnts + (l >> 2) * 32 + lane, 1u << ((l & 3) * 8));
        inert = __dadd_rn(inert, (double)b);
        if (OUT) {
            if (labels) labels[row] = l;
            if (best) best[row] = b;
        }
        if (!(b <= 3.0e38f)) bad = 1;
    }
};

template <int D, int K, bool OUT>
__global__ void __launch_bounds__(kThreads, 4) k_pass_lowd(PassArgs a) {
    static_assert(K % 2 == 0 && K <= 32, "K even, at most 32");
    constexpr int CPB = (D % 4 == 0) ? 16 : ((D % 2 == 0) ? 8 : 4);   // bytes per cp.async
    constexpr int NCP = D * 4 / CPB;
    constexpr unsigned IDXBITS = K <= 2 ? 1 : K <= 4 ? 2 : K <= 8 ? 3 : K <= 16 ? 4 : 5;
    using L = LowdSmem<D, K>;
    extern __shared__ __align__(16) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    float* sums_all = reinterpret_cast<float*>(smem + L::ring);
    unsigned* cnts_all = reinterpret_cast<unsigned*>(smem + L::ring + L::sums);
    double* fold_all = reinterpret_cast<double*>(smem + L::ring + L::sums + L::cnts);
    float* cs = reinterpret_cast<float*>(smem + L::ring + L::sums + L::cnts + L::fold);
    long long* acc = reinterpret_cast<long long*>(smem + L::ring + L::sums + L::cnts + L::fold + L::centers);

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
    // both keys' index bits move them by < 2^(IDXBITS-23) |key| <= 2^(IDXBITS-23) (|x|^2 + max|c|^2)
    st.coef = prep.win_coef + 1.0f / (float)(1u << (21 - IDXBITS));
    st.cmax2 = prep.cmax2;
    st.wabs = prep.win_abs;
    st.cs = cs;
    st.sums = sums_all + (size_t)warp * L::kSums;
    st.cnts = cnts_all + (size_t)warp * L::kCnts;
    st.lane = lane;
    st.k = k;
    st.inert = 0.0;
    st.rescored = 0;
    st.bad = 0;

    // Row of thread tid at step r of block b: b * kBlockRows + r * kThreads + tid.  Ring slot r % kStages
    // holds step r; the prefetch of step r + kStages - 1 is issued at step r into the slot read at step
    // r - 1, so this thread's reads of that slot have completed.
    const int64_t nblk = (n + kBlockRows - 1) / kBlockRows;
    float* myring = ring + (size_t)tid * D;
    constexpr int SLOT = kThreads * D;
    auto fetch = [&](int slot, int64_t row) {
        if (row < n) {
            const float* src = a.X + row * D;
            float* dst = myring + slot * SLOT;
#pragma unroll
            for (int q = 0; q < NCP; q++) cp_async<CPB>(dst + q * (CPB / 4), src + q * (CPB / 4));
        }
        cp_commit();
    };
    {
        const int64_t base0 = (int64_t)blockIdx.x * kBlockRows + tid;
#pragma unroll
        for (int s = 0; s < kStages - 1; s++) fetch(s, base0 + (int64_t)s * kThreads);
    }

    for (int64_t blk = blockIdx.x; blk < nblk; blk += gridDim.x) {
        const int64_t base = blk * kBlockRows + tid;
        const int64_t next = (blk + gridDim.x) * kBlockRows + tid;
        const bool full = (blk + 1) * kBlockRows <= n;
        auto steps = [&](auto check) {
            constexpr bool CHECK = decltype(check)::value;
            for (int ch = 0; ch < kRowsPerLane / kStages; ch++) {
#pragma unroll
                for (int s = 0; s < kStages; s++) {
                    const int r = ch * kStages + s;
                    const int pr = r + kStages - 1;
                    fetch((s + kStages - 1) & (kStages - 1),
                          pr < kRowsPerLane ? base + (int64_t)pr * kThreads
                                            : next + (int64_t)(pr - kRowsPerLane) * kThreads);
                    cp_wait<kStages - 1>();
                    float x[D];
                    load_row<D>(x, myring + s * SLOT);
                    st.template row<CHECK, OUT>(x, base + (int64_t)r * kThreads, n, a.labels, a.best);
                }
            }
        };
        if (full) steps(std::integral_constant<bool, false>{});
        else steps(std::integral_constant<bool, true>{});

        // ---- fold the lanes' slots into the CTA's int64 totals (fixed order => deterministic)
        __syncwarp();
        float* sums = st.sums;
        unsigned* cnts = st.cnts;
        for (int s = lane; s < K * D; s += 32) {
            float* col = sums + (size_t)s * 32;
            double sum = 0.0;
#pragma unroll 8
            for (int i = 0; i < 32; i++) {
                const int li = (i + lane) & 31;
                sum = __dadd_rn(sum, (double)col[li]);
                col[li] = 0.0f;
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
        if (lane == 0 && inert != 0.0)
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
    long long rescored = st.rescored;
    for (int o = 16; o; o >>= 1) rescored += __shfl_xor_sync(0xffffffffu, rescored, o);
    if (lane == 0 && rescored) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)rescored);
    if (st.bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
    (void)IDXBITS;
}

namespace {

template <int D, int K, bool OUT>
cudaError_t run(PassArgs a, cudaStream_t st) {
    using L = LowdSmem<D, K>;
    const size_t smem = L::total;
    static unsigned long long configured = 0;   // one bit per device: the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_pass_lowd<D, K, OUT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured |= 1ull << (dev & 63);
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pass_lowd<D, K, OUT>, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const int64_t nblk = (a.n + kBlockRows - 1) / kBlockRows;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > nblk) grid = nblk;
    if (grid < 1) grid = 1;
    k_pass_lowd<D, K, OUT><<<(int)grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <int D, int K>
cudaError_t run_out(PassArgs a, cudaStream_t st) {
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

int64_t lowd_block_rows() { return kBlockRows; }

cudaError_t launch_pass_lowd(PassArgs a, cudaStream_t st) {
    if (a.k > 32 || a.d > 8) return cudaErrorNotSupported;
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
