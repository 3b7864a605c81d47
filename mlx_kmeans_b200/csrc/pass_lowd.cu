// pass_lowd.cu -- the fused low-dimensional pass (d <= 16, k <= 32): one read of X, nearest center and
// per-cluster totals in one kernel, on CUDA cores.
//
// Reference: the one-hot fused kernel of core.py:1537-1675 (configs with d <= 16: rows assigned and summed
// per cluster in one read of X) and the rows kernel's label rule (core.py:263-274); built here for B200.
//
// Per thread, one row at a time (rows streamed through shared memory by cp.async, 8 steps ahead):
//   screen   score_c = |c|^2/2 - x.c for all k centers with packed fma.rn.f32x2 (two centers per
//            instruction, centers held in registers); each score carries its center index in the low
//            mantissa bits so one running min gives value and index together; the second-smallest key
//            is tracked for the error window.
//   window   when the two best keys are closer than the proven error bound (screen rounding + index bits +
//            the float64 rounding of D64), the whole warp re-scores that row in float64 -- one center per
//            lane, NumPy-pairwise D64, lowest index on ties -- so a label is never decided by rounding.
//   totals   residual t = x - c_label (the float32 `best` is built from it, square and add rounded on their
//            own), lane-private float32 slots in shared memory per (cluster, column) and a lane-private
//            count; every block of 64 rows per lane the warp folds the 32 lanes' slots in float64 in a fixed
//            order, adds count * c back (sum x = sum t + n c), rounds once to the fixed-point grid and adds
//            the integers into the CTA's int64 totals.  Inertia: float64 per lane, folded the same way.
// Block structure is a function of the local row index only, so results are bit-reproducible; with shard
// starts that are multiples of kBlockRows they are also identical for any number of GPUs.
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kThreads = 128;          // 4 warps per CTA
constexpr int kWarps = kThreads / 32;
constexpr int kStages = 8;             // cp.async rows in flight per thread
constexpr int kRowsPerLane = 64;       // rows per lane between slot folds
constexpr int kBlockRows = kThreads * kRowsPerLane;   // 8192 rows per block

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

// key = score with its low mantissa bits replaced by the center index
template <unsigned MASK>
__device__ __forceinline__ float keyed(float s, unsigned idx) {
    return __uint_as_float((__float_as_uint(s) & ~MASK) | idx);
}

__device__ __forceinline__ void cp_async(void* smem, const void* gmem, int bytes) {
    unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    if (bytes == 16)
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
    else if (bytes == 8)
        asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(s), "l"(gmem) : "memory");
    else
        asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// float64 distance in NumPy's pairwise order, row and center in registers / shared memory (D <= 16)
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
    for (int j = 0; j < 8; j++) r[j] = t[j < D ? j : 0];
    constexpr int full = D - (D % 8);
#pragma unroll
    for (int i = 8; i < full; i += 8)
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] = __dadd_rn(r[j], t[(i + j) < D ? i + j : 0]);
    double res = __dadd_rn(__dadd_rn(__dadd_rn(r[0], r[1]), __dadd_rn(r[2], r[3])),
                           __dadd_rn(__dadd_rn(r[4], r[5]), __dadd_rn(r[6], r[7])));
#pragma unroll
    for (int i = full; i < D; i++) res = __dadd_rn(res, t[i]);
    return __dadd_rn(0.0, res);
    }
}

}  // namespace

template <int D, int K>
struct LowdSmem {
    static constexpr int kSlotsPerWarp = K * (D + 1) * 32;           // floats
    static constexpr size_t ring = (size_t)kStages * kThreads * D * 4;
    static constexpr size_t slots = (size_t)kWarps * kSlotsPerWarp * 4;
    static constexpr size_t fold = (size_t)kWarps * K * (D + 1) * 8;  // per-warp float64 fold results
    static constexpr size_t centers = (size_t)32 * D * 4;
    static constexpr size_t acc = (size_t)K * (D + 2) * 8;
    static constexpr size_t total = ring + slots + fold + centers + acc;
};

template <int D, int K>
__global__ void __launch_bounds__(kThreads, 3) k_pass_lowd(PassArgs a) {
    static_assert(K % 2 == 0 && K <= 32, "K even, at most 32");
    constexpr unsigned IDXBITS = K <= 2 ? 1 : K <= 4 ? 2 : K <= 8 ? 3 : K <= 16 ? 4 : 5;
    constexpr unsigned MASK = (1u << IDXBITS) - 1u;
    constexpr int CPB = (D % 4 == 0) ? 16 : ((D % 2 == 0) ? 8 : 4);   // bytes per cp.async
    constexpr int NCP = D * 4 / CPB;
    using L = LowdSmem<D, K>;
    extern __shared__ __align__(16) unsigned char smem[];
    float* ring = reinterpret_cast<float*>(smem);
    float* slots_all = reinterpret_cast<float*>(smem + L::ring);
    double* fold_all = reinterpret_cast<double*>(smem + L::ring + L::slots);
    float* cs = reinterpret_cast<float*>(smem + L::ring + L::slots + L::fold);
    long long* acc = reinterpret_cast<long long*>(smem + L::ring + L::slots + L::fold + L::centers);

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int k = a.k;
    const int64_t n = a.n;
    float* slots = slots_all + (size_t)warp * L::kSlotsPerWarp;
    double* fold = fold_all + (size_t)warp * K * (D + 1);

    // centers: shared copy (residuals, re-scoring) and packed registers (screen)
    for (int e = tid; e < 32 * D; e += kThreads) {
        int c = e / D;
        cs[e] = c < k ? a.C[e] : 0.0f;
    }
    for (int e = tid; e < K * (D + 2); e += kThreads) acc[e] = 0;
    for (int e = tid; e < kWarps * L::kSlotsPerWarp; e += kThreads) slots_all[e] = 0.0f;
    __syncthreads();
    unsigned long long cp2[K / 2][D];
    unsigned long long hp2[K / 2];
#pragma unroll
    for (int p = 0; p < K / 2; p++) {
        const int c0 = 2 * p, c1 = 2 * p + 1;
        // padding centers score 2^126: finite, never below a real score of representable data
        float h0 = c0 < k ? a.hc[c0] : 8.5070591730234616e37f;
        float h1 = c1 < k ? a.hc[c1] : 8.5070591730234616e37f;
        hp2[p] = pack2(h0, h1);
#pragma unroll
        for (int j = 0; j < D; j++) cp2[p][j] = pack2(c0 < k ? cs[c0 * D + j] : 0.0f, c1 < k ? cs[c1 * D + j] : 0.0f);
    }
    const Prep prep = *a.prep;
    const float idx_slack = 1.0f / (float)(1u << (22 - IDXBITS));          // 2^(IDXBITS-22) per key

    const int64_t nblk = (n + kBlockRows - 1) / kBlockRows;
    int64_t my_blocks = nblk > blockIdx.x ? (nblk - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int64_t iters = my_blocks * kRowsPerLane;
    // row of iteration it of this thread
    auto row_of = [&](int64_t it) -> int64_t {
        int64_t b = blockIdx.x + (it / kRowsPerLane) * gridDim.x;
        int r = (int)(it % kRowsPerLane);
        return b * kBlockRows + (int64_t)r * kThreads + tid;
    };
    auto issue = [&](int64_t it) {
        if (it < iters) {
            int64_t row = row_of(it);
            if (row < n) {
                float* dst = ring + ((size_t)(it % kStages) * kThreads + tid) * D;
                const float* src = a.X + row * D;
#pragma unroll
                for (int q = 0; q < NCP; q++) cp_async(dst + q * (CPB / 4), src + q * (CPB / 4), CPB);
            }
        }
        cp_commit();
    };
    // stage it % kStages holds iteration it; the refill of a stage is issued one iteration after the stage
    // was read, so the thread's own shared-memory reads of it have completed
#pragma unroll
    for (int s = 0; s < kStages - 1; s++) issue(s);

    double inert = 0.0;
    long long rescored = 0;
    int bad = 0;
    for (int64_t it = 0; it < iters; it++) {
        issue(it + kStages - 1);
        cp_wait<kStages - 1>();
        const int64_t row = row_of(it);
        const bool valid = row < n;
        float x[D];
        {
            const float* src = ring + ((size_t)(it % kStages) * kThreads + tid) * D;
#pragma unroll
            for (int j = 0; j < D; j++) x[j] = valid ? src[j] : 0.0f;
        }

        // ---- screen
        unsigned long long nx2[D];
        float x2 = 0.0f;
#pragma unroll
        for (int j = 0; j < D; j++) {
            nx2[j] = pack2(-x[j], -x[j]);
            x2 = __fmaf_rn(x[j], x[j], x2);
        }
        float m1 = 3.0e38f, m2 = 3.0e38f;
#pragma unroll
        for (int p = 0; p < K / 2; p++) {
            unsigned long long s = hp2[p];
#pragma unroll
            for (int j = 0; j < D; j++) s = fma2(nx2[j], cp2[p][j], s);
            const float ka = keyed<MASK>(lo_of(s), 2u * p), kb = keyed<MASK>(hi_of(s), 2u * p + 1u);
            m2 = fminf(m2, fmaxf(m1, ka));
            m1 = fminf(m1, ka);
            m2 = fminf(m2, fmaxf(m1, kb));
            m1 = fminf(m1, kb);
        }
        int l = (int)(__float_as_uint(m1) & MASK);
        const float win = __fmaf_rn(prep.win_coef, x2 + prep.cmax2, prep.win_abs) +
                          (fabsf(m1) + fabsf(m2)) * idx_slack;
        const bool flag = valid && !(m2 - m1 > win);

        // ---- rows inside the window: float64, one center per lane, lowest index on ties
        unsigned fm = __ballot_sync(0xffffffffu, flag);
        if (fm) {
            rescored += (flag ? 1 : 0);
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

        // ---- residual, best, lane-private totals
        if (valid) {
            const float* cl = cs + l * D;
            float t[D];
            float b = 0.0f;
#pragma unroll
            for (int j = 0; j < D; j++) {
                t[j] = __fsub_rn(x[j], cl[j]);
                b = __fadd_rn(b, __fmul_rn(t[j], t[j]));
            }
            float* sl = slots + (size_t)l * (D + 1) * 32 + lane;
#pragma unroll
            for (int j = 0; j < D; j++) sl[j * 32] += t[j];
            sl[D * 32] += 1.0f;
            inert = __dadd_rn(inert, (double)b);
            if (a.labels) a.labels[row] = l;
            if (a.best) a.best[row] = b;
            if (!(b <= 3.0e38f)) bad = 1;
        }

        // ---- fold the lanes' slots into the CTA's int64 totals (fixed order => deterministic)
        if ((it % kRowsPerLane) == kRowsPerLane - 1) {
            __syncwarp();
            for (int s = lane; s < K * (D + 1); s += 32) {
                float* col = slots + (size_t)s * 32;
                double sum = 0.0;
#pragma unroll 8
                for (int i = 0; i < 32; i++) {
                    const int li = (i + lane) & 31;
                    sum = __dadd_rn(sum, (double)col[li]);
                    col[li] = 0.0f;
                }
                fold[s] = sum;
            }
            __syncwarp();
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
#pragma unroll
            for (int o = 16; o; o >>= 1) inert = __dadd_rn(inert, __shfl_xor_sync(0xffffffffu, inert, o));
            if (lane == 0 && inert != 0.0)
                atomicAdd(reinterpret_cast<unsigned long long*>(&acc[1]),
                          (unsigned long long)__double2ll_rn(__dmul_rn(inert, prep.scale_i)));
            inert = 0.0;
            __syncwarp();
        }
    }
    cp_wait<0>();
    __syncthreads();
    for (int e = tid; e < k * (D + 2); e += kThreads) {
        long long v = acc[e];
        if (v) atomicAdd(reinterpret_cast<unsigned long long*>(a.totals + e), (unsigned long long)v);
    }
    for (int o = 16; o; o >>= 1) rescored += __shfl_xor_sync(0xffffffffu, rescored, o);
    if (lane == 0 && rescored) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)rescored);
    if (bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
}

namespace {

template <int D, int K>
cudaError_t run(PassArgs a, cudaStream_t st) {
    using L = LowdSmem<D, K>;
    const size_t smem = L::total;
    static unsigned long long configured = 0;   // one bit per device: the attribute is per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (!(configured >> (dev & 63) & 1ull)) {
        cudaError_t e = cudaFuncSetAttribute(k_pass_lowd<D, K>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured |= 1ull << (dev & 63);
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pass_lowd<D, K>, kThreads, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorNotSupported;
    const int64_t nblk = (a.n + kBlockRows - 1) / kBlockRows;
    int64_t grid = (int64_t)num_sms() * per_sm;
    if (grid > nblk) grid = nblk;
    if (grid < 1) grid = 1;
    k_pass_lowd<D, K><<<(int)grid, kThreads, smem, st>>>(a);
    return cudaGetLastError();
}

template <int D>
cudaError_t run_k(PassArgs a, cudaStream_t st) {
    const int k = a.k;
    // register budget: K * (D + 1) packed center floats
    if (k <= 2) return run<D, 2>(a, st);
    if (k <= 4) return run<D, 4>(a, st);
    if (k <= 8) return run<D, 8>(a, st);
    if constexpr (D <= 5) {
        if (k <= 16) return run<D, 16>(a, st);
    }
    if constexpr (D <= 2) {
        if (k <= 32) return run<D, 32>(a, st);
    }
    return cudaErrorNotSupported;
}

}  // namespace

// Rows per block of the fused pass: shards whose first global row is a multiple of this give the same
// bits on any number of GPUs.
int64_t lowd_block_rows() { return kBlockRows; }

cudaError_t launch_pass_lowd(PassArgs a, cudaStream_t st) {
    if (a.k > 32 || a.d > 16) return cudaErrorNotSupported;
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
