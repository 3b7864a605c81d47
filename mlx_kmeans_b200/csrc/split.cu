// split.cu -- the operands and the totals of the tensor-core pass (d >= 32).
//
//   k_split_rows     once per dataset slice: x = xh + xl (bf16 hi / lo, row-major, columns padded to a
//                    multiple of 64 with zeros) and |x| rounded up, for assign_tc.cu
//   k_split_centers  once per pass: the same split of the centers (rows padded to the MMA tile), |c|^2/2 and
//                    max |c| (rounded up)
//   k_accum_split    per row: the label from assign_tc.cu (rows it flagged are decided here in float64,
//                    NumPy-pairwise D64 over all centers, lowest index on ties, one warp per flagged row),
//                    `best` (the reference's float32 distance), and the row's totals quantised on its own
//                    into int64 (shared-memory slots when k (d + 2) fits, else the global totals)
//
// Reference: the high-d exact path of core.py:289-377 / 675-844 and its accumulation (core.py:1292-1441); the
// label rule of core.py:263-274.
#include <cuda_bf16.h>

#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kSplitThreads = 256;

__device__ __forceinline__ void split_bf16(float v, __nv_bfloat16& h, __nv_bfloat16& l) {
    h = __float2bfloat16_rn(v);
    l = __float2bfloat16_rn(v - __bfloat162float(h));   // v - h is exact in float32
}

// one warp per row: the bf16 halves and |x| rounded up (float64 sum of squares, square root rounded up)
__global__ void __launch_bounds__(kSplitThreads) k_split_rows(const float* __restrict__ X, int64_t n, int d, int dp,
                                                             __nv_bfloat16* __restrict__ xh,
                                                             __nv_bfloat16* __restrict__ xl,
                                                             float* __restrict__ xn) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kSplitThreads / 32);
    for (int64_t r = (int64_t)blockIdx.x * (kSplitThreads / 32) + (threadIdx.x >> 5); r < n; r += warps) {
        const float* x = X + r * d;
        double s = 0.0;
        for (int j = lane; j < dp; j += 32) {
            const float v = j < d ? x[j] : 0.0f;
            __nv_bfloat16 h, l;
            split_bf16(v, h, l);
            xh[r * dp + j] = h;
            xl[r * dp + j] = l;
            s = __fma_ru((double)v, (double)v, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s = __dadd_ru(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) xn[r] = __double2float_ru(__dsqrt_ru(s));
    }
}

// one warp per (padded) center: halves, |c|^2 / 2 (float64, rounded to nearest float; padding 2^126), max |c|
__global__ void __launch_bounds__(kSplitThreads) k_split_centers(const float* __restrict__ C, int k, int d, int kp,
                                                                int dp, __nv_bfloat16* __restrict__ ch,
                                                                __nv_bfloat16* __restrict__ cl,
                                                                float* __restrict__ hs,
                                                                unsigned int* __restrict__ cmax_bits) {
    const int lane = threadIdx.x & 31;
    const int warps = gridDim.x * (kSplitThreads / 32);
    for (int c = blockIdx.x * (kSplitThreads / 32) + (threadIdx.x >> 5); c < kp; c += warps) {
        const bool real = c < k;
        double s = 0.0, su = 0.0;                         // |c|^2 rounded to nearest, and rounded up
        for (int j = lane; j < dp; j += 32) {
            const float v = (real && j < d) ? C[(int64_t)c * d + j] : 0.0f;
            __nv_bfloat16 h, l;
            split_bf16(v, h, l);
            ch[(int64_t)c * dp + j] = h;
            cl[(int64_t)c * dp + j] = l;
            s = __fma_rn((double)v, (double)v, s);
            su = __fma_ru((double)v, (double)v, su);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            s = __dadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
            su = __dadd_ru(su, __shfl_xor_sync(0xffffffffu, su, o));
        }
        if (lane == 0) {
            hs[c] = real ? (float)(0.5 * s) : 8.5070591730234616e37f;
            if (real) atomicMax(cmax_bits, __float_as_uint(__double2float_ru(__dsqrt_ru(su))));
        }
    }
}

// Decide the warp's rows flagged in `fm` in float64 over all k centers (lanes split the centers, ascending per
// lane, then a lowest-index reduction); returns the calling lane's label (`l` when its row is not flagged).
__device__ __noinline__ int rescore_all(unsigned fm, const float* __restrict__ X, int64_t row, int d,
                                        const float* __restrict__ C, int k, int lane, int l) {
    while (fm) {
        const int src = __ffs(fm) - 1;
        fm &= fm - 1;
        const int64_t r = __shfl_sync(0xffffffffu, row, src);
        const float* x = X + r * d;
        double bv = INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < k; c += 32) {
            const double v = d64_pairwise(x, C + (int64_t)c * d, d);
            if (v < bv) { bv = v; bi = c; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov < bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == src) l = bi;
    }
    return l;
}

// one thread per row
__global__ void __launch_bounds__(kSplitThreads) k_accum_split(PassArgs a, const int32_t* __restrict__ lab,
                                                              const int* __restrict__ tc_error) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int d = a.d, k = a.k;
    const int W = d + 2;
    long long* sacc = reinterpret_cast<long long*>(smem_raw);
    const int nslots = a.smem_acc ? k * W : 0;
    for (int s = threadIdx.x; s < nslots; s += blockDim.x) sacc[s] = 0;
    __syncthreads();
    const Prep prep = *a.prep;
    const bool all_flagged = *tc_error != 0;   // the tensor-core kernel gave up: decide every row here
    const int lane = threadIdx.x & 31;
    int rescored = 0, bad = 0;
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    // the loop bound is uniform over the warp (rows of a warp are consecutive), so the warp re-scores together
    for (int64_t base = (int64_t)blockIdx.x * blockDim.x; base < a.n; base += stride) {
        const int64_t i = base + threadIdx.x;
        const bool live = i < a.n;
        const uint32_t w = live ? (uint32_t)lab[i] : 0u;
        const bool flag = live && (all_flagged || (w >> 31) != 0);
        int l = (int)(w & 0x7fffffffu);
        const unsigned fm = __ballot_sync(0xffffffffu, flag);
        if (fm) {
            l = rescore_all(fm, a.X, i, d, a.C, k, lane, l);
            rescored += flag ? 1 : 0;
        }
        if (!live) continue;
        if (l >= k) l = 0;                     // a label past k only comes with a flag, which fixed it
        const float* xr = a.X + i * d;
        const float* cr = a.C + (int64_t)l * d;
        float b = 0.0f;
        for (int j = 0; j < d; j++) b = best32_term(b, xr[j], cr[j]);
        if (!isfinite(b)) bad = 1;
        if (a.labels) a.labels[i] = l;
        if (a.best) a.best[i] = b;
        long long* acc = a.smem_acc ? sacc + (size_t)l * W : a.totals + (size_t)l * W;
        atomicAdd(reinterpret_cast<unsigned long long*>(acc), 1ull);
        atomicAdd(reinterpret_cast<unsigned long long*>(acc + 1), (unsigned long long)quantize(b, prep.scale_i));
        for (int j = 0; j < d; j++)
            atomicAdd(reinterpret_cast<unsigned long long*>(acc + 2 + j),
                      (unsigned long long)quantize(xr[j], a.scale_x[j]));
    }
    __syncthreads();
    for (int s = threadIdx.x; s < nslots; s += blockDim.x)
        if (sacc[s]) atomicAdd(reinterpret_cast<unsigned long long*>(a.totals + s), (unsigned long long)sacc[s]);
    for (int o = 16; o; o >>= 1) rescored += __shfl_xor_sync(0xffffffffu, rescored, o);
    if (lane == 0 && rescored)
        atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)rescored);
    if (bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
}

int64_t a256(int64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

int split_dp(int d) { return (d + 63) / 64 * 64; }
int split_kp(int k) { return (k + tc_block_n(k) - 1) / tc_block_n(k) * tc_block_n(k); }

size_t split_rows_bytes(int64_t n, int d) {
    const int64_t nn = n > 0 ? n : 1, dp = split_dp(d);
    return (size_t)(2 * a256(nn * dp * 2) + 2 * a256(nn * 4));
}

size_t split_centers_bytes(int d, int k) {
    const int64_t dp = split_dp(d), kp = split_kp(k);
    return (size_t)(256 + 2 * a256(kp * dp * 2) + a256(kp * 4));
}

RowSplit carve_rows(void* base, int64_t n, int d) {
    RowSplit s;
    const int64_t nn = n > 0 ? n : 1, dp = split_dp(d);
    char* p = static_cast<char*>(base);
    s.xh = p;
    s.xl = p + a256(nn * dp * 2);
    s.xn = reinterpret_cast<float*>(p + 2 * a256(nn * dp * 2));
    s.lab = reinterpret_cast<int32_t*>(p + 2 * a256(nn * dp * 2) + a256(nn * 4));
    return s;
}

CenterSplit carve_centers(void* base, int d, int k) {
    CenterSplit s;
    const int64_t dp = split_dp(d), kp = split_kp(k);
    char* p = static_cast<char*>(base);
    s.cmax_bits = reinterpret_cast<unsigned int*>(p);
    s.error = reinterpret_cast<int*>(p + 4);
    s.ch = p + 256;
    s.cl = p + 256 + a256(kp * dp * 2);
    s.hs = reinterpret_cast<float*>(p + 256 + 2 * a256(kp * dp * 2));
    return s;
}

cudaError_t launch_split_rows(const float* X, int64_t n, int d, const RowSplit& s, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    int64_t blocks = (n + kSplitThreads / 32 - 1) / (kSplitThreads / 32);
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    k_split_rows<<<(int)blocks, kSplitThreads, 0, st>>>(X, n, d, split_dp(d), static_cast<__nv_bfloat16*>(s.xh),
                                                         static_cast<__nv_bfloat16*>(s.xl), s.xn);
    return cudaGetLastError();
}

cudaError_t launch_split_centers(const float* C, int k, int d, const CenterSplit& s, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(s.cmax_bits, 0, 8, st);   // max |c| and the tensor-core error flag
    if (e != cudaSuccess) return e;
    const int kp = split_kp(k);
    const int blocks = (kp + kSplitThreads / 32 - 1) / (kSplitThreads / 32);
    k_split_centers<<<blocks, kSplitThreads, 0, st>>>(C, k, d, kp, split_dp(d), static_cast<__nv_bfloat16*>(s.ch),
                                                       static_cast<__nv_bfloat16*>(s.cl), s.hs, s.cmax_bits);
    return cudaGetLastError();
}

cudaError_t launch_accum_split(PassArgs a, const int32_t* lab, const int* tc_error, cudaStream_t st) {
    const int W = a.d + 2;
    a.smem_acc = (size_t)a.k * W * 8 <= 96 * 1024 ? 1 : 0;
    const size_t smem = a.smem_acc ? (size_t)a.k * W * 8 : 0;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(k_accum_split, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    int64_t blocks = (a.n + kSplitThreads - 1) / kSplitThreads;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_accum_split<<<(int)blocks, kSplitThreads, smem, st>>>(a, lab, tc_error);
    return cudaGetLastError();
}

}  // namespace kmc
