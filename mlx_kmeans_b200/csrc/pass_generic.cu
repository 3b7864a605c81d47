// pass_generic.cu -- column maxima, per-pass constants, and the any-shape assignment pass.
//
// Reference: core.py:2018-2197 (_gpu_pass) with the rows kernel of core.py:263-274 as its label
// semantics, and the accumulation of core.py:236-243 ([count, inertia, sums...] per cluster).
// This is the path for shapes no specialised kernel covers; it is exact for every (n, d, k) and
// every input, and the specialised kernels are checked against it as well as against the oracle.
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

// ---------------------------------------------------------------- column maxima
// Per-column max |x| as float bits (|x| bits order like the values; NaN bits sort above inf).
// The grid stride is a multiple of d, so each thread always reads the same column.
__global__ void k_colmax(const float* __restrict__ X, int64_t total, int d, int64_t stride,
                         unsigned int* __restrict__ colmax) {
    extern __shared__ unsigned int smax[];
    for (int j = threadIdx.x; j < d; j += blockDim.x) smax[j] = 0u;
    __syncthreads();
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t < stride) {
        unsigned int m = 0u;
        for (int64_t e = t; e < total; e += stride) {
            unsigned int b = __float_as_uint(X[e]) & 0x7fffffffu;
            m = b > m ? b : m;
        }
        atomicMax(&smax[(int)(t % d)], m);
    }
    __syncthreads();
    for (int j = threadIdx.x; j < d; j += blockDim.x)
        if (smax[j]) atomicMax(&colmax[j], smax[j]);
}

// ---------------------------------------------------------------- per-row bounds: drift of the centers
// Run by the prepare CTA after the constants.  The drift of center c is |c - c_prev| (float64, rounded up); the
// bounds lose max_c drift per pass (Hamerly: the distance to any other center shrinks by at most its move).
// The running total goes to the pass as float32 bounds on both sides; the current centers become c_prev.  When
// the bounds are not valid yet the pass writes them all, so they are valid afterwards with zero drift.
//
// It also writes each center's half separation (Hamerly's s(c)/2 test): hsep[c] = (s_c / 2)^2 rounded down, s_c the
// distance from c to its nearest other center (float64, rounded down; +inf when k = 1).  A row at distance u from its
// stored label's center l with u < s_l / 2 is closer to l than to any other center c, since |x - c| >= s_l - u > u
// (the triangle inequality) -- whatever the centers did since its bound was stored.
__device__ void bounds_prepare_cta(const float* __restrict__ C, int k, int d, double* __restrict__ meta,
                                   float* __restrict__ cprev, float* __restrict__ hsep, Prep* __restrict__ prep) {
    for (int c = threadIdx.x; c < k; c += blockDim.x) {
        double s2 = INFINITY;
        for (int o = 0; o < k; o++) {
            if (o == c) continue;
            double t = 0.0;
            for (int j = 0; j < d; j++) {
                const double q = (double)C[(int64_t)c * d + j] - (double)C[(int64_t)o * d + j];   // exact
                t = __fma_rd(q, q, t);
            }
            s2 = fmin(s2, t);
        }
        hsep[c] = __double2float_rd(0.25 * s2);
    }
    __shared__ double s_dmax[32];
    const bool valid = meta[1] != 0.0;
    double mx = 0.0;
    if (valid) {
        for (int c = threadIdx.x; c < k; c += blockDim.x) {
            double s = 0.0;
            for (int j = 0; j < d; j++) {
                double q = (double)C[(int64_t)c * d + j] - (double)cprev[(int64_t)c * d + j];
                s = __fma_ru(q, q, s);
            }
            mx = fmax(mx, __dsqrt_ru(s));
        }
    }
    for (int o = 16; o; o >>= 1) mx = fmax(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) s_dmax[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) mx = fmax(mx, s_dmax[w]);
        const double cum = valid ? __dadd_ru(meta[0], mx) : 0.0;
        prep->bvalid = valid ? 1 : 0;
        prep->bcum_lo = __double2float_rd(cum);
        prep->bcum_up = __double2float_ru(cum);
        meta[0] = cum;
        meta[1] = 1.0;
    }
    __syncthreads();
    for (int64_t e = threadIdx.x; e < (int64_t)k * d; e += blockDim.x) cprev[e] = C[e];
}

// ---------------------------------------------------------------- per-pass constants
// One CTA.  Screen constants per center, the fixed-point grids, and the window of the float32 screen; it also
// clears the pass's totals and counters (when given: small totals, else the caller clears them) and, for a
// bounded pass, updates the drift of the centers (bounds_prepare_cta).
//
// Screen: score_c = |c|^2/2 - x.c, an fma chain of d steps from h_c = |c|^2/2 (itself d fmas).
// |score_c(fp32) - score_c| <= 1.5 gamma_{d+1} (|x|^2 + |c|^2), gamma_n = n u / (1 - n u), u = 2^-24,
// and D(c) - D(c') = 2 (score_c - score_c').  When the best two screen scores are further apart than
// twice that bound (taken with max |c|^2, a 4/3 margin, and the float64 rounding of D64 added) the
// float32 winner is the float64 winner; otherwise the row is re-scored in float64.
__global__ void k_prepare(const float* __restrict__ C, int k, int d, const unsigned int* __restrict__ colmax,
                          int64_t n_total, Prep* __restrict__ prep, double* __restrict__ scale_x,
                          float* __restrict__ hc, long long* __restrict__ zero_totals, int zero_n,
                          long long* __restrict__ zero_counters, double* __restrict__ bmeta,
                          float* __restrict__ bcprev, float* __restrict__ bhsep, int rule,
                          const LoopState* __restrict__ loop) {
    __shared__ float s_max[32];
    __shared__ float s_cmax2[32];
    __shared__ int s_bad;
    pdl_wait();
    if (loop && loop->state != kLoopRunning) {        // the device loop stopped: this step does nothing
        if (threadIdx.x == 0) prep->skip = 1;
        return;
    }
    if (threadIdx.x == 0) s_bad = 0;
    if (zero_totals)
        for (int e = threadIdx.x; e < zero_n; e += blockDim.x) zero_totals[e] = 0;
    if (zero_counters && threadIdx.x < 8) zero_counters[threadIdx.x] = 0;
    __syncthreads();
    float mx = 0.0f, cm2 = 0.0f;
    int bad = 0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        unsigned int b = colmax[j];
        if (b >= 0x7f800000u) bad = 1;
        float v = __uint_as_float(b);
        mx = fmaxf(mx, v);
        scale_x[j] = ldexp(1.0, column_shift(v, n_total));
    }
    if (d >= 32) {
        // a warp per center, coalesced: lane chains of ceil(d/32) fmas and a five-level tree, within the
        // error of a d-step chain for every d >= 32
        const int lane = threadIdx.x & 31, nw = blockDim.x >> 5;
        for (int c = threadIdx.x >> 5; c < k; c += nw) {
            float s = 0.0f, m = 0.0f;
            for (int j = lane; j < d; j += 32) {
                const float v = C[(int64_t)c * d + j];
                if (!isfinite(v)) bad = 1;
                m = fmaxf(m, fabsf(v));
                s = __fmaf_rn(v, v, s);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {          // xor tree: every lane ends with the same sum
                s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
                m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            }
            if (lane == 0) hc[c] = 0.5f * s;
            mx = fmaxf(mx, m);
            cm2 = fmaxf(cm2, s);
        }
    } else {
        for (int c = threadIdx.x; c < k; c += blockDim.x) {
            float s = 0.0f;
            for (int j = 0; j < d; j++) {
                float v = C[(int64_t)c * d + j];
                if (!isfinite(v)) bad = 1;
                mx = fmaxf(mx, fabsf(v));
                s = __fmaf_rn(v, v, s);
            }
            hc[c] = 0.5f * s;
            cm2 = fmaxf(cm2, s);
        }
    }
    for (int o = 16; o; o >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        cm2 = fmaxf(cm2, __shfl_xor_sync(0xffffffffu, cm2, o));
    }
    if (bad) atomicOr(&s_bad, 1);
    if ((threadIdx.x & 31) == 0) { s_max[threadIdx.x >> 5] = mx; s_cmax2[threadIdx.x >> 5] = cm2; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) { mx = fmaxf(mx, s_max[w]); cm2 = fmaxf(cm2, s_cmax2[w]); }
        Prep p;
        double M = mx > 0.0f ? (double)mx : 1.1754943508222875e-38;
        double bound = 4.0 * (double)d * M * M * (1.0 + 1.0 / 1048576.0);     // >= any best32
        int L = ceil_log2((double)(n_total > 0 ? n_total : 1));
        int si = 61 - L - ceil_log2(bound);
        si = si > 1000 ? 1000 : (si < -1000 ? -1000 : si);
        p.si = si;
        p.scale_i = ldexp(1.0, si);
        p.inv_scale_i = ldexp(1.0, -si);
        p.cmax2 = cm2 * (1.0f + 1.0f / 1048576.0f);
        p.win_coef = (float)(4.0 * (d + 2) / 16777216.0 + (double)d / 281474976710656.0 + (rule ? rule32_coef(d) : 0.0));
        p.win_abs = (float)((d + 2) * 7.174648137343064e-43);               // (d+2) 2^-140
        p.flags = (s_bad || bound > 3.0e38) ? kFlagNonFinite : 0;
        p.bvalid = 0;
        p.bcum_lo = 0.0f;
        p.bcum_up = 0.0f;
        p.rule = rule;
        p.skip = 0;
        *prep = p;
    }
    if (bmeta) {
        __syncthreads();
        bounds_prepare_cta(C, k, d, bmeta, bcprev, bhsep, prep);
    }
}

// ---------------------------------------------------------------- the any-shape pass
// One thread per row.  DMAX > 0: the row is held in registers (d <= DMAX); DMAX == 0: read from L1.
// Centers stream through shared memory in tiles.  Accumulators: shared int64 slots when k*(d+2) fits,
// else the global totals directly.
template <int DMAX>
__global__ void __launch_bounds__(256) k_pass_generic(PassArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int d = a.d, k = a.k;
    const int W = d + 2;
    long long* sacc = reinterpret_cast<long long*>(smem_raw);
    const int nslots = a.smem_acc ? k * W : 0;
    float* ctile = reinterpret_cast<float*>(smem_raw + (size_t)nslots * 8);
    float* htile = ctile + (size_t)a.ctile * d;
    for (int s = threadIdx.x; s < nslots; s += blockDim.x) sacc[s] = 0;
    const Prep prep = *a.prep;
    if (prep.skip) return;
    const double scale_i = prep.scale_i;
    int rescored = 0, bad = 0;

    const int64_t rows_per_cta = (a.n + gridDim.x - 1) / gridDim.x;
    const int64_t r_begin = (int64_t)blockIdx.x * rows_per_cta;
    const int64_t r_end = min(a.n, r_begin + rows_per_cta);
    for (int64_t base = r_begin; base < r_end; base += blockDim.x) {
        const int64_t i = base + threadIdx.x;
        const bool live = i < r_end;
        const float* xr = a.X + (live ? i : r_begin) * (int64_t)d;
        float xreg[DMAX > 0 ? DMAX : 1];
        float x2 = 0.0f;
        if (DMAX > 0) {
#pragma unroll
            for (int j = 0; j < (DMAX > 0 ? DMAX : 1); j++) {
                xreg[j] = j < d ? xr[j] : 0.0f;
                x2 = __fmaf_rn(xreg[j], xreg[j], x2);
            }
        } else {
            for (int j = 0; j < d; j++) x2 = __fmaf_rn(xr[j], xr[j], x2);
        }
        float s1 = INFINITY, s2 = INFINITY;
        int l1 = 0;
        for (int c0 = 0; c0 < k; c0 += a.ctile) {
            const int ct = min(a.ctile, k - c0);
            __syncthreads();
            for (int e = threadIdx.x; e < ct * d; e += blockDim.x) ctile[e] = a.C[(int64_t)c0 * d + e];
            for (int e = threadIdx.x; e < ct; e += blockDim.x) htile[e] = a.hc[c0 + e];
            __syncthreads();
            for (int cc = 0; cc < ct; cc++) {
                const float* cr = ctile + (size_t)cc * d;
                float s = htile[cc];
                if (DMAX > 0) {
#pragma unroll
                    for (int j = 0; j < (DMAX > 0 ? DMAX : 1); j++)
                        if (j < d) s = __fmaf_rn(-xreg[j], cr[j], s);
                } else {
                    for (int j = 0; j < d; j++) s = __fmaf_rn(-xr[j], cr[j], s);
                }
                if (s < s1) { s2 = s1; s1 = s; l1 = c0 + cc; }
                else if (s < s2) s2 = s;
            }
        }
        if (!live) continue;
        int l = l1;
        const float win = __fmaf_rn(prep.win_coef, x2 + prep.cmax2, prep.win_abs);
        if (!(s2 - s1 > win)) {             // inside the window (or not finite): decide by the label rule
            double bd = INFINITY;
            int bl = 0;
            for (int c = 0; c < k; c++) {
                const double v = prep.rule ? (double)best32(xr, a.C + (int64_t)c * d, d)
                                           : d64_pairwise(xr, a.C + (int64_t)c * d, d);
                if (v < bd) { bd = v; bl = c; }
            }
            l = bl;
            rescored++;
        }
        const float* cl = a.C + (int64_t)l * d;
        float b = 0.0f;
        for (int j = 0; j < d; j++) b = best32_term(b, xr[j], cl[j]);
        if (!isfinite(b)) bad = 1;
        if (a.labels) a.labels[i] = l;
        if (a.best) a.best[i] = b;
        long long* acc = a.smem_acc ? sacc + (size_t)l * W : a.totals + (size_t)l * W;
        atomicAdd(reinterpret_cast<unsigned long long*>(acc), 1ull);
        atomicAdd(reinterpret_cast<unsigned long long*>(acc + 1), (unsigned long long)quantize(b, scale_i));
        for (int j = 0; j < d; j++)
            atomicAdd(reinterpret_cast<unsigned long long*>(acc + 2 + j),
                      (unsigned long long)quantize(xr[j], a.scale_x[j]));
    }
    __syncthreads();
    for (int s = threadIdx.x; s < nslots; s += blockDim.x)
        if (sacc[s]) atomicAdd(reinterpret_cast<unsigned long long*>(a.totals + s), (unsigned long long)sacc[s]);
    if (rescored) atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[0]), (unsigned long long)rescored);
    if (bad) atomicOr(reinterpret_cast<unsigned long long*>(&a.counters[1]), (unsigned long long)kFlagNonFinite);
}

// ---------------------------------------------------------------- launchers

cudaError_t launch_colmax(const float* X, int64_t n, int d, unsigned int* colmax, cudaStream_t st) {
    const int threads = 256;
    int64_t total = n * (int64_t)d;
    int64_t want = (int64_t)num_sms() * 8 * threads;
    int64_t stride = (want / d) * d;
    if (stride < d) stride = d;
    if (stride > total) stride = ((total + d - 1) / d) * d;
    int blocks = (int)((stride + threads - 1) / threads);
    k_colmax<<<blocks, threads, sizeof(unsigned int) * d, st>>>(X, total, d, stride, colmax);
    return cudaGetLastError();
}

cudaError_t launch_prepare(const float* C, int k, int d, const unsigned int* colmax, int64_t n_total, Prep* prep,
                           double* scale_x, float* hc, long long* zero_totals, long long* zero_counters,
                           double* bmeta, float* bcprev, float* bhsep, int rule, cudaStream_t st,
                           const void* loop) {
    const int64_t zn = (int64_t)k * (d + 2);
    if (zero_totals && zn > 16384 && !loop) {  // large totals: a memset is faster than one CTA
        cudaError_t e = cudaMemsetAsync(zero_totals, 0, sizeof(long long) * (size_t)zn, st);
        if (e != cudaSuccess) return e;
        zero_totals = nullptr;
    }
    return launch_pdl(k_prepare, dim3(1), dim3(1024), 0, st, C, k, d, colmax, n_total, prep, scale_x, hc, zero_totals,
                      (int)zn, zero_counters, bmeta, bcprev, bhsep, rule, static_cast<const LoopState*>(loop));
}

cudaError_t launch_pass_generic(PassArgs a, cudaStream_t st) {
    const int W = a.d + 2;
    const size_t budget = 200 * 1024;
    a.smem_acc = (size_t)a.k * W * 8 <= 96 * 1024 ? 1 : 0;
    size_t acc_bytes = a.smem_acc ? (size_t)a.k * W * 8 : 0;
    size_t per_center = (size_t)(a.d + 1) * 4;
    size_t room = budget - acc_bytes;
    int ct = (int)(room / per_center);
    if (ct > a.k) ct = a.k;
    if (ct > 1024) ct = 1024;
    if (ct < 1) return cudaErrorInvalidValue;
    a.ctile = ct;
    size_t smem = acc_bytes + (size_t)ct * per_center;
    const int threads = 256;
    int64_t blocks64 = (a.n + threads - 1) / threads;
    int cap = num_sms() * (a.smem_acc ? 2 : 4);
    int blocks = (int)(blocks64 < cap ? blocks64 : cap);
    if (blocks < 1) blocks = 1;
    cudaError_t e;
#define KMC_GENERIC_CASE(DM)                                                                            \
    e = cudaFuncSetAttribute(k_pass_generic<DM>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e != cudaSuccess) return e;                                                                     \
    k_pass_generic<DM><<<blocks, threads, smem, st>>>(a);
    if (a.d <= 8) { KMC_GENERIC_CASE(8) }
    else if (a.d <= 16) { KMC_GENERIC_CASE(16) }
    else if (a.d <= 32) { KMC_GENERIC_CASE(32) }
    else if (a.d <= 64) { KMC_GENERIC_CASE(64) }
    else { KMC_GENERIC_CASE(0) }
#undef KMC_GENERIC_CASE
    return cudaGetLastError();
}

}  // namespace kmc
