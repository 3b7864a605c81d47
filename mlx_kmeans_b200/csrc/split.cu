// split.cu -- the operands and the totals of the tensor-core pass (d >= 32).
//
//   k_split_rows     once per dataset slice: x = xh + xl (bf16 hi / lo, row-major, columns padded to a
//                    multiple of 64 with zeros) and |x| rounded up, for assign_tc.cu
//   k_split_centers  once per pass: the same split of the centers (rows padded to the MMA tile), |c|^2/2 and
//                    max |c| (rounded up)
//   k_flag_list      the rows assign_tc.cu flagged (label bit 31), listed (staged per CTA in shared memory)
//   k_decide_cands   their decision by the label rule (NumPy-pairwise D64 of the two candidate centers, a thread
//                    per row for d <= 128, a warp per row beyond; or the float32 direct sum), lowest index on
//                    ties; rows with more candidates:
//   k_rescore_tc     one CTA per row: a float32 screen of every center, then the label rule's distance of each
//                    center in its window
//   k_fix_labels     per row: the histogram of the labels; the optional labels / best outputs (best: the
//                    reference's float32 distance, each operation rounded on its own, in column order)
//   k_scan_labels, k_scatter_rows   the rows grouped by label (a counting sort; the labels in grouped order too)
//   k_reduce_slab    d % 4 == 0: the grouped rows streamed by cp.async in column slabs, every value quantised on
//                    its own into lane-private int64 sums, flushed to the global totals when the label changes, so
//                    the totals are exact integers whatever the order (and equal to the CUDA-core pass's); inertia
//                    from each (row, lane) float64 partial distance, quantised the same way
//   k_reduce_rows    the same for any d, one warp per run of 256 grouped rows
//
// Reference: the high-d exact path of core.py:289-377 / 675-844, its sorted accumulation for large k
// (core.py:1292-1441, mx.argsort grouping at 976-987), and the label rule of core.py:263-274.
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
                                                             float* __restrict__ xn, float* __restrict__ xsq_lo) {
    const int lane = threadIdx.x & 31;
    const int64_t warps = (int64_t)gridDim.x * (kSplitThreads / 32);
    for (int64_t r = (int64_t)blockIdx.x * (kSplitThreads / 32) + (threadIdx.x >> 5); r < n; r += warps) {
        const float* x = X + r * d;
        double s = 0.0, sd = 0.0;                         // |x|^2 rounded up and rounded down
        for (int j = lane; j < dp; j += 32) {
            const float v = j < d ? x[j] : 0.0f;
            __nv_bfloat16 h, l;
            split_bf16(v, h, l);
            xh[r * dp + j] = h;
            xl[r * dp + j] = l;
            s = __fma_ru((double)v, (double)v, s);
            sd = __fma_rd((double)v, (double)v, sd);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            s = __dadd_ru(s, __shfl_xor_sync(0xffffffffu, s, o));
            sd = __dadd_rd(sd, __shfl_xor_sync(0xffffffffu, sd, o));
        }
        if (lane == 0) {
            xn[r] = __double2float_ru(__dsqrt_ru(s));
            xsq_lo[r] = __double2float_rd(sd);
        }
    }
}

// one warp per (padded) center: halves, |c|^2 / 2 (float64, rounded to nearest float; padding 2^126), max |c|
__global__ void __launch_bounds__(kSplitThreads) k_split_centers(const float* __restrict__ C, int k, int d, int kp,
                                                                int dp, __nv_bfloat16* __restrict__ ch,
                                                                __nv_bfloat16* __restrict__ cl,
                                                                float* __restrict__ hs,
                                                                unsigned int* __restrict__ cmax_bits,
                                                                float* __restrict__ ct) {
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
            if (real && j < d) ct[(int64_t)j * k + c] = v;
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

// The rows the tensor-core kernel flagged (label bit 31), listed by a coalesced scan of the labels: each CTA
// takes kFlagRows rows, stages its flagged rows in shared memory (room for all of them) and reserves their
// places in the global lists with one atomic per list; the rows with more than two candidates go straight to
// the overflow list.
constexpr int kSplitWarps = kSplitThreads / 32;
constexpr int kFlagRows = 4096;
__global__ void __launch_bounds__(kSplitThreads) k_flag_list(const int32_t* __restrict__ lab, int64_t n,
                                                            const int4* __restrict__ cands,
                                                            const int* __restrict__ tc_error,
                                                            uint32_t* __restrict__ list, unsigned int* __restrict__ nlist,
                                                            uint32_t* __restrict__ ovf, unsigned int* __restrict__ novf,
                                                            long long* __restrict__ counters) {
    __shared__ uint32_t s_list[kFlagRows], s_ovf[kFlagRows];
    __shared__ unsigned s_nl, s_no, s_at_l, s_at_o;
    if (*tc_error) return;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (threadIdx.x == 0) s_nl = s_no = 0u;
    __syncthreads();
    constexpr int kPerWarp = kFlagRows / kSplitWarps;       // 512 rows: 16 chunks of 32, loaded 4 at a time
    const int64_t w0 = (int64_t)blockIdx.x * kFlagRows + (int64_t)warp * kPerWarp;
    for (int c0 = 0; c0 < kPerWarp; c0 += 4 * 32) {
        int32_t lv[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int64_t row = w0 + c0 + q * 32 + lane;
            lv[q] = row < n ? lab[row] : 0;
        }
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int64_t row = w0 + c0 + q * 32 + lane;
            const bool f = lv[q] < 0;
            const bool over = f && cands[row].w == -2;
            const unsigned fm = __ballot_sync(0xffffffffu, f && !over), om = __ballot_sync(0xffffffffu, over);
            const unsigned below = (1u << lane) - 1u;
            if (fm) {
                unsigned at = 0;
                if (lane == 0) at = atomicAdd(&s_nl, (unsigned)__popc(fm));
                at = __shfl_sync(0xffffffffu, at, 0);
                if (f && !over) s_list[at + __popc(fm & below)] = (uint32_t)row;
            }
            if (om) {
                unsigned at = 0;
                if (lane == 0) at = atomicAdd(&s_no, (unsigned)__popc(om));
                at = __shfl_sync(0xffffffffu, at, 0);
                if (over) s_ovf[at + __popc(om & below)] = (uint32_t)row;
            }
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        s_at_l = s_nl ? atomicAdd(nlist, s_nl) : 0u;
        s_at_o = s_no ? atomicAdd(novf, s_no) : 0u;
        if (s_nl + s_no)
            atomicAdd(reinterpret_cast<unsigned long long*>(&counters[0]), (unsigned long long)(s_nl + s_no));
    }
    __syncthreads();
    for (unsigned e = threadIdx.x; e < s_nl; e += kSplitThreads) list[s_at_l + e] = s_list[e];
    for (unsigned e = threadIdx.x; e < s_no; e += kSplitThreads) ovf[s_at_o + e] = s_ovf[e];
}

// The listed rows: the float64 distance (NumPy-pairwise D64) of each of a row's (two) candidate centers; the
// smallest, lowest index on ties, is the label.  d <= 128 (one leaf of the pairwise tree): a thread per row;
// longer rows: a warp per row (d64_warp).
__global__ void __launch_bounds__(kSplitThreads) k_decide_cands(const float* __restrict__ X, int d,
                                                               const float* __restrict__ C,
                                                               const uint32_t* __restrict__ list,
                                                               const unsigned int* __restrict__ nlist,
                                                               const int4* __restrict__ cands,
                                                               const int* __restrict__ tc_error,
                                                               const Prep* __restrict__ prep,
                                                               int32_t* __restrict__ lab) {
    __shared__ __align__(8) unsigned char scratch[kSplitWarps][kD64WarpScratch];
    if (*tc_error) return;
    const int64_t cnt = *nlist;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rule = prep->rule;
    const bool wide = d > 128;
    const int64_t per = wide ? (int64_t)gridDim.x * kSplitWarps : (int64_t)gridDim.x * kSplitThreads;
    const int64_t first = wide ? (int64_t)blockIdx.x * kSplitWarps + warp : (int64_t)blockIdx.x * kSplitThreads + threadIdx.x;
    for (int64_t f = first; f < cnt; f += per) {
        const int64_t row = list[f];
        const int4 c4 = cands[row];
        const float* x = X + row * d;
        const int cs[4] = {c4.x, c4.y, c4.z, c4.w};
        double bv = INFINITY;
        int bi = c4.x;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            if (cs[i] < 0) continue;
            // (the float32 label rule's direct sum is sequential: every lane of a wide row computes it alike)
            const double v = rule ? (double)best32(x, C + (int64_t)cs[i] * d, d)
                             : wide ? d64_warp(x, C + (int64_t)cs[i] * d, d, scratch[warp])
                                    : d64_pairwise(x, C + (int64_t)cs[i] * d, d);
            if (v < bv || (v == bv && cs[i] < bi)) { bv = v; bi = cs[i]; }
        }
        if (!wide || lane == 0) lab[row] = bi;
    }
}

// The rows the tensor-core kernel could not decide from two candidates, one CTA per row: a float32 screen of all scores
// hc_c - x.c (an FMA chain from hc over the columns in order: the CUDA-core pass's form and error window;
// the transposed centers make the loads coalesced), then the float64 distance (NumPy-pairwise D64) of every
// center within the window of the smallest score; the smallest D64, lowest index on ties, is the label.
// If the tensor-core kernel gave up, every row is decided here.
constexpr int kRescoreThreads = 256;
constexpr int kRescoreList = 1024;       // window candidates decided a warp each; more: a thread each
__global__ void __launch_bounds__(kRescoreThreads) k_rescore_tc(const float* __restrict__ X, int64_t n, int d,
                                                               const float* __restrict__ C,
                                                               const float* __restrict__ ct,
                                                               const float* __restrict__ hc, int k,
                                                               const Prep* __restrict__ prep_p,
                                                               const uint32_t* __restrict__ list,
                                                               const unsigned int* __restrict__ nlist,
                                                               const int* __restrict__ tc_error,
                                                               int32_t* __restrict__ lab,
                                                               long long* __restrict__ counters) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    float* xs = reinterpret_cast<float*>(smem_raw);                 // d
    float* sc = xs + d;                                              // k scores
    __shared__ int cl[kRescoreList];                                 // the centers inside the window
    __shared__ __align__(8) unsigned char scratch[kRescoreThreads / 32][kD64WarpScratch];
    __shared__ int s_nc;
    __shared__ float rmin[kRescoreThreads / 32];
    __shared__ double rbv[kRescoreThreads / 32];
    __shared__ int rbi[kRescoreThreads / 32];
    __shared__ float sx2;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const Prep prep = *prep_p;
    const bool all = *tc_error != 0;
    const int64_t cnt = all ? n : (int64_t)*nlist;
    for (int64_t f = blockIdx.x; f < cnt; f += gridDim.x) {
        const int64_t row = all ? f : (int64_t)list[f];
        const float* x = X + row * d;
        for (int j = tid; j < d; j += kRescoreThreads) xs[j] = x[j];
        __syncthreads();
        if (tid == 0) {
            float x2 = 0.0f;
            for (int j = 0; j < d; j++) x2 = __fmaf_rn(xs[j], xs[j], x2);
            sx2 = x2;
        }
        float m = INFINITY;
        // four of the thread's centers at a time: four independent chains (each in column order from hc, as the
        // window assumes) and four coalesced loads per column
        for (int c0 = tid; c0 < k; c0 += 4 * kRescoreThreads) {
            float v[4];
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int c = c0 + i * kRescoreThreads;
                v[i] = c < k ? hc[c] : 0.0f;
            }
#pragma unroll 4
            for (int j = 0; j < d; j++) {
                const float xj = -xs[j];
                const float* row = ct + (int64_t)j * k;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const int c = c0 + i * kRescoreThreads;
                    if (c < k) v[i] = __fmaf_rn(xj, row[c], v[i]);
                }
            }
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int c = c0 + i * kRescoreThreads;
                if (c < k) {
                    sc[c] = v[i];
                    m = fminf(m, v[i]);
                }
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fminf(m, __shfl_xor_sync(0xffffffffu, m, o));
        if (lane == 0) rmin[warp] = m;
        __syncthreads();
        m = rmin[0];
        for (int w = 1; w < kRescoreThreads / 32; w++) m = fminf(m, rmin[w]);
        const float lim = m + __fmaf_rn(prep.win_coef, sx2 + prep.cmax2, prep.win_abs);
        if (tid == 0) s_nc = 0;
        __syncthreads();
        for (int c = tid; c < k; c += kRescoreThreads) {
            if (!(sc[c] > lim)) {                                      // (a NaN score is a candidate too)
                const int e = atomicAdd(&s_nc, 1);
                if (e < kRescoreList) cl[e] = c;
            }
        }
        __syncthreads();
        const int nc = s_nc;
        double bv = INFINITY;
        int bi = 0x7fffffff;
        if (nc <= kRescoreList) {
            // a warp per candidate (the list's order does not matter: smallest D64, then lowest index)
            for (int e = warp; e < nc; e += kRescoreThreads / 32) {
                const int c = cl[e];
                const double v = prep.rule ? (double)best32(xs, C + (int64_t)c * d, d)
                                           : d64_warp(xs, C + (int64_t)c * d, d, scratch[warp]);
                if (v < bv || (v == bv && c < bi)) { bv = v; bi = c; }
            }
        } else {
            for (int c = tid; c < k; c += kRescoreThreads) {
                if (sc[c] > lim) continue;
                const double v = prep.rule ? (double)best32(xs, C + (int64_t)c * d, d)
                                           : d64_pairwise(xs, C + (int64_t)c * d, d);
                if (v < bv || (v == bv && c < bi)) { bv = v; bi = c; }
            }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const double ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov < bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (lane == 0) { rbv[warp] = bv; rbi[warp] = bi; }
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < kRescoreThreads / 32; w++)
                if (rbv[w] < bv || (rbv[w] == bv && rbi[w] < bi)) { bv = rbv[w]; bi = rbi[w]; }
            lab[row] = bi == 0x7fffffff ? 0 : bi;
        }
        __syncthreads();
    }
    if (all && blockIdx.x == 0 && tid == 0 && cnt)
        atomicAdd(reinterpret_cast<unsigned long long*>(&counters[0]), (unsigned long long)cnt);
}

constexpr int kHistMax = 8192;           // labels counted in shared memory up to this k
constexpr int kRun = 256;                // grouped rows per warp in k_reduce_rows
constexpr int kReduceWarps = 8;

// one thread per row: the histogram of the final labels and the optional labels / best outputs
__global__ void __launch_bounds__(kSplitThreads) k_fix_labels(const float* __restrict__ X, int64_t n, int d,
                                                             const float* __restrict__ C, int k,
                                                             const int32_t* __restrict__ lab,
                                                             unsigned int* __restrict__ hist,
                                                             int32_t* __restrict__ labels_out,
                                                             float* __restrict__ best_out) {
    __shared__ unsigned int sh[kHistMax];
    const bool local = k <= kHistMax;
    if (local)
        for (int c = threadIdx.x; c < k; c += blockDim.x) sh[c] = 0u;
    __syncthreads();
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n; i0 += 4 * stride) {
        int lv[4];                                  // four rows' labels loaded before any is counted
#pragma unroll
        for (int q = 0; q < 4; q++) lv[q] = i0 + q * stride < n ? lab[i0 + q * stride] : -1;
#pragma unroll
        for (int q = 0; q < 4; q++) {
            const int64_t i = i0 + q * stride;
            const int l = lv[q];
            if (l < 0) continue;
            if (local) atomicAdd(&sh[l], 1u);
            else atomicAdd(&hist[l], 1u);
            if (labels_out) labels_out[i] = l;
            if (best_out) {
                const float* xr = X + i * d;
                const float* cr = C + (int64_t)l * d;
                float b = 0.0f;
                for (int j = 0; j < d; j++) b = best32_term(b, xr[j], cr[j]);
                best_out[i] = b;
            }
        }
    }
    __syncthreads();
    if (local)
        for (int c = threadIdx.x; c < k; c += blockDim.x)
            if (sh[c]) atomicAdd(&hist[c], sh[c]);
}

// one CTA: exclusive prefix sum of the label counts -> each label's first slot (the scatter's cursors)
__global__ void __launch_bounds__(1024) k_scan_labels(const unsigned int* __restrict__ hist, int k,
                                                      unsigned int* __restrict__ cursor) {
    __shared__ unsigned int part[1024];
    const int t = threadIdx.x;
    const int per = (k + 1023) / 1024;
    const int lo = min(k, t * per), hi = min(k, lo + per);
    unsigned int s = 0;
    for (int c = lo; c < hi; c++) s += hist[c];
    part[t] = s;
    __syncthreads();
    for (int o = 1; o < 1024; o <<= 1) {     // inclusive Hillis-Steele scan of the per-thread sums
        const unsigned int v = t >= o ? part[t - o] : 0u;
        __syncthreads();
        part[t] += v;
        __syncthreads();
    }
    unsigned int run = t ? part[t - 1] : 0u;
    for (int c = lo; c < hi; c++) {
        cursor[c] = run;
        run += hist[c];
    }
}

// Rows grouped by label.  Per CTA and chunk of kScatterRows rows: a shared histogram, one global atomic per
// label present to reserve its slots, then each row's place in them (k above kScatterMax: one global atomic
// per row).  The order inside a label is not fixed; the totals do not depend on it.
constexpr int kScatterRows = 8192;
constexpr int kScatterMax = 4096;
__global__ void __launch_bounds__(kSplitThreads) k_scatter_rows(const int32_t* __restrict__ lab, int64_t n, int k,
                                                               unsigned int* __restrict__ cursor,
                                                               uint32_t* __restrict__ perm,
                                                               int32_t* __restrict__ glab) {
    __shared__ unsigned int cnt[kScatterMax];
    __shared__ unsigned int at[kScatterMax];
    const bool local = k <= kScatterMax;
    for (int64_t c0 = (int64_t)blockIdx.x * kScatterRows; c0 < n; c0 += (int64_t)gridDim.x * kScatterRows) {
        const int64_t c1 = min(n, c0 + kScatterRows);
        if (!local) {
            for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
                const int l = lab[i];
                const unsigned pos = atomicAdd(&cursor[l], 1u);
                perm[pos] = (uint32_t)i;
                glab[pos] = l;
            }
            continue;
        }
        for (int c = threadIdx.x; c < k; c += blockDim.x) cnt[c] = 0u;
        __syncthreads();
        for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) atomicAdd(&cnt[lab[i]], 1u);
        __syncthreads();
        for (int c = threadIdx.x; c < k; c += blockDim.x) {
            at[c] = cnt[c] ? atomicAdd(&cursor[c], cnt[c]) : 0u;
            cnt[c] = 0u;
        }
        __syncthreads();
        for (int64_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
            const int l = lab[i];
            const unsigned pos = at[l] + atomicAdd(&cnt[l], 1u);
            perm[pos] = (uint32_t)i;
            glab[pos] = l;
        }
        __syncthreads();
    }
}

// One warp per run of kRun grouped rows.  Lane-private int64 sums of column j = lane + 32 m live in shared
// memory (d per warp); they go to the global totals (one atomic per column) whenever the label changes.  The
// inertia is each row's float64 squared distance, quantised per (row, lane) partial: integer sums, so no order
// matters.  Rows are taken 8 at a time (their indices and labels in one load each), and for d <= 32 * XR the
// 8 rows' values are loaded before any is used.
template <int XR>
__global__ void __launch_bounds__(32 * kReduceWarps) k_reduce_rows(const float* __restrict__ X, int64_t n, int d,
                                                                  const float* __restrict__ C,
                                                                  const int32_t* __restrict__ lab,
                                                                  const uint32_t* __restrict__ perm,
                                                                  const double* __restrict__ scale_x,
                                                                  const Prep* __restrict__ prep,
                                                                  long long* __restrict__ totals,
                                                                  long long* __restrict__ counters) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    long long* acc = reinterpret_cast<long long*>(smem_raw) + (size_t)warp * d;
    for (int j = lane; j < d; j += 32) acc[j] = 0;
    const double scale_i = prep->scale_i;
    const int W = d + 2;
    bool bad = false;
    const int64_t runs = (n + kRun - 1) / kRun;
    for (int64_t run = (int64_t)blockIdx.x * kReduceWarps + warp; run < runs;
         run += (int64_t)gridDim.x * kReduceWarps) {
        const int64_t r0 = run * kRun, r1 = min(n, r0 + kRun);
        int cur = -1;
        long long cnt = 0, iq = 0;
        auto flush = [&]() {
            if (cur < 0) return;
            long long* t = totals + (size_t)cur * W;
            for (int j = lane; j < d; j += 32) {
                if (acc[j]) atomicAdd(reinterpret_cast<unsigned long long*>(t + 2 + j), (unsigned long long)acc[j]);
                acc[j] = 0;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) iq += __shfl_xor_sync(0xffffffffu, iq, o);
            if (lane == 0) {
                atomicAdd(reinterpret_cast<unsigned long long*>(t), (unsigned long long)cnt);
                if (iq) atomicAdd(reinterpret_cast<unsigned long long*>(t + 1), (unsigned long long)iq);
            }
            cnt = 0;
            iq = 0;
        };
        auto add = [&](const float* x, const float* c, int j, float v) {
            acc[j] += quantize(v, scale_x[j]);
            const double q = (double)v - (double)c[j];
            return q * q;
        };
        for (int64_t r = r0; r < r1; r += 8) {
            const int m = (int)min((int64_t)8, r1 - r);
            const uint32_t pr = lane < m ? perm[r + lane] : 0u;
            const int pl = lane < m ? lab[pr] : 0;
            float xv[8][XR > 0 ? XR : 1];
            if constexpr (XR > 0) {
#pragma unroll
                for (int u = 0; u < 8; u++) {
                    const int64_t row = __shfl_sync(0xffffffffu, pr, u);
#pragma unroll
                    for (int t = 0; t < XR; t++) {
                        const int j = lane + 32 * t;
                        xv[u][t] = (u < m && j < d) ? X[row * d + j] : 0.0f;
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < 8; u++) {          // unrolled, so xv stays in registers
                if (u >= m) break;
                const int64_t row = __shfl_sync(0xffffffffu, pr, u);
                const int l = __shfl_sync(0xffffffffu, pl, u);
                if (l != cur) {
                    flush();
                    cur = l;
                }
                const float* x = X + row * d;
                const float* c = C + (int64_t)l * d;
                double b = 0.0;
                if constexpr (XR > 0) {
#pragma unroll
                    for (int t = 0; t < XR; t++) {
                        const int j = lane + 32 * t;
                        if (j < d) b += add(x, c, j, xv[u][t]);
                    }
                } else {
                    for (int j = lane; j < d; j += 32) b += add(x, c, j, x[j]);
                }
                if (!(b <= 1.0e300)) bad = true;
                else iq += __double2ll_rn(__dmul_rn(b, scale_i));
                cnt++;
            }
        }
        flush();
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0)
        atomicOr(reinterpret_cast<unsigned long long*>(&counters[1]), (unsigned long long)kFlagNonFinite);
}

// Rows of d % 4 == 0 columns (X 16-byte aligned) as float4 groups.  A work item is a stretch of G * kSlabRows
// grouped rows and a slab of SW = 4 LPR V columns: LPR lanes per row and G = 32 / LPR rows side by side (group g
// takes the g-th kSlabRows rows of the stretch); lane i of a group owns the column groups i + LPR t (t < V) of
// the slab.  The rows' values stream into shared memory by cp.async, kSlabStages chunks of U rows ahead (each
// lane copies and later reads only its own float4s; the grouped labels go through a per-warp table).  Per
// group: the current label's center in registers (float64), lane-private int64 sums in registers, flushed to
// the totals when the label changes and at the end of the item.  Each value is quantised on its own, as in
// k_reduce_rows, so the totals are the same integers.  MAGIC (n_total >= 2048: every quantised value is below
// 2^50 in magnitude): v * 2^s is rounded to an integer by adding 1.5 * 2^52 inside the fma and the bits of the
// sum are accumulated; the count times the constant's bits comes off at the flush (modulo 2^64, the true sum
// being below 2^61).  The inertia is each (row, lane) float64 partial, quantised the same way.
constexpr int kSlabRows = 256;
constexpr int kSlabStages = 4;
constexpr int kSlabThreads = 128;
constexpr double kMagic = 6755399441055744.0;                  // 1.5 * 2^52
constexpr unsigned long long kMagicBits = 0x4338000000000000ull;

constexpr int slab_rows_in_flight(int lpr, int v) { return v == 1 ? (lpr < 8 ? lpr : 8) : 4; }
constexpr size_t slab_smem(int lpr, int v) {
    return (size_t)(kSlabThreads / 32) * kSlabStages * slab_rows_in_flight(lpr, v) * v * 32 * 16;
}

__device__ __forceinline__ void cp_async16(unsigned dst, const void* src, int bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }
__device__ __forceinline__ float f4_at(const float4& v, int e) { return e == 0 ? v.x : e == 1 ? v.y : e == 2 ? v.z : v.w; }

template <int LPR, int V, bool MAGIC>
__global__ void __launch_bounds__(kSlabThreads) k_reduce_slab(const float* __restrict__ X, int64_t n, int d,
                                                              const float* __restrict__ C,
                                                              const int32_t* __restrict__ glab,
                                                              const uint32_t* __restrict__ perm,
                                                              const double* __restrict__ scale_x,
                                                              const Prep* __restrict__ prep,
                                                              long long* __restrict__ totals,
                                                              long long* __restrict__ counters) {
    constexpr int G = 32 / LPR;
    constexpr int U = slab_rows_in_flight(LPR, V);             // rows per group and chunk
    constexpr int P = kSlabStages;
    constexpr int NCH = kSlabRows / U;
    constexpr int SW = 4 * LPR * V;
    static_assert(G * U <= 32 && kSlabRows % U == 0, "slab layout");
    extern __shared__ __align__(16) float4 slab_buf[];
    __shared__ int s_lbl[kSlabThreads / 32][P][32];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane / LPR, i = lane % LPR;
    float4* xs = slab_buf + (size_t)warp * P * U * V * 32;
    const unsigned xs_s = (unsigned)__cvta_generic_to_shared(xs);
    const int W = d + 2;
    const double scale_i = prep->scale_i;
    const int nslab = (d + SW - 1) / SW;
    const int64_t span = (int64_t)G * kSlabRows;
    const int64_t items = (n + span - 1) / span * nslab;
    const int64_t nwarps = ((int64_t)gridDim.x * kSlabThreads) >> 5;
    bool bad = false;
    for (int64_t item = ((int64_t)blockIdx.x * kSlabThreads + threadIdx.x) >> 5; item < items; item += nwarps) {
        const int z = (int)(item % nslab);
        const int64_t s0 = (item / nslab) * span + (int64_t)g * kSlabRows;
        const int64_t s1 = min(n, s0 + kSlabRows);
        int jc[V];
        double sc[V][4], cd[V][4];
        unsigned long long acc[V][4];
#pragma unroll
        for (int t = 0; t < V; t++) {
            jc[t] = z * SW + 4 * (i + LPR * t);
#pragma unroll
            for (int e = 0; e < 4; e++) {
                sc[t][e] = jc[t] < d ? scale_x[jc[t] + e] : 0.0;
                cd[t][e] = 0.0;
                acc[t][e] = 0ull;
            }
        }
        int cur = -1;
        long long cnt = 0, iq = 0;
        auto flush = [&]() {
            if (cur < 0) return;
            long long* tt = totals + (size_t)cur * W;
#pragma unroll
            for (int t = 0; t < V; t++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    const long long v = MAGIC ? (long long)(acc[t][e] - (unsigned long long)cnt * kMagicBits)
                                              : (long long)acc[t][e];
                    if (jc[t] < d && v) atomicAdd(reinterpret_cast<unsigned long long*>(tt + 2 + jc[t] + e),
                                                  (unsigned long long)v);
                    acc[t][e] = 0ull;
                }
            }
            if (z == 0 && i == 0) atomicAdd(reinterpret_cast<unsigned long long*>(tt), (unsigned long long)cnt);
            if (iq) atomicAdd(reinterpret_cast<unsigned long long*>(tt + 1), (unsigned long long)iq);
            cnt = 0;
            iq = 0;
        };
        // lane i < U of a group holds the index and label of row i of a chunk
        auto load_idx = [&](int c, uint32_t& pr, int& pl) {
            const int64_t pos = s0 + (int64_t)c * U + i;
            const bool ok = i < U && c < NCH && pos < s1;
            pr = ok ? perm[pos] : 0u;
            pl = ok ? glab[pos] : -1;
        };
        // chunk c into stage c % P (an empty group past the last chunk keeps the group count uniform)
        auto issue = [&](int c, uint32_t pr, int pl) {
            const int st = c % P;
            if (i < U) s_lbl[warp][st][g * U + i] = pl;
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int64_t row = __shfl_sync(0xffffffffu, pr, g * LPR + u);
                const bool valid = c < NCH && s0 + (int64_t)c * U + u < s1;
#pragma unroll
                for (int t = 0; t < V; t++) {
                    const bool live = valid && jc[t] < d;
                    cp_async16(xs_s + (unsigned)((((st * U + u) * V + t) * 32 + lane) * 16),
                               live ? (const void*)(X + row * d + jc[t]) : (const void*)X, live ? 16 : 0);
                }
            }
            cp_async_commit();
        };
        {
            uint32_t pr0[P + 1];
            int pl0[P + 1];
#pragma unroll
            for (int c = 0; c <= P; c++) load_idx(c, pr0[c], pl0[c]);
            __syncwarp();                      // the previous item's last reads of the label table are done
#pragma unroll
            for (int c = 0; c < P; c++) issue(c, pr0[c], pl0[c]);
            uint32_t pr = pr0[P];
            int pl = pl0[P];
            for (int c = 0; c < NCH; c++) {
                cp_async_wait<P - 1>();        // this lane's copies of chunk c have landed
                __syncwarp();                  // and every lane's labels of it
                const int st = c % P;
#pragma unroll
                for (int u = 0; u < U; u++) {
                    if (!(s0 + (int64_t)c * U + u < s1)) continue;
                    const int l = s_lbl[warp][st][g * U + u];
                    if (l != cur) {
                        flush();
                        cur = l;
#pragma unroll
                        for (int t = 0; t < V; t++)
#pragma unroll
                            for (int e = 0; e < 4; e++)
                                cd[t][e] = jc[t] < d ? (double)C[(int64_t)l * d + jc[t] + e] : 0.0;
                    }
                    double b = 0.0;
#pragma unroll
                    for (int t = 0; t < V; t++) {
                        const float4 xv = xs[((st * U + u) * V + t) * 32 + lane];
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const double v = (double)f4_at(xv, e);
                            if constexpr (MAGIC)
                                acc[t][e] += (unsigned long long)__double_as_longlong(__fma_rn(v, sc[t][e], kMagic));
                            else
                                acc[t][e] += (unsigned long long)__double2ll_rn(__dmul_rn(v, sc[t][e]));
                            const double q = __dsub_rn(v, cd[t][e]);
                            b = __fma_rn(q, q, b);
                        }
                    }
                    if (!(b <= 1.0e300)) bad = true;
                    else if constexpr (MAGIC)
                        iq += (long long)((unsigned long long)__double_as_longlong(__fma_rn(b, scale_i, kMagic)) -
                                          kMagicBits);
                    else
                        iq += __double2ll_rn(__dmul_rn(b, scale_i));
                    cnt++;
                }
                __syncwarp();                  // stage c % P is read: it takes chunk c + P
                issue(c + P, pr, pl);
                load_idx(c + P + 1, pr, pl);
            }
            cp_async_wait<0>();                // (the trailing empty chunks) before the next item's copies
        }
        flush();
    }
    cp_async_wait<0>();
    if (__any_sync(0xffffffffu, bad) && lane == 0)
        atomicOr(reinterpret_cast<unsigned long long*>(&counters[1]), (unsigned long long)kFlagNonFinite);
}

int64_t a256(int64_t v) { return (v + 255) / 256 * 256; }

}  // namespace

int split_dp(int d) { return (d + 63) / 64 * 64; }
int split_kp(int k) { return (k + tc_block_n(k) - 1) / tc_block_n(k) * tc_block_n(k); }

size_t split_rows_bytes(int64_t n, int d) {
    const int64_t nn = n > 0 ? n : 1, dp = split_dp(d);
    return (size_t)(2 * a256(nn * dp * 2) + 5 * a256(nn * 4) + a256(nn * 16));
}

size_t split_centers_bytes(int d, int k) {
    const int64_t dp = split_dp(d), kp = split_kp(k);
    return (size_t)(256 + 2 * a256(kp * dp * 2) + 3 * a256(kp * 4) + a256((int64_t)k * d * 4));
}

RowSplit carve_rows(void* base, int64_t n, int d) {
    RowSplit s;
    const int64_t nn = n > 0 ? n : 1, dp = split_dp(d);
    char* p = static_cast<char*>(base);
    s.xh = p;
    s.xl = p + a256(nn * dp * 2);
    s.xn = reinterpret_cast<float*>(p + 2 * a256(nn * dp * 2));
    s.lab = reinterpret_cast<int32_t*>(p + 2 * a256(nn * dp * 2) + a256(nn * 4));
    s.perm = reinterpret_cast<uint32_t*>(p + 2 * a256(nn * dp * 2) + 2 * a256(nn * 4));
    s.ovf = reinterpret_cast<uint32_t*>(p + 2 * a256(nn * dp * 2) + 3 * a256(nn * 4));
    s.cands = reinterpret_cast<int4*>(p + 2 * a256(nn * dp * 2) + 4 * a256(nn * 4));
    s.xsq_lo = reinterpret_cast<float*>(p + 2 * a256(nn * dp * 2) + 4 * a256(nn * 4) + a256(nn * 16));
    return s;
}

CenterSplit carve_centers(void* base, int d, int k) {
    CenterSplit s;
    const int64_t dp = split_dp(d), kp = split_kp(k);
    char* p = static_cast<char*>(base);
    s.cmax_bits = reinterpret_cast<unsigned int*>(p);
    s.error = reinterpret_cast<int*>(p + 4);
    s.nflag = reinterpret_cast<unsigned int*>(p + 8);
    s.novf = reinterpret_cast<unsigned int*>(p + 12);
    s.ch = p + 256;
    s.cl = p + 256 + a256(kp * dp * 2);
    s.hs = reinterpret_cast<float*>(p + 256 + 2 * a256(kp * dp * 2));
    s.hist = reinterpret_cast<unsigned int*>(p + 256 + 2 * a256(kp * dp * 2) + a256(kp * 4));
    s.cursor = reinterpret_cast<unsigned int*>(p + 256 + 2 * a256(kp * dp * 2) + 2 * a256(kp * 4));
    s.ct = reinterpret_cast<float*>(p + 256 + 2 * a256(kp * dp * 2) + 3 * a256(kp * 4));
    return s;
}

// kmc_d64: one warp per (row, center) pair
__global__ void __launch_bounds__(kSplitThreads) k_d64_pairs(const float* __restrict__ X,
                                                            const float* __restrict__ C, int d, int64_t m,
                                                            double* __restrict__ out) {
    __shared__ __align__(8) unsigned char scratch[kSplitWarps][kD64WarpScratch];
    const int warp = threadIdx.x >> 5;
    const int64_t stride = (int64_t)gridDim.x * kSplitWarps;
    for (int64_t i = (int64_t)blockIdx.x * kSplitWarps + warp; i < m; i += stride) {
        const double v = d64_warp(X + i * d, C + i * d, d, scratch[warp]);
        if ((threadIdx.x & 31) == 0) out[i] = v;
    }
}

cudaError_t launch_d64(const float* X, const float* C, int d, int64_t m, double* out, cudaStream_t st) {
    int64_t blocks = (m + kSplitWarps - 1) / kSplitWarps;
    if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
    k_d64_pairs<<<(int)blocks, kSplitThreads, 0, st>>>(X, C, d, m, out);
    return cudaGetLastError();
}

cudaError_t launch_split_rows(const float* X, int64_t n, int d, const RowSplit& s, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    int64_t blocks = (n + kSplitThreads / 32 - 1) / (kSplitThreads / 32);
    const int64_t cap = (int64_t)num_sms() * 16;
    if (blocks > cap) blocks = cap;
    k_split_rows<<<(int)blocks, kSplitThreads, 0, st>>>(X, n, d, split_dp(d), static_cast<__nv_bfloat16*>(s.xh),
                                                         static_cast<__nv_bfloat16*>(s.xl), s.xn, s.xsq_lo);
    return cudaGetLastError();
}

cudaError_t launch_split_centers(const float* C, int k, int d, const CenterSplit& s, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(s.cmax_bits, 0, 16, st);   // max |c|, error flag, flagged and overflow counts
    if (e != cudaSuccess) return e;
    const int kp = split_kp(k);
    const int blocks = (kp + kSplitThreads / 32 - 1) / (kSplitThreads / 32);
    k_split_centers<<<blocks, kSplitThreads, 0, st>>>(C, k, d, kp, split_dp(d), static_cast<__nv_bfloat16*>(s.ch),
                                                       static_cast<__nv_bfloat16*>(s.cl), s.hs, s.cmax_bits, s.ct);
    return cudaGetLastError();
}

cudaError_t launch_accum_split(PassArgs a, const RowSplit& rs, const CenterSplit& cs, cudaStream_t st) {
    if (a.n == 0) return cudaSuccess;
    cudaError_t e = cudaMemsetAsync(cs.hist, 0, sizeof(unsigned int) * (size_t)a.k, st);
    if (e != cudaSuccess) return e;
    int64_t blocks = (a.n + kSplitThreads - 1) / kSplitThreads;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    const size_t rsm = sizeof(float) * ((size_t)a.d + a.k);
    if (rsm > 32 * 1024) {                   // (12 KB of static shared memory besides)
        e = cudaFuncSetAttribute(k_rescore_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rsm);
        if (e != cudaSuccess) return e;
    }
    const int64_t fb = (a.n + kFlagRows - 1) / kFlagRows;
    k_flag_list<<<(int)fb, kSplitThreads, 0, st>>>(rs.lab, a.n, rs.cands, cs.error, rs.perm, cs.nflag, rs.ovf,
                                                   cs.novf, a.counters);
    k_decide_cands<<<num_sms() * 4, kSplitThreads, 0, st>>>(a.X, a.d, a.C, rs.perm, cs.nflag, rs.cands, cs.error,
                                                             a.prep, rs.lab);
    k_rescore_tc<<<num_sms() * 8, kRescoreThreads, rsm, st>>>(a.X, a.n, a.d, a.C, cs.ct, a.hc, a.k, a.prep, rs.ovf,
                                                              cs.novf, cs.error, rs.lab, a.counters);
    // each CTA flushes up to k counters: enough rows per CTA that the flush stays small
    int64_t hb = (a.n + 4 * (int64_t)a.k - 1) / (4 * (int64_t)a.k);
    if (hb > blocks) hb = blocks;
    if (hb < 1) hb = 1;
    k_fix_labels<<<(int)hb, kSplitThreads, 0, st>>>(a.X, a.n, a.d, a.C, a.k, rs.lab, cs.hist, a.labels, a.best);
    const bool aligned4 = a.d % 4 == 0 && (reinterpret_cast<uintptr_t>(a.X) & 15) == 0;
    k_scan_labels<<<1, 1024, 0, st>>>(cs.hist, a.k, cs.cursor);
    int64_t sb = (a.n + kScatterRows - 1) / kScatterRows;
    if (sb > cap) sb = cap;
    // grouped labels (the scatter's second output) in the overflow list's space, free from here on
    int32_t* glab = reinterpret_cast<int32_t*>(rs.ovf);
    k_scatter_rows<<<(int)sb, kSplitThreads, 0, st>>>(rs.lab, a.n, a.k, cs.cursor, rs.perm, glab);
    if (aligned4) {
        const int d4 = a.d / 4;
        const int lpr = d4 <= 4 ? 4 : d4 <= 8 ? 8 : d4 <= 16 ? 16 : 32;
        const int v = d4 > 32 ? 2 : 1;
        const int64_t span = (int64_t)(32 / lpr) * kSlabRows;
        const int64_t items = (a.n + span - 1) / span * ((a.d + 4 * lpr * v - 1) / (4 * lpr * v));
        const int64_t want = (items + kSlabThreads / 32 - 1) / (kSlabThreads / 32);
        const bool magic = a.n_total >= 2048;
        const size_t ssm = slab_smem(lpr, v);
        cudaError_t e3 = cudaSuccess;
        auto slab = [&](auto kern) {
            e3 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ssm);
            int per_sm = 0;
            if (e3 == cudaSuccess)
                e3 = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kSlabThreads, ssm);
            if (e3 != cudaSuccess) return;
            const int64_t cap = (int64_t)num_sms() * (per_sm > 0 ? per_sm : 1);   // one resident wave
            const int64_t blocks = want < cap ? want : cap;
            kern<<<(int)blocks, kSlabThreads, ssm, st>>>(a.X, a.n, a.d, a.C, glab, rs.perm, a.scale_x, a.prep,
                                                         a.totals, a.counters);
        };
        if (lpr == 4) magic ? slab(k_reduce_slab<4, 1, true>) : slab(k_reduce_slab<4, 1, false>);
        else if (lpr == 8) magic ? slab(k_reduce_slab<8, 1, true>) : slab(k_reduce_slab<8, 1, false>);
        else if (lpr == 16) magic ? slab(k_reduce_slab<16, 1, true>) : slab(k_reduce_slab<16, 1, false>);
        else if (v == 1) magic ? slab(k_reduce_slab<32, 1, true>) : slab(k_reduce_slab<32, 1, false>);
        else magic ? slab(k_reduce_slab<32, 2, true>) : slab(k_reduce_slab<32, 2, false>);
        if (e3 != cudaSuccess) return e3;
        return cudaGetLastError();
    }
    const size_t smem = (size_t)kReduceWarps * a.d * 8;
    const int64_t runs = (a.n + kRun - 1) / kRun;
    int64_t rb = (runs + kReduceWarps - 1) / kReduceWarps;
    const int64_t rcap = (int64_t)num_sms() * 8;
    if (rb > rcap) rb = rcap;
    auto go = [&](auto kern) -> cudaError_t {
        if (smem > 48 * 1024) {
            cudaError_t e2 = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e2 != cudaSuccess) return e2;
        }
        kern<<<(int)rb, 32 * kReduceWarps, smem, st>>>(a.X, a.n, a.d, a.C, rs.lab, rs.perm, a.scale_x, a.prep,
                                                       a.totals, a.counters);
        return cudaSuccess;
    };
    e = a.d <= 32 ? go(k_reduce_rows<1>) : a.d <= 64 ? go(k_reduce_rows<2>) : a.d <= 128 ? go(k_reduce_rows<4>)
                                                                            : go(k_reduce_rows<0>);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace kmc
