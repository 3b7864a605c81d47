// elkan.cu -- per-center lower bounds between passes for the tensor-core shapes (Elkan 2003).
//
// Reference: the bounded high-d path of core.py:1690-2015 (one lower bound per (row, center) kept between
// iterations; a pass visits only the centers whose bound fell below the row's distance to its own center).
// Built here for B200 on the tensor-core pipeline:
//   - the bounds are n x k float16, rounded toward zero, so a stored bound never exceeds the value it stands for;
//     the tensor-core pass writes them from its scores (assign_tc.cu, with the window's error bound subtracted);
//   - a bounded pass (k_elkan, a warp per row) lowers every bound by its center's drift since (k_elkan_drift,
//     float64 rounded up), recomputes the row's distance to its previous label in float32, and computes the
//     distance only to the centers whose lowered bound does not exceed the window above it -- every center that
//     could be the label, or tie with it, is among them (ties included: the test is <=, the distance is inflated
//     by its rounding bound and by the decision window);
//   - a row whose two best computed distances are within the window goes to the same float64 / float32-rule
//     decision as the tensor-core pass's flagged rows (label bit 31 and its candidates, split.cu), so labels are the
//     full pass's, bit for bit, and the totals (grouped reduction, split.cu) too.
// Every visited center's bound is replaced by its computed distance, rounded down; the others keep the lowered
// bound.
//
// The prefix-pruning cascade (kmc_pass_cascade; the reference's two-stage exact assignment, core.py:1091-1260)
// shares the bounded pass's scoring and decision: k_cascade_ub sets each row's threshold from its previous label,
// the tensor-core pass over the prefix columns marks the centers whose prefix lower bound does not exceed it (one
// bit per (row, center), assign_tc.cu), and k_cascade scores the marked centers in full.
#include <cuda_fp16.h>

#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kElkanThreads = 256;          // 8 warps, one row each at a time
constexpr int kElkanWarps = kElkanThreads / 32;

// drift[c] = |c - c_prev| (float64, rounded up, as float rounded up), then c_prev = c; a warp per center
__global__ void __launch_bounds__(kElkanThreads) k_elkan_drift(const float* __restrict__ C, float* __restrict__ cprev,
                                                              int k, int d, float* __restrict__ drift) {
    const int lane = threadIdx.x & 31;
    const int nw = gridDim.x * kElkanWarps;
    for (int c = blockIdx.x * kElkanWarps + (threadIdx.x >> 5); c < k; c += nw) {
        double s = 0.0;
        for (int j = lane; j < d; j += 32) {
            const double q = (double)C[(int64_t)c * d + j] - (double)cprev[(int64_t)c * d + j];   // exact
            s = __fma_ru(q, q, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s = __dadd_ru(s, __shfl_xor_sync(0xffffffffu, s, o));
        if (lane == 0) drift[c] = __double2float_ru(__dsqrt_ru(s));
        for (int j = lane; j < d; j += 32) cprev[(int64_t)c * d + j] = C[(int64_t)c * d + j];   // (own elements)
    }
}

// The two smallest (value, index) pairs -- lower index first on equal values -- and the third smallest value.
struct Best3 {
    float m0, m1, m2;
    int l0, l1;
    __device__ __forceinline__ void init() {
        m0 = m1 = m2 = INFINITY;
        l0 = l1 = 0x7fffffff;
    }
    __device__ __forceinline__ void push(float s, int c) {
        const bool a0 = s < m0 || (s == m0 && c < l0), a1 = s < m1 || (s == m1 && c < l1), a2 = s < m2;
        m2 = a1 ? m1 : (a2 ? s : m2);
        m1 = a0 ? m0 : (a1 ? s : m1);
        l1 = a0 ? l0 : (a1 ? c : l1);
        m0 = a0 ? s : m0;
        l0 = a0 ? c : l0;
    }
};

// Squared distance of the row (the lane's XR values in registers; XR == 0: read from memory) to center c: per lane
// a float32 fma chain over its columns, then an xor tree (every lane ends with the same sum).
template <int XR>
__device__ __forceinline__ float warp_dist(const float (&xv)[XR > 0 ? XR : 1], const float* __restrict__ x,
                                           const float* __restrict__ c, int d, int lane) {
    float s = 0.0f;
    if constexpr (XR > 0) {
#pragma unroll
        for (int m = 0; m < XR; m++) {
            const int j = lane + 32 * m;
            if (j < d) {
                const float t = xv[m] - __ldg(c + j);
                s = __fmaf_rn(t, t, s);
            }
        }
    } else {
        for (int j = lane; j < d; j += 32) {
            const float t = x[j] - __ldg(c + j);
            s = __fmaf_rn(t, t, s);
        }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    return s;
}

// A computed squared distance is within g of the exact one (a subtraction and a square per term, an fma chain of
// ceil(d/32) terms per lane, a five-level tree: nonnegative terms, taken twice over).  A center can be the label
// only if its computed distance is within W of the smallest: (1 + g) / (1 - g), the label rule's own rounding
// (float64: 2^-40 of margin; the float32 rule: rule32_coef(d)), and a 2^-20 margin.
struct Window {
    float g, W;
    __device__ Window(int d, int rule) {
        const int mcols = (d + 31) / 32;
        const double gd = (mcols + 8) / 8388608.0;
        g = (float)gd;
        W = (float)((1.0 + gd) / (1.0 - gd) * (1.0 + (rule ? rule32_coef(d) : 1.0 / 1099511627776.0)) *
                    (1.0 + 1.0 / 1048576.0));
    }
};

// A row's label from the distances computed for it: decided when no other center is within the window of the
// smallest, else flagged (bit 31) with its candidates for the label rule's decision (split.cu).
__device__ __forceinline__ void decide(const Best3& b, float W, int k, int64_t row, int32_t* lab, int4* cands) {
    const float hi = __fmul_ru(b.m0, W);
    if (!(b.m1 <= hi) && b.m0 <= 3.0e38f) {
        lab[row] = b.l0;
    } else {
        const bool many = b.m2 <= hi || !(b.m0 <= 3.0e38f) || b.l1 == 0x7fffffff;
        lab[row] = (int32_t)((uint32_t)(b.l0 < k ? b.l0 : 0) | 0x80000000u);
        cands[row] = make_int4(b.l0 < k ? b.l0 : 0, b.l1 < k ? b.l1 : -1, -1, many ? -2 : -1);
    }
}

template <int XR>
__global__ void __launch_bounds__(kElkanThreads) k_elkan(const float* __restrict__ X, int64_t n, int d,
                                                        const float* __restrict__ C, int k,
                                                        const float* __restrict__ drift, __half* __restrict__ lb,
                                                        int32_t* __restrict__ lab, int4* __restrict__ cands,
                                                        const uint32_t* __restrict__ order,
                                                        const Prep* __restrict__ prep,
                                                        long long* __restrict__ counters) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kElkanWarps;
    const Window wn(d, prep->rule);
    const float g = wn.g, W = wn.W;
    long long visited = 0;
    // rows in the order of the previous pass's grouping by label (a permutation of the rows): neighbouring warps
    // take rows of the same cluster, which visit the same few centers, so those centers' vectors stay in L1
    for (int64_t idx = (int64_t)blockIdx.x * kElkanWarps + (threadIdx.x >> 5); idx < n; idx += nw) {
        const int64_t row = order[idx];
        if (row >= n) continue;                    // (a permutation after any pass on the split; never out of range)
        const float* x = X + row * d;
        float xv[XR > 0 ? XR : 1];
        if constexpr (XR > 0) {
#pragma unroll
            for (int m = 0; m < XR; m++) {
                const int j = lane + 32 * m;
                xv[m] = j < d ? __ldg(x + j) : 0.0f;
            }
        }
        int l = lab[row] & 0x7fffffff;
        if (l >= k) l = 0;
        const float Dl = warp_dist<XR>(xv, x, C + (int64_t)l * d, d, lane);
        // every center whose exact distance can be within W of this row's smallest (<= its distance to l) is
        // visited: its bound, a lower bound on its exact distance, is at most sqrt(Dl (1 + g) W)
        const float thr = __fsqrt_ru(__fmul_ru(__fmul_ru(Dl, 1.0f + g), W));
        Best3 b;
        b.init();
        b.push(Dl, l);
        for (int base = 0; base < k; base += 32) {
            const int c = base + lane;
            const bool valid = c < k;
            const __half* bp = lb + row * (int64_t)k + c;
            float lbn = valid ? __fsub_rd(__half2float(*bp), __ldg(drift + c)) : INFINITY;
            const bool cand = valid && c != l && !(lbn > thr);
            unsigned mask = __ballot_sync(0xffffffffu, cand);
            float out = lbn > 0.0f ? lbn : 0.0f;
            if (c == l) out = __fsqrt_rd(__fmul_rd(Dl, 1.0f - g));
            if (lane == 0) visited += __popc(mask);
            while (mask) {
                const int src = __ffs(mask) - 1;
                mask &= mask - 1;
                const float Dc = warp_dist<XR>(xv, x, C + (int64_t)(base + src) * d, d, lane);
                if (lane == src) out = __fsqrt_rd(__fmul_rd(Dc, 1.0f - g));
                b.push(Dc, base + src);
            }
            if (valid) *const_cast<__half*>(bp) = __float2half_rz(out);
        }
        if (lane == 0) decide(b, W, k, row, lab, cands);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) visited += __shfl_xor_sync(0xffffffffu, visited, o);
    if (lane == 0 && visited) atomicAdd(reinterpret_cast<unsigned long long*>(&counters[2]), (unsigned long long)visited);
}

// The cascade's threshold (kmc_pass_cascade, before its prefix pass): each row's float32 squared distance to its
// previous label, times (1 + g) W, rounded up.  A center that can be the row's label, or tie with it, has an exact
// distance within W of the smallest, which is at most the exact distance to the previous label, which is at most
// the computed one times (1 + g); so its prefix lower bound cannot exceed this.  A warp per row.
template <int XR>
__global__ void __launch_bounds__(kElkanThreads) k_cascade_ub(const float* __restrict__ X, int64_t n, int d,
                                                             const float* __restrict__ C, int k,
                                                             const int32_t* __restrict__ lab,
                                                             const Prep* __restrict__ prep, float* __restrict__ ub) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kElkanWarps;
    const Window wn(d, prep->rule);
    for (int64_t row = (int64_t)blockIdx.x * kElkanWarps + (threadIdx.x >> 5); row < n; row += nw) {
        const float* x = X + row * d;
        float xv[XR > 0 ? XR : 1];
        if constexpr (XR > 0) {
#pragma unroll
            for (int m = 0; m < XR; m++) {
                const int j = lane + 32 * m;
                xv[m] = j < d ? __ldg(x + j) : 0.0f;
            }
        }
        int l = lab[row] & 0x7fffffff;
        if (l >= k) l = 0;
        const float Dl = warp_dist<XR>(xv, x, C + (int64_t)l * d, d, lane);
        if (lane == 0) ub[row] = __fmul_ru(__fmul_ru(Dl, 1.0f + wn.g), wn.W);
    }
}

// The cascade's second stage: every row the prefix pass listed (a surviving center besides its previous label) has
// its surviving centers (its bits in the prefix pass's mask) scored in full, as k_elkan scores the centers its bounds
// leave, with the previous label first; the same decision.  A row not listed keeps its previous label: every other
// center's distance is more than the window above it (its threshold was finite, or every bit would be set).  The
// list's order does not matter: each row's result is its own.
template <int XR>
__global__ void __launch_bounds__(kElkanThreads) k_cascade(const float* __restrict__ X, int64_t n, int d,
                                                          const float* __restrict__ C, int k,
                                                          const uint32_t* __restrict__ mask,
                                                          const uint32_t* __restrict__ srows,
                                                          const unsigned int* __restrict__ nsrows,
                                                          int32_t* __restrict__ lab, int4* __restrict__ cands,
                                                          const Prep* __restrict__ prep,
                                                          long long* __restrict__ counters) {
    const int lane = threadIdx.x & 31;
    const int64_t nw = (int64_t)gridDim.x * kElkanWarps;
    const int kw = (k + 31) / 32;
    const float W = Window(d, prep->rule).W;
    const int64_t count = *nsrows;
    long long visited = 0;
    for (int64_t idx = (int64_t)blockIdx.x * kElkanWarps + (threadIdx.x >> 5); idx < count; idx += nw) {
        const int64_t row = srows[idx];
        if (row >= n) continue;
        int l = lab[row] & 0x7fffffff;
        if (l >= k) l = 0;
        const float* x = X + row * d;
        float xv[XR > 0 ? XR : 1];
        if constexpr (XR > 0) {
#pragma unroll
            for (int m = 0; m < XR; m++) {
                const int j = lane + 32 * m;
                xv[m] = j < d ? __ldg(x + j) : 0.0f;
            }
        }
        const float Dl = warp_dist<XR>(xv, x, C + (int64_t)l * d, d, lane);
        Best3 b;
        b.init();
        b.push(Dl, l);
        // the row's survivor words, 32 at a time (one per lane); only the nonzero ones are walked
        const uint32_t* mrow = mask + row * (int64_t)kw;
        for (int w0 = 0; w0 < kw; w0 += 32) {
            const int w = w0 + lane;
            uint32_t word = w < kw ? __ldg(mrow + w) : 0u;
            if ((l >> 5) == w) word &= ~(1u << (l & 31));
            visited += __popc(word);
            unsigned nz = __ballot_sync(0xffffffffu, word != 0u);
            while (nz) {
                const int src = __ffs(nz) - 1;
                nz &= nz - 1;
                uint32_t bits = __shfl_sync(0xffffffffu, word, src);
                while (bits) {
                    const int c = (w0 + src) * 32 + __ffs(bits) - 1;
                    bits &= bits - 1;
                    b.push(warp_dist<XR>(xv, x, C + (int64_t)c * d, d, lane), c);
                }
            }
        }
        if (lane == 0) decide(b, W, k, row, lab, cands);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) visited += __shfl_xor_sync(0xffffffffu, visited, o);
    if (lane == 0 && visited) atomicAdd(reinterpret_cast<unsigned long long*>(&counters[2]), (unsigned long long)visited);
}

template <int XR>
cudaError_t run_elkan(const float* X, int64_t n, int d, const float* C, int k, const float* drift, void* lb,
                      int32_t* lab, int4* cands, const uint32_t* order, const Prep* prep, long long* counters,
                      cudaStream_t st) {
    int64_t blocks = (n + kElkanWarps - 1) / kElkanWarps;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_elkan<XR><<<(int)blocks, kElkanThreads, 0, st>>>(X, n, d, C, k, drift, static_cast<__half*>(lb), lab, cands,
                                                       order, prep, counters);
    return cudaGetLastError();
}

template <int XR>
cudaError_t run_cascade(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                        int32_t* lab, int4* cands, const Prep* prep, long long* counters, bool threshold,
                        cudaStream_t st) {
    int64_t blocks = (n + kElkanWarps - 1) / kElkanWarps;
    const int64_t cap = (int64_t)num_sms() * 8;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    if (threshold)
        k_cascade_ub<XR><<<(int)blocks, kElkanThreads, 0, st>>>(X, n, d, C, k, lab, prep, cs.ub);
    else
        k_cascade<XR><<<(int)blocks, kElkanThreads, 0, st>>>(X, n, d, C, k, cs.mask, cs.srows, cs.nsrows, lab,
                                                             cands, prep, counters);
    return cudaGetLastError();
}

cudaError_t cascade_dispatch(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                             int32_t* lab, int4* cands, const Prep* prep, long long* counters, bool threshold,
                             cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const int m = (d + 31) / 32;
#define KMC_CASCADE(XR) run_cascade<XR>(X, n, d, C, k, cs, lab, cands, prep, counters, threshold, st)
    if (m <= 4) return KMC_CASCADE(4);
    if (m <= 8) return KMC_CASCADE(8);
    if (m <= 16) return KMC_CASCADE(16);
    return KMC_CASCADE(0);
#undef KMC_CASCADE
}

}  // namespace

int64_t a256e(int64_t v) { return (v + 255) / 256 * 256; }

size_t cascade_bytes(int64_t n, int k) {
    const int64_t nn = n > 0 ? n : 1;
    return (size_t)(256 + a256e(nn * 4) + a256e(nn * ((k + 31) / 32) * 4) + a256e(nn * 4));
}

CascadeState carve_cascade(void* base, int64_t n, int k) {
    const int64_t nn = n > 0 ? n : 1;
    CascadeState c;
    char* p = static_cast<char*>(base);
    c.nsrows = reinterpret_cast<unsigned int*>(p);
    c.ub = reinterpret_cast<float*>(p + 256);
    c.mask = reinterpret_cast<uint32_t*>(p + 256 + a256e(nn * 4));
    c.srows = reinterpret_cast<uint32_t*>(p + 256 + a256e(nn * 4) + a256e(nn * ((k + 31) / 32) * 4));
    return c;
}

cudaError_t launch_cascade_ub(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                              const int32_t* lab, const Prep* prep, cudaStream_t st) {
    cudaError_t e = cudaMemsetAsync(cs.nsrows, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    return cascade_dispatch(X, n, d, C, k, cs, const_cast<int32_t*>(lab), nullptr, prep, nullptr, true, st);
}

cudaError_t launch_cascade(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                           int32_t* lab, int4* cands, const Prep* prep, long long* counters, cudaStream_t st) {
    return cascade_dispatch(X, n, d, C, k, cs, lab, cands, prep, counters, false, st);
}

size_t elkan_bytes(int64_t n, int d, int k) {
    const int64_t nn = n > 0 ? n : 1;
    return (size_t)(a256e((int64_t)k * d * 4) + a256e((int64_t)k * 4) + a256e(nn * k * 2));
}

ElkanState carve_elkan(void* base, int64_t n, int d, int k) {
    (void)n;
    ElkanState e;
    char* p = static_cast<char*>(base);
    e.cprev = reinterpret_cast<float*>(p);
    e.drift = reinterpret_cast<float*>(p + a256e((int64_t)k * d * 4));
    e.lb = p + a256e((int64_t)k * d * 4) + a256e((int64_t)k * 4);
    return e;
}

cudaError_t launch_elkan_drift(const float* C, const ElkanState& e, int k, int d, cudaStream_t st) {
    int blocks = (k + kElkanWarps - 1) / kElkanWarps;
    if (blocks > num_sms() * 8) blocks = num_sms() * 8;
    k_elkan_drift<<<blocks, kElkanThreads, 0, st>>>(C, e.cprev, k, d, e.drift);
    return cudaGetLastError();
}

cudaError_t launch_elkan(const float* X, int64_t n, int d, const float* C, int k, const ElkanState& e, int32_t* lab,
                         int4* cands, const uint32_t* order, const Prep* prep, long long* counters, cudaStream_t st) {
    if (n == 0) return cudaSuccess;
    const int m = (d + 31) / 32;
    if (m <= 1) return run_elkan<1>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 2) return run_elkan<2>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 4) return run_elkan<4>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 8) return run_elkan<8>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 16) return run_elkan<16>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 24) return run_elkan<24>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    if (m <= 32) return run_elkan<32>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
    return run_elkan<0>(X, n, d, C, k, e.drift, e.lb, lab, cands, order, prep, counters, st);
}

}  // namespace kmc
