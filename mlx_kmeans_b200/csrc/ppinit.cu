// ppinit.cu -- greedy k-means++ seeding on a device-resident sample (reference: core.py:153-192).
//
// Round r picks T = 2 + floor(ln k) candidate rows by the Gumbel-max trick -- row i wins trial t with
// the largest max(d2_i, 1e-30) / E_it, E_it = -log(u_it) an exponential draw from Philox4x32-10 keyed by
// the round's seed (the reference orders by log d2 - log(-log u), the same order) -- then keeps the
// candidate whose distances lower the total d2 the most (core.py:189).  Totals are exact int64 fixed
// point, so the choice never depends on summation order; ties go to the first row / first trial.
// Three launches per round, no host round trip until the end.
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

struct PPWs {
    float* d2;               // m
    float* mins;             // m x T
    long long* cand;         // T
    long long* tot;          // T
    unsigned int* maxbits;   // 1
    int* shift;              // 1
};

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

PPWs pp_carve(void* base, int64_t m, int T) {
    char* p = static_cast<char*>(base);
    PPWs w;
    w.d2 = reinterpret_cast<float*>(p); p += align256(sizeof(float) * m);
    w.mins = reinterpret_cast<float*>(p); p += align256(sizeof(float) * m * T);
    w.cand = reinterpret_cast<long long*>(p); p += align256(sizeof(long long) * T);
    w.tot = reinterpret_cast<long long*>(p); p += align256(sizeof(long long) * T);
    w.maxbits = reinterpret_cast<unsigned int*>(p); p += 256;
    w.shift = reinterpret_cast<int*>(p); p += 256;
    return w;
}

int trials_for(int k) {
    if (k <= 1) return 1;
    return 2 + (int)floor(log((double)k));
}

}  // namespace

size_t pp_workspace_bytes(int64_t m, int d, int k) {
    (void)d;
    int T = trials_for(k);
    return align256(sizeof(float) * m) + align256(sizeof(float) * m * T) + 2 * align256(sizeof(long long) * T) + 512;
}

__device__ __forceinline__ float dist32(const float* __restrict__ a, const float* __restrict__ b, int d) {
    float s = 0.0f;
    for (int j = 0; j < d; j++) s = best32_term(s, a[j], b[j]);
    return s;
}

__global__ void k_pp_first(const float* __restrict__ S, int64_t m, int d, int64_t first, float* __restrict__ d2,
                           unsigned int* __restrict__ maxbits) {
    unsigned int mb = 0u;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
        float v = dist32(S + i * d, S + first * d, d);
        d2[i] = v;
        unsigned int b = __float_as_uint(v);
        mb = b > mb ? b : mb;
    }
    for (int o = 16; o; o >>= 1) {
        unsigned int ob = __shfl_xor_sync(0xffffffffu, mb, o);
        mb = ob > mb ? ob : mb;
    }
    if ((threadIdx.x & 31) == 0) atomicMax(maxbits, mb);
}

// 61 - ceil_log2(m) - ceil_log2(max d2): m quantised values of at most max d2 sum below 2^61.
__global__ void k_pp_shift(const unsigned int* maxbits, int64_t m, int* shift) {
    float mx = __uint_as_float(*maxbits);
    int s = 0;
    if (mx > 0.0f && isfinite(mx)) {
        s = 61 - ceil_log2((double)m) - ceil_log2((double)mx);
        s = s > 1000 ? 1000 : (s < -1000 ? -1000 : s);
    }
    *shift = s;
}

__device__ __forceinline__ double pp_key(float d2, uint64_t key, uint64_t row, uint32_t trial) {
    uint32_t c[4] = {(uint32_t)row, (uint32_t)(row >> 32), trial, 0x6B6D7070u};
    philox4x32_10(c, (uint32_t)key, (uint32_t)(key >> 32));
    uint64_t b = (((uint64_t)c[0] << 32) | c[1]) >> 11;
    double u = __dmul_rn(__dadd_rn((double)b, 0.5), 1.1102230246251565e-16);   // 2^-53
    double ex = -kmc_log(u);
    double dd = (double)(d2 > 1e-30f ? d2 : 1e-30f);
    return __ddiv_rn(dd, ex);
}

// One CTA per trial: argmax of the key over the sample (first row on ties).
__global__ void __launch_bounds__(1024) k_pp_pick(const float* __restrict__ d2, int64_t m,
                                                  const uint64_t* __restrict__ seeds, int round,
                                                  long long* __restrict__ cand, long long* __restrict__ tot) {
    const int t = blockIdx.x;
    const uint64_t key = seeds[round - 1];
    double bk = -1.0;
    long long bi = 0;
    for (int64_t i = threadIdx.x; i < m; i += blockDim.x) {
        double v = pp_key(d2[i], key, (uint64_t)i, (uint32_t)t);
        if (v > bk) { bk = v; bi = i; }
    }
    __shared__ double sk[32];
    __shared__ long long si[32];
    for (int o = 16; o; o >>= 1) {
        double ok = __shfl_xor_sync(0xffffffffu, bk, o);
        long long oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ok > bk || (ok == bk && oi < bi)) { bk = ok; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { sk[threadIdx.x >> 5] = bk; si[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (sk[w] > bk || (sk[w] == bk && si[w] < bi)) { bk = sk[w]; bi = si[w]; }
        cand[t] = bi;
        tot[t] = 0;
    }
}

// mins[i][t] = min(d2_i, |S_i - S_cand_t|^2) and the per-trial totals (exact int64).
__global__ void __launch_bounds__(256) k_pp_eval(const float* __restrict__ S, int64_t m, int d, int T,
                                                 const float* __restrict__ d2, const long long* __restrict__ cand,
                                                 const int* __restrict__ shift, float* __restrict__ mins,
                                                 long long* __restrict__ tot) {
    __shared__ long long part[16];
    if (threadIdx.x < 16) part[threadIdx.x] = 0;
    __syncthreads();
    const double scale = ldexp(1.0, *shift);
    for (int t = 0; t < T; t++) {
        const float* c = S + cand[t] * d;
        long long acc = 0;
        for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x) {
            float s = dist32(S + i * d, c, d);
            float v = d2[i] < s ? d2[i] : s;
            mins[i * T + t] = v;
            acc += quantize(v, scale);
        }
        for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if ((threadIdx.x & 31) == 0) atomicAdd(reinterpret_cast<unsigned long long*>(&part[t]), (unsigned long long)acc);
    }
    __syncthreads();
    if (threadIdx.x < T) atomicAdd(reinterpret_cast<unsigned long long*>(&tot[threadIdx.x]), (unsigned long long)part[threadIdx.x]);
}

__global__ void k_pp_update(int64_t m, int T, const float* __restrict__ mins, const long long* __restrict__ cand,
                            const long long* __restrict__ tot, float* __restrict__ d2, long long* __restrict__ picks,
                            int round) {
    int bt = 0;
    for (int t = 1; t < T; t++) if (tot[t] < tot[bt]) bt = t;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += (int64_t)gridDim.x * blockDim.x)
        d2[i] = mins[i * T + bt];
    if (blockIdx.x == 0 && threadIdx.x == 0) picks[round] = cand[bt];
}

__global__ void k_pp_gather(const float* __restrict__ S, int d, int k, const long long* __restrict__ picks,
                            float* __restrict__ C) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < (int64_t)k * d; e += (int64_t)gridDim.x * blockDim.x) {
        int c = (int)(e / d), j = (int)(e % d);
        C[e] = S[picks[c] * d + j];
    }
}

__global__ void k_pp_set_first(long long* picks, int64_t first) { picks[0] = first; }

cudaError_t launch_pp_init(const float* S, int64_t m, int d, int k, int64_t first, const uint64_t* seeds,
                           int64_t* picks, float* C_out, void* ws, size_t ws_bytes, cudaStream_t st) {
    const int T = trials_for(k);
    if (T > 16) return cudaErrorInvalidValue;
    if (ws_bytes < pp_workspace_bytes(m, d, k)) return cudaErrorInvalidValue;
    PPWs w = pp_carve(ws, m, T);
    long long* pk = reinterpret_cast<long long*>(picks);
    cudaError_t e = cudaMemsetAsync(w.maxbits, 0, sizeof(unsigned int), st);
    if (e != cudaSuccess) return e;
    int blocks = (int)((m + 255) / 256);
    int cap = num_sms() * 4;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    k_pp_first<<<blocks, 256, 0, st>>>(S, m, d, first, w.d2, w.maxbits);
    k_pp_shift<<<1, 1, 0, st>>>(w.maxbits, m, w.shift);
    k_pp_set_first<<<1, 1, 0, st>>>(pk, first);
    for (int r = 1; r < k; r++) {
        k_pp_pick<<<T, 1024, 0, st>>>(w.d2, m, seeds, r, w.cand, w.tot);
        k_pp_eval<<<blocks, 256, 0, st>>>(S, m, d, T, w.d2, w.cand, w.shift, w.mins, w.tot);
        k_pp_update<<<blocks, 256, 0, st>>>(m, T, w.mins, w.cand, w.tot, w.d2, pk, r);
    }
    int gb = (int)(((int64_t)k * d + 255) / 256);
    if (gb > 4096) gb = 4096;
    k_pp_gather<<<gb > 0 ? gb : 1, 256, 0, st>>>(S, d, k, pk, C_out);
    return cudaGetLastError();
}

}  // namespace kmc
