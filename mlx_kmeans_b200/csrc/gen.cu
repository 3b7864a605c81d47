// gen.cu -- synthetic inputs of the benchmark configurations, generated on the device.
//
// Every value is a function of (seed, global row, column) through Philox4x32-10, so a shard generated
// on GPU r from row0 = r * n / P holds exactly the rows the single-GPU run holds.  The reference
// generates on the GPU the same way from a splitmix64 hash (core.py:43-63, 111-129).
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

// 4 uniform words for (row, block of 4 columns, stream)
__device__ __forceinline__ void philox_words(uint64_t seed, int64_t row, uint32_t blk, uint32_t stream, uint32_t out[4]) {
    out[0] = (uint32_t)row;
    out[1] = (uint32_t)((uint64_t)row >> 32);
    out[2] = blk;
    out[3] = stream;
    philox4x32_10(out, (uint32_t)seed, (uint32_t)(seed >> 32));
}

__device__ __forceinline__ float u01_open(uint32_t w) {            // (0, 1)
    return ((float)(w >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ float u01(uint32_t w) {                 // [0, 1)
    return (float)(w >> 8) * (1.0f / 16777216.0f);
}

}  // namespace

// kind 0: uniform [0, 1)
__global__ void k_gen_uniform(float* __restrict__ X, int64_t n, int d, int64_t row0, uint64_t seed) {
    const int nb = (d + 3) / 4;
    const int64_t total = n * nb;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / nb;
        const int b = (int)(e % nb);
        uint32_t w[4];
        philox_words(seed, row0 + r, (uint32_t)b, 0u, w);
#pragma unroll
        for (int q = 0; q < 4; q++) {
            int j = 4 * b + q;
            if (j < d) X[r * d + j] = u01(w[q]);
        }
    }
}

// kinds 1, 2: Gaussian mixture, one thread per row.
__global__ void k_gen_mixture(float* __restrict__ X, int64_t n, int d, int64_t row0, uint64_t seed,
                              const float* __restrict__ means, const float* __restrict__ sds, int ncomp, float lo,
                              float hi, int unit) {
    for (int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; r < n; r += (int64_t)gridDim.x * blockDim.x) {
        const int64_t g = row0 + r;
        uint32_t w[4];
        philox_words(seed, g, 0xffffffffu, 1u, w);
        const int comp = (int)(((uint64_t)w[0] * (uint64_t)ncomp) >> 32);
        const float* mu = means + (int64_t)comp * d;
        const float* sd = sds + (int64_t)comp * d;
        float* xr = X + r * d;
        double nrm = 0.0;
        for (int b = 0; b < (d + 3) / 4; b++) {
            philox_words(seed, g, (uint32_t)b, 2u, w);
            // Box-Muller: two normals per pair of words
            float z[4];
#pragma unroll
            for (int p = 0; p < 2; p++) {
                float u1 = u01_open(w[2 * p]), u2 = u01(w[2 * p + 1]);
                float rad = sqrtf(-2.0f * logf(u1));
                float s, c;
                sincospif(2.0f * u2, &s, &c);
                z[2 * p] = rad * c;
                z[2 * p + 1] = rad * s;
            }
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int j = 4 * b + q;
                if (j >= d) break;
                float v = fmaf(sd[j], z[q], mu[j]);
                if (lo < hi) v = fminf(fmaxf(v, lo), hi);
                xr[j] = v;
                nrm += (double)v * (double)v;
            }
        }
        if (unit) {
            double inv = nrm > 0.0 ? 1.0 / sqrt(nrm) : 0.0;
            for (int j = 0; j < d; j++) xr[j] = (float)((double)xr[j] * inv);
        }
    }
}

cudaError_t launch_gen(int kind, float* X, int64_t n, int d, int64_t row0, uint64_t seed, const float* means,
                       const float* sds, int ncomp, float lo, float hi, cudaStream_t st) {
    if (n <= 0) return cudaSuccess;
    int blocks = num_sms() * 8;
    if (kind == 0) {
        k_gen_uniform<<<blocks, 256, 0, st>>>(X, n, d, row0, seed);
    } else if (kind == 1 || kind == 2) {
        if (means == nullptr || sds == nullptr || ncomp < 1) return cudaErrorInvalidValue;
        k_gen_mixture<<<blocks, 256, 0, st>>>(X, n, d, row0, seed, means, sds, ncomp, lo, hi, kind == 2);
    } else {
        return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// ---------------------------------------------------------------- column sums and standardisation
// sums[0][j] = sum of x_j and sums[1][j] = sum of x_j^2, each as exact int64 fixed point on its own grid
// (column_shift of max|x_j| and of max|x_j|^2), so the mean and variance do not depend on the split of rows.
__global__ void k_colsums(const float* __restrict__ X, int64_t total, int d, int64_t stride,
                          const unsigned int* __restrict__ colmax, int64_t n_total, long long* __restrict__ sums) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= stride) return;
    const int j = (int)(t % d);
    const float m = __uint_as_float(colmax[j]);
    const double s1 = ldexp(1.0, column_shift(m, n_total));
    const double s2 = ldexp(1.0, column_shift(m * m, n_total));
    long long a = 0, b = 0;
    for (int64_t e = t; e < total; e += stride) {
        const double v = (double)X[e];
        a += __double2ll_rn(__dmul_rn(v, s1));
        b += __double2ll_rn(__dmul_rn(__dmul_rn(v, v), s2));
    }
    atomicAdd(reinterpret_cast<unsigned long long*>(&sums[j]), (unsigned long long)a);
    atomicAdd(reinterpret_cast<unsigned long long*>(&sums[d + j]), (unsigned long long)b);
}

cudaError_t launch_colsums(const float* X, int64_t n, int d, const unsigned int* colmax, int64_t n_total,
                           long long* sums, cudaStream_t st) {
    int64_t total = n * (int64_t)d;
    if (total == 0) return cudaSuccess;
    int64_t want = (int64_t)num_sms() * 8 * 256;
    int64_t stride = (want / d) * d;
    if (stride < d) stride = d;
    if (stride > total) stride = ((total + d - 1) / d) * d;
    int blocks = (int)((stride + 255) / 256);
    k_colsums<<<blocks, 256, 0, st>>>(X, total, d, stride, colmax, n_total, sums);
    return cudaGetLastError();
}

// mean and population standard deviation (ddof 0) in float64 from the exact sums
__global__ void k_meanstd(const long long* __restrict__ sums, const unsigned int* __restrict__ colmax, int d,
                          int64_t n_total, double* __restrict__ mean_std) {
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const float m = __uint_as_float(colmax[j]);
        const double s1 = ldexp(1.0, column_shift(m, n_total));
        const double s2 = ldexp(1.0, column_shift(m * m, n_total));
        const double mean = ((double)sums[j] / s1) / (double)n_total;
        const double ex2 = ((double)sums[d + j] / s2) / (double)n_total;
        const double var = ex2 - mean * mean;
        mean_std[j] = mean;
        mean_std[d + j] = var > 0.0 ? sqrt(var) : 1.0;
    }
}

__global__ void k_standardize(float* __restrict__ X, int64_t total, int d, const double* __restrict__ mean_std) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int j = (int)(e % d);
        X[e] = __double2float_rn(__ddiv_rn(__dsub_rn((double)X[e], mean_std[j]), mean_std[d + j]));
    }
}

cudaError_t launch_standardize(float* X, int64_t n, int d, const long long* sums, const unsigned int* colmax,
                               int64_t n_total, double* mean_std, cudaStream_t st) {
    k_meanstd<<<1, 256, 0, st>>>(sums, colmax, d, n_total, mean_std);
    int64_t total = n * (int64_t)d;
    if (total > 0) k_standardize<<<num_sms() * 8, 256, 0, st>>>(X, total, d, mean_std);
    return cudaGetLastError();
}

}  // namespace kmc
