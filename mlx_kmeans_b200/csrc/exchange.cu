// exchange.cu -- the all-reduce of the per-cluster totals over the GPUs of one node as a kernel of its own
// (kmc_exchange_sum): one CTA running exchange_cta (exchange.cuh: protocol, buffer layout, bounded waits), or,
// for wide totals (k (d + 2) >= kExchangeWideMin values: 4.3 MB at k = 4096, d = 128, which one CTA sums at
// NVLink latency in about 1.5 ms), up to kExchangeRows CTAs, each exchanging its own range through its own flag
// row.  kmc_exchange_finish runs the one-CTA exchange at the start of k_finish instead, one launch fewer per
// step, and the wide one as a launch of its own before k_finish.
#include <cstdlib>

#include "exchange.cuh"

namespace kmc {

namespace {

constexpr int kExThreads = 256;

__global__ void __launch_bounds__(kExThreads) k_exchange_sum(long long* __restrict__ totals, int64_t W,
                                                            const unsigned long long* __restrict__ peers, int world,
                                                            int rank, unsigned long long step,
                                                            unsigned long long timeout_ns,
                                                            long long* __restrict__ counters) {
    __shared__ int s_fail;
    pdl_wait();                                      // the pass's totals
    exchange_cta(totals, W, 0, W, 0, peers, world, rank, step, timeout_ns, counters, &s_fail);
}

// CTA b exchanges the b-th of gridDim.x equal ranges through flag row b.
__global__ void __launch_bounds__(kExThreads) k_exchange_wide(long long* __restrict__ totals, int64_t W,
                                                             const unsigned long long* __restrict__ peers, int world,
                                                             int rank, unsigned long long step,
                                                             unsigned long long timeout_ns,
                                                             long long* __restrict__ counters) {
    __shared__ int s_fail;
    pdl_wait();                                      // the pass's totals
    const int64_t per = (W + gridDim.x - 1) / gridDim.x;
    const int64_t e0 = (int64_t)blockIdx.x * per;
    const int64_t e1 = e0 + per < W ? e0 + per : W;
    exchange_cta(totals, W, e0, e1, (int)blockIdx.x, peers, world, rank, step, timeout_ns, counters, &s_fail);
}

}  // namespace

bool exchange_wide(int k, int d) { return (int64_t)k * (d + 2) >= kExchangeWideMin; }

size_t exchange_bytes(int k, int d) { return (size_t)kExchangeHeader + 2 * (size_t)k * (d + 2) * 8; }

// How long a rank waits for its peers before the exchange gives up: KMC_EXCHANGE_TIMEOUT_MS milliseconds
// (read on every call, so a test can shorten it), 30 s by default.
unsigned long long exchange_timeout_ns() {
    const char* v = std::getenv("KMC_EXCHANGE_TIMEOUT_MS");
    long long ms = v ? std::atoll(v) : 0;
    if (ms <= 0) ms = 30000;
    return (unsigned long long)ms * 1000000ull;
}

cudaError_t launch_exchange_sum(long long* totals, int k, int d, const unsigned long long* peers, int world, int rank,
                                unsigned long long step, long long* counters, cudaStream_t st) {
    const int64_t W = (int64_t)k * (d + 2);
    if (exchange_wide(k, d)) {
        // ranges of at least 4096 values (32 KB per peer), at most one CTA per flag row
        int64_t g = (W + 4095) / 4096;
        if (g > kExchangeRows) g = kExchangeRows;
        return launch_pdl(k_exchange_wide, dim3((unsigned)g), dim3(kExThreads), 0, st, totals, W, peers, world, rank,
                          step, exchange_timeout_ns(), counters);
    }
    return launch_pdl(k_exchange_sum, dim3(1), dim3(kExThreads), 0, st, totals, W, peers, world, rank, step,
                      exchange_timeout_ns(), counters);
}

}  // namespace kmc
