// exchange.cu -- the all-reduce of the per-cluster totals over the GPUs of one node as a kernel of its own
// (kmc_exchange_sum): one CTA running exchange_cta (exchange.cuh: protocol, buffer layout, bounded waits).
// kmc_exchange_finish runs the same code at the start of k_finish instead, one launch fewer per step.
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
    exchange_cta(totals, W, peers, world, rank, step, timeout_ns, counters, &s_fail);
}

}  // namespace

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
    k_exchange_sum<<<1, kExThreads, 0, st>>>(totals, (int64_t)k * (d + 2), peers, world, rank, step,
                                             exchange_timeout_ns(), counters);
    return cudaGetLastError();
}

}  // namespace kmc
