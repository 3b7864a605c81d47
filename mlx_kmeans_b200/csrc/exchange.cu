// exchange.cu -- the all-reduce of the per-cluster totals over the GPUs of one node, through peer memory.
//
// One kernel per step replaces the NCCL all-reduce of the int64 totals (k (d+2) values, 768 bytes at
// configuration 3): the rank copies its totals into its own exchange buffer, raises its flag in every peer's
// buffer (a release store over NVLink), waits for every peer's flag (acquire loads of its own buffer, bounded),
// and sums all ranks' totals with plain peer loads.  The sum of integers does not depend on the order, so the
// result is the same as NCCL's and the same on every rank.
//
// Exchange buffer of a rank (kmc_exchange_alloc; the peers map it through CUDA IPC):
//   [flags: 64 x uint64; flag r = the last step rank r has published]  [slot 0: W int64]  [slot 1: W int64]
// Step s publishes into slot s & 1.  A rank writes slot s & 1 again at step s + 2 only after it has seen every
// peer's flag for step s + 1, which each peer raises after it finished reading step s: two slots suffice.
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

namespace {

constexpr int kExThreads = 256;
constexpr uint32_t kExSpin = 1u << 26;   // polls before a wait gives up (a few seconds)

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kExThreads) k_exchange_sum(long long* __restrict__ totals, int64_t W,
                                                            const unsigned long long* __restrict__ peers, int world,
                                                            int rank, unsigned long long step,
                                                            long long* __restrict__ counters) {
    __shared__ int s_fail;
    const int tid = threadIdx.x;
    if (tid == 0) s_fail = 0;
    const size_t slot_off = (size_t)kExchangeHeader + (size_t)(step & 1) * (size_t)W * 8;
    char* mine = reinterpret_cast<char*>(peers[rank]);
    long long* my_slot = reinterpret_cast<long long*>(mine + slot_off);
    for (int64_t e = tid; e < W; e += kExThreads) my_slot[e] = totals[e];
    __threadfence_system();
    __syncthreads();
    const unsigned long long tag = step + 1;
    if (tid < world && tid != rank) {
        unsigned long long* flag = reinterpret_cast<unsigned long long*>(peers[tid]) + rank;
        st_release_sys(flag, tag);
    }
    if (tid < world && tid != rank) {
        const unsigned long long* flag = reinterpret_cast<const unsigned long long*>(mine) + tid;
        uint32_t i = 0;
        while (ld_acquire_sys(flag) < tag) {
            if (++i == kExSpin) {
                s_fail = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (s_fail) {
        if (tid == 0) atomicOr(reinterpret_cast<unsigned long long*>(&counters[1]), (unsigned long long)kFlagExchange);
        return;
    }
    for (int64_t e = tid; e < W; e += kExThreads) {
        long long s = 0;
        for (int r = 0; r < world; r++) {
            const long long* slot = reinterpret_cast<const long long*>(reinterpret_cast<const char*>(peers[r]) + slot_off);
            s += slot[e];
        }
        totals[e] = s;
    }
}

}  // namespace

size_t exchange_bytes(int k, int d) { return (size_t)kExchangeHeader + 2 * (size_t)k * (d + 2) * 8; }

cudaError_t launch_exchange_sum(long long* totals, int k, int d, const unsigned long long* peers, int world, int rank,
                                unsigned long long step, long long* counters, cudaStream_t st) {
    k_exchange_sum<<<1, kExThreads, 0, st>>>(totals, (int64_t)k * (d + 2), peers, world, rank, step, counters);
    return cudaGetLastError();
}

}  // namespace kmc
