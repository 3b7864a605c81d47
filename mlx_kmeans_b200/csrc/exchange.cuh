// exchange.cuh -- the all-reduce of the per-cluster totals over the GPUs of one node, through peer memory, as
// the work of one CTA (k_exchange_sum launches it alone; k_finish runs it first when the step's tail is fused).
//
// The rank copies its totals into its own exchange buffer, raises its flag in every peer's buffer (a release
// store over NVLink), waits for every peer's flag (acquire loads of its own buffer, for at most a set time), and sums all
// ranks' totals with plain peer loads.  The sum of integers does not depend on the order, so the result is the
// same as NCCL's and the same on every rank.
//
// Exchange buffer of a rank (kmc_exchange_alloc; the peers map it through CUDA IPC):
//   [flags: 64 x uint64; flag r = the last step rank r has published]  [slot 0: W int64]  [slot 1: W int64]
// Step s publishes into slot s & 1.  A rank writes slot s & 1 again at step s + 2 only after it has seen every
// peer's flag for step s + 1, which each peer raises after it finished reading step s: two slots suffice.
#pragma once
#include "common.cuh"
#include "kmc_internal.h"

namespace kmc {

// A wait on a peer gives up after timeout_ns nanoseconds of the GPU's global timer (the limit comes from the
// host: exchange_timeout_ns()).
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The whole CTA calls this; `fail` is a shared int.  On a timeout the totals keep the rank's own values and
// counters[1] gets kFlagExchange.  Ends with the summed totals visible to the CTA (a barrier).
__device__ inline void exchange_cta(long long* __restrict__ totals, int64_t W,
                                    const unsigned long long* __restrict__ peers, int world, int rank,
                                    unsigned long long step, unsigned long long timeout_ns,
                                    long long* __restrict__ counters, int* fail) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) *fail = 0;
    const size_t slot_off = (size_t)kExchangeHeader + (size_t)(step & 1) * (size_t)W * 8;
    char* mine = reinterpret_cast<char*>(peers[rank]);
    long long* my_slot = reinterpret_cast<long long*>(mine + slot_off);
    for (int64_t e = tid; e < W; e += nt) my_slot[e] = totals[e];
    __threadfence_system();
    __syncthreads();
    const unsigned long long tag = step + 1;
    if (tid < world && tid != rank) {
        unsigned long long* flag = reinterpret_cast<unsigned long long*>(peers[tid]) + rank;
        st_release_sys(flag, tag);
        const unsigned long long* own = reinterpret_cast<const unsigned long long*>(mine) + tid;
        const unsigned long long t0 = global_ns();
        uint32_t i = 0;
        while (ld_acquire_sys(own) < tag) {
            if ((++i & 63u) == 0 && global_ns() - t0 > timeout_ns) {
                *fail = 1;
                break;
            }
        }
    }
    __syncthreads();
    if (*fail) {
        if (tid == 0) atomicOr(reinterpret_cast<unsigned long long*>(&counters[1]), (unsigned long long)kFlagExchange);
        __syncthreads();
        return;
    }
    for (int64_t e = tid; e < W; e += nt) {
        long long s = 0;
        for (int r = 0; r < world; r++) {
            const long long* slot = reinterpret_cast<const long long*>(reinterpret_cast<const char*>(peers[r]) + slot_off);
            s += slot[e];
        }
        totals[e] = s;
    }
    __syncthreads();
}

}  // namespace kmc
