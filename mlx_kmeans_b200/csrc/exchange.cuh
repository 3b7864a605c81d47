// exchange.cuh -- the all-reduce of the per-cluster totals over the GPUs of one node, through peer memory, as
// the work of one CTA (k_exchange_sum launches it alone; k_finish runs it first when the step's tail is fused).
//
// The rank copies its totals into its own exchange buffer, raises its flag in every peer's buffer (a release
// store over NVLink, after a CTA barrier), waits for every peer's flag (acquire loads of its own buffer, for at most a set time), and sums all
// ranks' totals with plain peer loads.  The sum of integers does not depend on the order, so the result is the
// same as NCCL's and the same on every rank.
//
// Exchange buffer of a rank (kmc_exchange_alloc; the peers map it through CUDA IPC):
//   [flags: 64 rows x 64 uint64; flag (b, r) = the last step rank r has published through row b]
//   [slot 0: W int64]  [slot 1: W int64]
// Step s publishes into slot s & 1.  One CTA exchanges a range of the totals through one flag row: row 0 and
// every value for narrow totals, CTA b of the wide exchange (k_exchange_wide) row b and the b-th range.  A rank
// writes slot s & 1 again at step s + 2 only after it has seen, in some row, every peer's flag for step s + 1;
// a peer raises a flag for step s + 1 in a kernel that starts after its step-s kernel (every CTA of it) finished
// reading, so two slots suffice whichever rows the steps used.
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

// The whole CTA calls this for the values [e0, e1) of the W totals, through flag row `row`; `fail` is a shared
// int.  On a timeout those totals keep the rank's own values and counters[1] gets kFlagExchange.  Ends with the
// summed totals visible to the CTA (a barrier).
__device__ inline void exchange_cta(long long* __restrict__ totals, int64_t W, int64_t e0, int64_t e1, int row,
                                    const unsigned long long* __restrict__ peers, int world, int rank,
                                    unsigned long long step, unsigned long long timeout_ns,
                                    long long* __restrict__ counters, int* fail) {
    const int tid = threadIdx.x, nt = blockDim.x;
    if (tid == 0) *fail = 0;
    const size_t slot_off = (size_t)kExchangeHeader + (size_t)(step & 1) * (size_t)W * 8;
    char* mine = reinterpret_cast<char*>(peers[rank]);
    long long* my_slot = reinterpret_cast<long long*>(mine + slot_off);
    for (int64_t e = e0 + tid; e < e1; e += nt) my_slot[e] = totals[e];
    // the barrier orders every thread's slot writes before the flag stores below, and a system-scope release store
    // is cumulative: a peer that acquires the flag sees the whole range (no fence per thread)
    __syncthreads();
    const unsigned long long tag = step + 1;
    if (tid < world && tid != rank) {
        unsigned long long* flag = reinterpret_cast<unsigned long long*>(peers[tid]) + row * 64 + rank;
        st_release_sys(flag, tag);
        const unsigned long long* own = reinterpret_cast<const unsigned long long*>(mine) + row * 64 + tid;
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
    // Two values per thread per round, and the values of up to eight ranks requested before any is added: all of
    // those loads are in flight over NVLink together, so the sum costs one round trip per eight ranks rather than
    // one per rank (an add that waits on each load before the next is issued serialises the ranks)
    constexpr int R = 8, U = 2;
    for (int64_t e = e0 + tid; e < e1; e += U * (int64_t)nt) {
        long long s[U] = {};
        for (int r0 = 0; r0 < world; r0 += R) {
            const long long* slot[R];
#pragma unroll
            for (int j = 0; j < R; j++)
                slot[j] = r0 + j < world
                              ? reinterpret_cast<const long long*>(reinterpret_cast<const char*>(peers[r0 + j]) + slot_off)
                              : nullptr;
            long long v[R][U];
#pragma unroll
            for (int j = 0; j < R; j++)
#pragma unroll
                for (int u = 0; u < U; u++)
                    v[j][u] = (slot[j] != nullptr && e + (int64_t)u * nt < e1) ? slot[j][e + (int64_t)u * nt] : 0;
#pragma unroll
            for (int j = 0; j < R; j++)
#pragma unroll
                for (int u = 0; u < U; u++) s[u] += v[j][u];
        }
#pragma unroll
        for (int u = 0; u < U; u++)
            if (e + (int64_t)u * nt < e1) totals[e + (int64_t)u * nt] = s[u];
    }
    __syncthreads();
}

}  // namespace kmc
