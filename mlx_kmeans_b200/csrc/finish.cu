// finish.cu -- the end of a Lloyd step on the device: far-row candidates, empty-cluster relocation,
// center divide, still-empty rule, statistics (reference: core.py:2223-2241), and the unpacking of
// totals into the float64 sums / int64 counts that core.py:2200-2206 `assign_mlx` returns.
#include "common.cuh"
#include "kmc_internal.h"
#include "exchange.cuh"

namespace kmc {

// ---------------------------------------------------------------- far rows (radix select)
// Key of a row: best's float bits in the high word (best >= 0, so the bits order like the values),
// ~local_index in the low word, so larger key = farther, then lower row index: the order of
// core.py:2227-2229.  Keys are unique; an MSB-first radix select finds the cand_rows-th largest key in
// eight 8-bit passes, then every row with a key at least that large is collected and ranked.
__device__ __forceinline__ unsigned long long far_key(const float* best, int64_t i) {
    unsigned int b = __float_as_uint(best[i]);
    if (b & 0x80000000u) b = 0u;                     // -0.0 (cannot occur) sorts as 0
    return ((unsigned long long)b << 32) | (unsigned long long)(0xffffffffu - (unsigned int)i);
}

__global__ void k_rs_hist(const float* __restrict__ best, int64_t n, const unsigned long long* __restrict__ rs,
                          int shift, unsigned int* __restrict__ hist) {
    __shared__ unsigned int h[256];
    h[threadIdx.x] = 0u;
    __syncthreads();
    const unsigned long long prefix = rs[0], mask = rs[1];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        unsigned long long key = far_key(best, i);
        if ((key & mask) == prefix) atomicAdd(&h[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (h[threadIdx.x]) atomicAdd(&hist[threadIdx.x], h[threadIdx.x]);
}

// rs: [0] prefix, [1] mask, [2] rows still to take, [3] 1 when fewer rows than wanted exist (take all)
__global__ void k_rs_pick(unsigned long long* rs, unsigned int* hist, int shift) {
    if (threadIdx.x != 0) return;
    unsigned long long rem = rs[2];
    unsigned long long cum = 0;
    int b = 255;
    for (; b >= 0; b--) {
        if (cum + hist[b] >= rem) break;
        cum += hist[b];
    }
    if (b < 0) {                                     // fewer candidates than wanted: take every row
        rs[0] = 0ull;
        rs[1] = ~0ull;
        rs[3] = 1ull;
        rs[2] = 0ull;
    } else if (!rs[3]) {
        rs[0] |= (unsigned long long)b << shift;
        rs[1] |= 255ull << shift;
        rs[2] = rem - cum;
    }
    for (int i = 0; i < 256; i++) hist[i] = 0u;
}

__global__ void k_rs_collect(const float* __restrict__ best, int64_t n, const unsigned long long* __restrict__ rs,
                             unsigned long long* __restrict__ keys, unsigned long long* __restrict__ count,
                             int64_t cap) {
    const unsigned long long thr = rs[3] ? 0ull : rs[0];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        unsigned long long key = far_key(best, i);
        if (key >= thr) {
            unsigned long long slot = atomicAdd(count, 1ull);
            if ((int64_t)slot < cap) keys[slot] = key;
        }
    }
}

// Rank the collected keys (descending) and write the candidate records.
__global__ void k_rs_emit(const float* __restrict__ X, int d, const int32_t* __restrict__ labels,
                          const float* __restrict__ best, int64_t row0, const unsigned long long* __restrict__ keys,
                          const unsigned long long* __restrict__ count, int64_t cap, uint32_t* __restrict__ cands) {
    const int64_t m = (int64_t)(*count < (unsigned long long)cap ? *count : (unsigned long long)cap);
    const int W = d + 4;
    for (int64_t s = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; s < cap; s += (int64_t)gridDim.x * blockDim.x) {
        if (s >= m) {                                // padding record
            uint32_t* r = cands + s * W;
            r[0] = __float_as_uint(-1.0f);
            r[1] = 0xffffffffu;
            r[2] = 0x7fffffffu;
            r[3] = 0u;
            continue;
        }
        const unsigned long long key = keys[s];
        int64_t rank = 0;
        for (int64_t t = 0; t < m; t++) rank += keys[t] > key;
        const int64_t i = (int64_t)(0xffffffffu - (unsigned int)(key & 0xffffffffull));
        const int64_t g = row0 + i;
        uint32_t* r = cands + rank * W;
        r[0] = __float_as_uint(best[i]);
        r[1] = (uint32_t)(g & 0xffffffff);
        r[2] = (uint32_t)(g >> 32);
        r[3] = (uint32_t)labels[i];
        for (int j = 0; j < d; j++) r[4 + j] = __float_as_uint(X[i * d + j]);
    }
}

__global__ void k_rs_init(unsigned long long* rs, unsigned int* hist, unsigned long long want) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0u;
    if (threadIdx.x < 8) rs[threadIdx.x] = threadIdx.x == 2 ? want : 0ull;
}

cudaError_t launch_far_rows(const float* X, int64_t n, int d, const int32_t* labels, const float* best, int64_t row0,
                            int64_t cand_rows, uint32_t* cands, const FarWorkspace& ws, cudaStream_t st) {
    k_rs_init<<<1, 256, 0, st>>>(ws.rs, ws.hist, (unsigned long long)cand_rows);
    int blocks = num_sms() * 4;
    int64_t need = (n + 255) / 256;
    if (need < blocks) blocks = (int)(need > 0 ? need : 1);
    for (int shift = 56; shift >= 0; shift -= 8) {
        k_rs_hist<<<blocks, 256, 0, st>>>(best, n, ws.rs, shift, ws.hist);
        k_rs_pick<<<1, 32, 0, st>>>(ws.rs, ws.hist, shift);
    }
    unsigned long long* count = ws.rs + 4;           // rs[4]: collected rows (zeroed by k_rs_init)
    k_rs_collect<<<blocks, 256, 0, st>>>(best, n, ws.rs, ws.keys, count, cand_rows);
    int eb = (int)((cand_rows + 255) / 256);
    k_rs_emit<<<eb > 0 ? eb : 1, 256, 0, st>>>(X, d, labels, best, row0, ws.keys, count, cand_rows, cands);
    return cudaGetLastError();
}

// ---------------------------------------------------------------- finish
// One CTA of 1024 threads.  totals are updated in place by the relocation (counts and sums move).  Above
// kFinishOneCta center values the divide (steps 4 and 5) runs on a grid instead (k_finish_centers): the CTA
// leaves the largest cluster in counters[3] and whether to write the centers in counters[4].
constexpr int64_t kFinishOneCta = 32768;

struct FinishArgs {
    long long* totals;
    int k, d;
    const double* scale_x;
    const Prep* prep;
    const uint32_t* cands;
    int64_t cand_rows;
    int ranks;
    float* C_new;
    Stats* stats;
    long long* counters;
    int* reloc;
    long long* empty;
    bool grid_centers;
    const unsigned long long* peers;   // the all-reduce over peer memory first (nullptr: none)
    int world, rank;
    unsigned long long step;
    unsigned long long timeout_ns;     // how long the exchange waits for a peer
    LoopState* loop;                   // a device Lloyd loop's record (kmc_lloyd), or nullptr
};

// After a step of a device Lloyd loop (thread 0 of k_finish): the reference's stopping rule (estimator.py:132-150).
__device__ void loop_after_step(LoopState* L, const Stats& s) {
    if (s.flags & kFlagNonFinite || !(s.inertia <= 1.0e308)) {
        L->state = kLoopNonFinite;
        return;
    }
    if (s.needs_reloc) {                     // the host relocates, finishes this step and resumes the loop
        L->state = kLoopRelocate;
        return;
    }
    L->steps += 1;
    if (L->have_prev && fabs(L->prev_inertia - s.inertia) <= L->tol * L->prev_inertia) L->state = kLoopConverged;
    else if (L->steps >= L->max_steps) L->state = kLoopMaxSteps;
    L->prev_inertia = s.inertia;
    L->have_prev = 1;
}

__global__ void k_loop_init(LoopState* L, double tol, long long max_steps, long long steps, double prev, int have_prev) {
    L->prev_inertia = prev;
    L->tol = tol;
    L->steps = steps;
    L->max_steps = max_steps;
    L->state = steps >= max_steps ? kLoopMaxSteps : kLoopRunning;
    L->have_prev = have_prev;
    L->reserved[0] = L->reserved[1] = 0;
}

// center c, column j of the new centers (cnt = the cluster's count, > 0): sums / counts in float64, rounded
// once to float32; a cluster relocated into from a single row is that row
__device__ __forceinline__ float new_center(const FinishArgs& a, int c, int j, long long cnt) {
    if (a.reloc[c] >= 0 && cnt == 1) return __uint_as_float(a.cands[(int64_t)a.reloc[c] * (a.d + 4) + 4 + j]);
    const double s = __dmul_rn((double)a.totals[(size_t)c * (a.d + 2) + 2 + j], 1.0 / a.scale_x[j]);
    return __double2float_rn(__ddiv_rn(s, (double)cnt));
}

__global__ void __launch_bounds__(1024) k_finish(FinishArgs a) {
    const int k = a.k, d = a.d, W = d + 2;
    const int tid = threadIdx.x, nt = blockDim.x;
    __shared__ long long s_in[32];
    __shared__ long long s_ne[32];
    __shared__ long long s_bigc[32];
    __shared__ int s_bigi[32];
    __shared__ long long sh_n_empty, sh_inert, sh_nreloc;
    __shared__ int sh_big, sh_write, sh_xfail;
    pdl_wait();                                        // the pass's totals (or the exchange's)
    if (a.loop && a.loop->state != kLoopRunning) {    // the device loop stopped: nothing to do (read before any
        if (tid == 0 && a.grid_centers) a.counters[4] = 0;   // thread writes the record, after the barriers below)
        return;
    }
    // 0. (fused step tail) the totals summed over the ranks
    if (a.peers)
        exchange_cta(a.totals, (int64_t)k * W, 0, (int64_t)k * W, 0, a.peers, a.world, a.rank, a.step, a.timeout_ns,
                     a.counters, &sh_xfail);
    // 1. inertia (exact int64 sum) and empty count, before any relocation (core.py:2223)
    long long in = 0, ne = 0;
    for (int c = tid; c < k; c += nt) {
        in += a.totals[(size_t)c * W + 1];
        ne += a.totals[(size_t)c * W] == 0;
        a.reloc[c] = -1;
    }
    for (int o = 16; o; o >>= 1) {
        in += __shfl_xor_sync(0xffffffffu, in, o);
        ne += __shfl_xor_sync(0xffffffffu, ne, o);
    }
    if ((tid & 31) == 0) { s_in[tid >> 5] = in; s_ne[tid >> 5] = ne; }
    __syncthreads();
    if (tid == 0) {
        long long ti = 0, tn = 0;
        for (int w = 0; w < nt / 32; w++) { ti += s_in[w]; tn += s_ne[w]; }
        sh_inert = ti;
        sh_n_empty = tn;
        sh_nreloc = 0;
        sh_write = 1;
        // 2. relocation (core.py:2224-2236): empties in ascending order, farthest rows first
        if (tn > 0) {
            if (a.cands == nullptr) {
                sh_write = 0;                        // the caller gathers candidates and finishes again
            } else {
                int ne_list = 0;
                for (int c = 0; c < k; c++) if (a.totals[(size_t)c * W] == 0) a.empty[ne_list++] = c;
                const int R = d + 4;
                const int64_t E = a.cand_rows;
                // ranks' lists are each sorted; merge by (best desc, global row asc)
                int64_t head[64];
                for (int r = 0; r < a.ranks && r < 64; r++) head[r] = 0;
                float best_max = -1.0f;
                long long moved = 0;
                for (int e = 0; e < ne_list; e++) {
                    int pick = -1;
                    float pb = 0.0f;
                    unsigned long long pg = 0;
                    for (int r = 0; r < a.ranks && r < 64; r++) {
                        if (head[r] >= E) continue;
                        const uint32_t* rec = a.cands + ((int64_t)r * E + head[r]) * R;
                        float b = __uint_as_float(rec[0]);
                        if (b < 0.0f) continue;       // padding
                        unsigned long long g = (unsigned long long)rec[1] | ((unsigned long long)rec[2] << 32);
                        if (pick < 0 || b > pb || (b == pb && g < pg)) { pick = r; pb = b; pg = g; }
                    }
                    if (pick < 0) break;
                    if (e == 0) best_max = pb;
                    if (!(best_max > 0.0f)) break;    // core.py:2226: only when some row is off its center
                    const uint32_t* rec = a.cands + ((int64_t)pick * E + head[pick]) * R;
                    head[pick]++;
                    const int c_new = (int)a.empty[e];
                    const int old = (int)rec[3];
                    long long* to = a.totals + (size_t)old * W;
                    long long* tn_ = a.totals + (size_t)c_new * W;
                    to[0] -= 1;
                    tn_[0] = 1;
                    for (int j = 0; j < d; j++) {
                        long long q = quantize(__uint_as_float(rec[4 + j]), a.scale_x[j]);
                        to[2 + j] -= q;
                        tn_[2 + j] = q;
                    }
                    a.reloc[c_new] = (int)(((int64_t)pick * E + head[pick] - 1));
                    moved++;
                }
                sh_nreloc = moved;
            }
        }
    }
    __syncthreads();
    if (!sh_write) {
        if (tid == 0 && a.grid_centers) a.counters[4] = 0;
        if (tid == 0) {
            Stats s;
            s.inertia = (double)sh_inert * a.prep->inv_scale_i;
            s.n_empty = sh_n_empty;
            s.n_relocated = 0;
            s.needs_reloc = 1;
            s.flags = (long long)a.prep->flags | a.counters[1];
            s.rescored = a.counters[0];
            s.screened = a.counters[2];
            s.pad = 0;
            *a.stats = s;
            if (a.loop) loop_after_step(a.loop, s);
        }
        return;
    }
    // 3. largest cluster (np.argmax: first maximum), after relocation
    long long bc = -1;
    int bi = 0;
    for (int c = tid; c < k; c += nt) {
        long long v = a.totals[(size_t)c * W];
        if (v > bc) { bc = v; bi = c; }
    }
    for (int o = 16; o; o >>= 1) {
        long long ov = __shfl_xor_sync(0xffffffffu, bc, o);
        int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bc || (ov == bc && oi < bi)) { bc = ov; bi = oi; }
    }
    if ((tid & 31) == 0) { s_bigc[tid >> 5] = bc; s_bigi[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
        long long b = s_bigc[0];
        int i = s_bigi[0];
        for (int w = 1; w < nt / 32; w++)
            if (s_bigc[w] > b || (s_bigc[w] == b && s_bigi[w] < i)) { b = s_bigc[w]; i = s_bigi[w]; }
        sh_big = i;
        if (a.grid_centers) {
            a.counters[3] = i;
            a.counters[4] = 1;
        }
    }
    if (!a.grid_centers) {
        // 4. C_new = sums / counts (float64, rounded once to float32); a relocated cluster is its row
        for (int64_t e = tid; e < (int64_t)k * d; e += nt) {
            const int c = (int)(e / d), j = (int)(e % d);
            const long long cnt = a.totals[(size_t)c * W];
            if (cnt > 0) a.C_new[e] = new_center(a, c, j, cnt);
        }
        __syncthreads();
        // 5. a cluster still empty takes the largest cluster's center (core.py:2241)
        const int big = sh_big;
        for (int64_t e = tid; e < (int64_t)k * d; e += nt) {
            const int c = (int)(e / d), j = (int)(e % d);
            if (a.totals[(size_t)c * W] <= 0) a.C_new[e] = a.C_new[(int64_t)big * d + j];
        }
    }
    if (tid == 0) {
        Stats s;
        s.inertia = (double)sh_inert * a.prep->inv_scale_i;
        s.n_empty = sh_n_empty;
        s.n_relocated = sh_nreloc;
        s.needs_reloc = 0;
        s.flags = (long long)a.prep->flags | a.counters[1];
        s.rescored = a.counters[0];
        s.screened = a.counters[2];
        s.pad = 0;
        *a.stats = s;
        if (a.loop) loop_after_step(a.loop, s);
    }
}

// Steps 4 and 5 of k_finish over a grid (many center values): every value computed from the totals, an empty
// cluster's from the largest cluster's, so no value waits for another thread's.
__global__ void __launch_bounds__(256) k_finish_centers(FinishArgs a) {
    pdl_wait();                                      // k_finish's record
    if (a.counters[4] == 0) return;                  // relocation pending: the centers are not written
    const int k = a.k, d = a.d, W = d + 2;
    const int big = (int)a.counters[3];
    const long long cb = a.totals[(size_t)big * W];
    const int64_t total = (int64_t)k * d;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e / d), j = (int)(e % d);
        const long long cnt = a.totals[(size_t)c * W];
        if (cnt > 0) a.C_new[e] = new_center(a, c, j, cnt);
        else a.C_new[e] = cb > 0 ? new_center(a, big, j, cb) : a.C_new[(int64_t)big * d + j];
    }
}

cudaError_t launch_finish(long long* totals, int k, int d, const uint32_t* cands, int64_t cand_rows, int ranks,
                          float* C_new, void* stats, const Workspace& ws, cudaStream_t st,
                          const unsigned long long* peers, int world, int rank, unsigned long long step,
                          void* loop) {
    if (peers && exchange_wide(k, d)) {         // wide totals: the multi-CTA exchange as a launch of its own
        cudaError_t e = launch_exchange_sum(totals, k, d, peers, world, rank, step, ws.counters, st);
        if (e != cudaSuccess) return e;
        peers = nullptr;
    }
    FinishArgs a;
    a.loop = static_cast<LoopState*>(loop);
    a.totals = totals;
    a.k = k;
    a.d = d;
    a.scale_x = ws.scale_x;
    a.prep = ws.prep;
    a.cands = cands;
    a.cand_rows = cand_rows;
    a.ranks = ranks;
    a.C_new = C_new;
    a.stats = reinterpret_cast<Stats*>(stats);
    a.counters = ws.counters;
    a.reloc = ws.reloc;
    a.empty = ws.empty;
    a.peers = peers;
    a.world = world;
    a.rank = rank;
    a.step = step;
    a.timeout_ns = peers ? exchange_timeout_ns() : 0;
    const int64_t total = (int64_t)k * d;
    a.grid_centers = total > kFinishOneCta;
    cudaError_t e = launch_pdl(k_finish, dim3(1), dim3(1024), 0, st, a);
    if (e != cudaSuccess) return e;
    if (a.grid_centers) {
        int64_t blocks = (total + 255) / 256;
        if (blocks > (int64_t)num_sms() * 8) blocks = (int64_t)num_sms() * 8;
        e = launch_pdl(k_finish_centers, dim3((unsigned)blocks), dim3(256), 0, st, a);
    }
    return e;
}

// ---------------------------------------------------------------- unpack (assign_mlx's return values)
__global__ void k_unpack(const long long* __restrict__ totals, int k, int d, const double* __restrict__ scale_x,
                         const Prep* __restrict__ prep, const long long* __restrict__ counters,
                         double* __restrict__ sums, int64_t* __restrict__ counts, double* __restrict__ inertia) {
    const int W = d + 2;
    const int64_t total = (int64_t)k * d;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(e / d), j = (int)(e % d);
        sums[e] = __dmul_rn((double)totals[(size_t)c * W + 2 + j], 1.0 / scale_x[j]);
    }
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < k; c += (int64_t)gridDim.x * blockDim.x)
        counts[c] = totals[(size_t)c * W];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        long long t = 0;
        for (int c = 0; c < k; c++) t += totals[(size_t)c * W + 1];
        const bool bad = (prep->flags | counters[1]) & kFlagNonFinite;
        *inertia = bad ? __longlong_as_double(0x7ff8000000000000ll) : (double)t * prep->inv_scale_i;
    }
}

cudaError_t launch_loop_init(void* loop, double tol, long long max_steps, long long steps, double prev_inertia,
                             int have_prev, cudaStream_t st) {
    k_loop_init<<<1, 1, 0, st>>>(static_cast<LoopState*>(loop), tol, max_steps, steps, prev_inertia, have_prev);
    return cudaGetLastError();
}

cudaError_t launch_unpack(const long long* totals, int k, int d, const double* scale_x, const Prep* prep,
                          const long long* counters, double* sums, int64_t* counts, double* inertia, cudaStream_t st) {
    int64_t total = (int64_t)k * d;
    int blocks = (int)((total + 255) / 256);
    if (blocks > 1024) blocks = 1024;
    k_unpack<<<blocks, 256, 0, st>>>(totals, k, d, scale_x, prep, counters, sums, counts, inertia);
    return cudaGetLastError();
}

}  // namespace kmc
