// kmc_internal.h -- shared declarations of the kmc CUDA library (not part of the public ABI).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

#include "common.cuh"

namespace kmc {

int num_sms();

// The launch of a kernel that begins with pdl_wait(): with programmatic stream serialisation it is scheduled as
// the kernel before it in the stream finishes (its launch and set-up overlap that kernel's tail) instead of after.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Arguments of the pass kernels.
struct PassArgs {
    const float* X;
    int64_t n;
    int d, k;
    const float* C;
    const float* hc;          // k: |c|^2 / 2 (float32)
    const double* scale_x;    // d: 2^shift per column
    const Prep* prep;
    long long* totals;        // k x (d+2)
    int32_t* labels;          // optional
    float* best;              // optional
    long long* counters;      // [0] rows re-scored, [1] flags
    int smem_acc;             // generic kernel: accumulate in shared memory
    int ctile;                // generic kernel: centers per shared tile
    unsigned key_keep;        // fused low-d kernel: ~(center index bits) of a key
    uint32_t* brows;          // bounded pass: one bound word per row (nullptr: plain pass)
    const float* hsep;        // bounded pass: per center, (half its distance to the nearest other center)^2
    int64_t n_total;          // rows of the whole dataset (all slices and GPUs): sets the fixed-point grids
    int rpl;                  // fused low-d kernels: rows per lane between folds (from n_total: the block size)
};

// Bounds state of one slice (caller memory): [meta: double drift, double valid; at byte 128: hsep, k <= 32 floats]
// [centers of the last pass][one word per row].
struct BoundsState {
    double* meta;
    float* hsep;              // k: (s_c / 2)^2 rounded down, s_c = distance from center c to its nearest other one
    float* cprev;             // k x d
    uint32_t* rows;           // n
};
BoundsState carve_bounds(void* base, int64_t n, int d, int k);
size_t bounds_bytes(int64_t n, int d, int k);
bool lowd_supports(int d, int k);

// Pass workspace carve-up (256-byte aligned pieces): kmc_pass writes prep/scale_x/hc/counters,
// kmc_finish and kmc_totals_unpack read them.
struct Workspace {
    Prep* prep;
    long long* counters;      // 8: [0] rows re-scored, [1] flags, [2] rows screened, [3] largest cluster and
                              // [4] centers to write (k_finish -> k_finish_centers)
    double* scale_x;          // d
    float* hc;                // k
    int* reloc;               // k: candidate slot relocated into cluster c, or -1
    long long* empty;         // k: empty cluster list
    size_t bytes;
};
Workspace carve(void* base, int d, int k);

// Far-rows workspace.
struct FarWorkspace {
    unsigned long long* rs;   // radix-select state: [0] prefix [1] mask [2] remaining [3] take-all [4] collected
    unsigned int* hist;       // 256
    unsigned long long* keys; // cand_rows collected keys
    size_t bytes;
};
FarWorkspace carve_far(void* base, int64_t cand_rows);

cudaError_t launch_d64(const float* X, const float* C, int d, int64_t m, double* out, cudaStream_t st);
cudaError_t launch_colmax(const float* X, int64_t n, int d, unsigned int* colmax, cudaStream_t st);
// per-pass constants; optionally clears the totals and counters, and (bmeta != nullptr) prepares a bounded pass
cudaError_t launch_prepare(const float* C, int k, int d, const unsigned int* colmax, int64_t n_total, Prep* prep,
                           double* scale_x, float* hc, long long* zero_totals, long long* zero_counters,
                           double* bmeta, float* bcprev, float* bhsep, int rule, cudaStream_t st,
                           const void* loop = nullptr);
cudaError_t launch_pass_generic(PassArgs a, cudaStream_t st);
// Specialised low-dimensional fused pass; returns cudaErrorNotSupported when (d, k) has no instance.
cudaError_t launch_pass_lowd(PassArgs a, cudaStream_t st);
int64_t lowd_block_rows(int64_t n_total);

// Tensor-core pass (d >= 32): per-slice operands, computed once per dataset ...
struct RowSplit {
    void* xh;                 // n x dp bf16, x rounded to bf16
    void* xl;                 // n x dp bf16, the rest rounded to bf16
    float* xn;                // n: |x| rounded up
    int32_t* lab;             // n: label | flag << 31 from the tensor-core kernel, then the final label
    uint32_t* perm;           // n: rows grouped by label (before that: the rows the tensor-core kernel flagged)
    int4* cands;              // n: each flagged row's candidate centers (x, y; w = -2: more than two)
    uint32_t* ovf;            // n: flagged rows with more than two candidates
    float* xsq_lo;            // n: |x|^2 rounded down (the Elkan bounds' lower bound on distances)
};
// ... and per-pass center operands
struct CenterSplit {
    unsigned int* cmax_bits;  // max |c| rounded up (float bits)
    int* error;               // set when the tensor-core kernel timed out on a barrier
    unsigned int* nflag;      // rows the tensor-core kernel left to float64 (listed in RowSplit::perm)
    unsigned int* novf;       // of those, rows with more than two candidates (listed in RowSplit::ovf)
    float* ct;                // d x k: the centers transposed, for the float64 decision's float32 screen
    void* ch;                 // kp x dp bf16
    void* cl;                 // kp x dp bf16
    float* hs;                // kp: |c|^2 / 2 (padding centers 2^126)
    unsigned int* hist;       // k: rows per label
    unsigned int* cursor;     // k: next slot of each label in the grouped rows
};
struct TcSplit {
    int64_t n;
    int dp, kp, k;
    const void *xh, *xl, *ch, *cl;
    const float* hs;
    const float* xn;
    const float* cmax;
    int32_t* lab;
    int4* cands;
    int* error;
    float* dump;              // kmc_tc_dot: n x k raw scores x.c, or nullptr
    int rule;                 // label rule (Prep::rule): widens the window
    int approx;               // exact=False: one bf16 MMA per product (hi parts), no window
    void* lb;                 // Elkan bounds to build (n x k half), or nullptr
    const float* xsq_lo;      // n: |x|^2 rounded down (with lb or mask)
    void* mask = nullptr;     // the cascade's survivor bits to build (n x ceil(k/32) words), or nullptr
    const float* ub = nullptr;   // n: the cascade's per-row threshold (with mask)
    const int32_t* plab = nullptr;   // n: the previous labels (with mask)
    uint32_t* srows = nullptr;       // the rows with survivors besides that label (with mask), and their count
    unsigned int* nsrows = nullptr;
};
int split_dp(int d);
int split_kp(int k);
int tc_block_n(int k);
size_t split_rows_bytes(int64_t n, int d);
size_t split_centers_bytes(int d, int k);
RowSplit carve_rows(void* base, int64_t n, int d);
CenterSplit carve_centers(void* base, int d, int k);
cudaError_t launch_split_rows(const float* X, int64_t n, int d, const RowSplit& s, cudaStream_t st);
cudaError_t launch_split_centers(const float* C, int k, int d, const CenterSplit& s, cudaStream_t st);
cudaError_t launch_assign_tc(const TcSplit& s, cudaStream_t st);
cudaError_t launch_accum_split(PassArgs a, const RowSplit& rs, const CenterSplit& cs, cudaStream_t st);

// Per-center lower bounds between passes for the tensor-core shapes (elkan.cu): caller memory
// [centers the bounds refer to: k x d float][drift: k float][bounds: n x k half].
// The prefix-pruning cascade's per-slice state (elkan.cu): caller memory [count of listed rows][threshold: n float]
// [survivors: n x ceil(k/32) 32-bit words][listed rows: n].
struct CascadeState {
    unsigned int* nsrows;
    float* ub;
    uint32_t* mask;
    uint32_t* srows;
};
size_t cascade_bytes(int64_t n, int k);
CascadeState carve_cascade(void* base, int64_t n, int k);
cudaError_t launch_cascade_ub(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                              const int32_t* lab, const Prep* prep, cudaStream_t st);
cudaError_t launch_cascade(const float* X, int64_t n, int d, const float* C, int k, const CascadeState& cs,
                           int32_t* lab, int4* cands, const Prep* prep, long long* counters, cudaStream_t st);

struct ElkanState {
    float* cprev;
    float* drift;
    void* lb;
};
size_t elkan_bytes(int64_t n, int d, int k);
ElkanState carve_elkan(void* base, int64_t n, int d, int k);
cudaError_t launch_elkan_drift(const float* C, const ElkanState& e, int k, int d, cudaStream_t st);
cudaError_t launch_elkan(const float* X, int64_t n, int d, const float* C, int k, const ElkanState& e, int32_t* lab,
                         int4* cands, const uint32_t* order, const Prep* prep, long long* counters, cudaStream_t st);

// Peer-memory all-reduce of the totals (exchange.cu).
constexpr int kExchangeRows = 64;         // flag rows: the exchange of wide totals runs one CTA per row
constexpr int kExchangeHeader = kExchangeRows * 64 * 8;   // 64 rows x 64 ranks' flags of 8 bytes before the slots
constexpr int64_t kExchangeWideMin = 16384;  // totals of at least this many int64 values take the multi-CTA exchange
size_t exchange_bytes(int k, int d);
unsigned long long exchange_timeout_ns();
cudaError_t launch_exchange_sum(long long* totals, int k, int d, const unsigned long long* peers, int world, int rank,
                                unsigned long long step, long long* counters, cudaStream_t st);
bool exchange_wide(int k, int d);

cudaError_t launch_far_rows(const float* X, int64_t n, int d, const int32_t* labels, const float* best, int64_t row0,
                            int64_t cand_rows, uint32_t* cands, const FarWorkspace& ws, cudaStream_t st);
cudaError_t launch_finish(long long* totals, int k, int d, const uint32_t* cands, int64_t cand_rows, int ranks,
                          float* C_new, void* stats, const Workspace& ws, cudaStream_t st,
                          const unsigned long long* peers = nullptr, int world = 1, int rank = 0,
                          unsigned long long step = 0, void* loop = nullptr);
cudaError_t launch_loop_init(void* loop, double tol, long long max_steps, long long steps, double prev_inertia,
                             int have_prev, cudaStream_t st);
cudaError_t launch_unpack(const long long* totals, int k, int d, const double* scale_x, const Prep* prep,
                          const long long* counters, double* sums, int64_t* counts, double* inertia, cudaStream_t st);

cudaError_t launch_pp_init(const float* S, int64_t m, int d, int k, int64_t first, const uint64_t* seeds,
                           int64_t* picks, float* C_out, void* ws, size_t ws_bytes, cudaStream_t st);
size_t pp_workspace_bytes(int64_t m, int d, int k);

cudaError_t launch_gen(int kind, float* X, int64_t n, int d, int64_t row0, uint64_t seed, const float* means,
                       const float* sds, int ncomp, float lo, float hi, cudaStream_t st);
cudaError_t launch_colsums(const float* X, int64_t n, int d, const unsigned int* colmax, int64_t n_total,
                           long long* sums, cudaStream_t st);
cudaError_t launch_standardize(float* X, int64_t n, int d, const long long* sums, const unsigned int* colmax,
                               int64_t n_total, double* mean_std, cudaStream_t st);

}  // namespace kmc
