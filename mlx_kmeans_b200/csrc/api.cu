// api.cu -- the C ABI of libkmc.so (declared in include/kmc.h).  Argument checks, workspace carve-up,
// dispatch to the kernels, and the error reporting: every entry point returns a status and records a
// message for kmc_last_error(); nothing is thrown across the ABI.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include <cuda.h>

#include "../../include/kmc.h"
#include "kmc_internal.h"

namespace kmc {

namespace {
thread_local std::string g_err;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_err = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char* where) {
    return fail(KMC_ERR_CUDA, "%s: %s", where, cudaGetErrorString(e));
}

size_t a256(size_t v) { return (v + 255) & ~size_t(255); }

int check_shape(int64_t n, int d, int k) {
    if (n < 0) return fail(KMC_ERR_INVALID, "n must be >= 0, got %lld", (long long)n);
    if (d < 1) return fail(KMC_ERR_INVALID, "dims must be >= 1, got %d", d);
    if (d > KMC_MAX_DIMS) return fail(KMC_ERR_UNSUPPORTED, "dims %d above the supported maximum %d", d, KMC_MAX_DIMS);
    if (k < 1) return fail(KMC_ERR_INVALID, "k must be >= 1, got %d", k);
    return KMC_OK;
}
}  // namespace

int num_sms() {
    static thread_local int dev = -1, sms = 0;
    int cur = 0;
    cudaGetDevice(&cur);
    if (cur != dev || sms == 0) {
        dev = cur;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cur) != cudaSuccess || sms <= 0) sms = 148;
    }
    return sms;
}

Workspace carve(void* base, int d, int k) {
    Workspace w;
    char* p = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) { char* q = p ? p + off : nullptr; off += a256(bytes); return q; };
    w.prep = reinterpret_cast<Prep*>(take(sizeof(Prep)));
    w.counters = reinterpret_cast<long long*>(take(sizeof(long long) * 8));
    w.scale_x = reinterpret_cast<double*>(take(sizeof(double) * d));
    w.hc = reinterpret_cast<float*>(take(sizeof(float) * k));
    w.reloc = reinterpret_cast<int*>(take(sizeof(int) * k));
    w.empty = reinterpret_cast<long long*>(take(sizeof(long long) * k));
    w.bytes = off;
    return w;
}

FarWorkspace carve_far(void* base, int64_t cand_rows) {
    FarWorkspace w;
    char* p = static_cast<char*>(base);
    size_t off = 0;
    auto take = [&](size_t bytes) { char* q = p ? p + off : nullptr; off += a256(bytes); return q; };
    w.rs = reinterpret_cast<unsigned long long*>(take(sizeof(unsigned long long) * 8));
    w.hist = reinterpret_cast<unsigned int*>(take(sizeof(unsigned int) * 256));
    w.keys = reinterpret_cast<unsigned long long*>(take(sizeof(unsigned long long) * (cand_rows > 0 ? cand_rows : 1)));
    w.bytes = off;
    return w;
}

BoundsState carve_bounds(void* base, int64_t n, int d, int k) {
    BoundsState b;
    char* p = static_cast<char*>(base);
    b.meta = reinterpret_cast<double*>(p);
    b.hsep = reinterpret_cast<float*>(p + 128);
    b.cprev = reinterpret_cast<float*>(p + 256);
    b.rows = reinterpret_cast<uint32_t*>(p + 256 + a256(sizeof(float) * (size_t)k * d));
    (void)n;
    return b;
}

size_t bounds_bytes(int64_t n, int d, int k) {
    return 256 + a256(sizeof(float) * (size_t)k * d) + a256(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
}

// ---------------------------------------------------------------- kmc_pass_static
// The pass with its scratch in a file-scope device array instead of a caller buffer, for callers that
// cannot allocate device memory.  Every context that loads the library's module holds one copy
// (KMC_STATIC_SCRATCH_BYTES) until the process exits.  Host code cannot hand the array's name to a kernel (on
// the host it is only a stand-in symbol), so the address of the current context's copy is looked up with
// cudaGetSymbolAddress, with that context current, and cached per context: a __device__ variable has its own
// address in every context (a runtime that drives the GPU through a driver-API context of its own gets a copy
// separate from the primary context's).
static __device__ __align__(256) unsigned char g_static_scratch[KMC_STATIC_SCRATCH_BYTES];

namespace {
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
std::mutex g_static_mu;
struct StaticSlot {
    CUcontext ctx;
    void* addr;
};
constexpr int kStaticSlots = 64;
StaticSlot g_static_slots[kStaticSlots];
int g_static_used = 0;

// cuCtxGetCurrent through the runtime's driver entry point (the library does not link libcuda itself)
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static bool tried = false;
    if (!tried) {
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(p);
    }
    return fn;
}

// The current context's copy of g_static_scratch (the first call in a context looks it up).
int static_scratch(const char* who, void** out) {
    std::lock_guard<std::mutex> lock(g_static_mu);
    CtxGetCurrentFn get = ctx_get_current();
    if (!get) return fail(KMC_ERR_CUDA, "%s: cuCtxGetCurrent is not available from the driver", who);
    CUcontext ctx = nullptr;
    if (get(&ctx) != CUDA_SUCCESS) return fail(KMC_ERR_CUDA, "%s: cuCtxGetCurrent failed", who);
    if (ctx)
        for (int i = 0; i < g_static_used; i++)
            if (g_static_slots[i].ctx == ctx) {
                *out = g_static_slots[i].addr;
                return KMC_OK;
            }
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);   // makes the device's primary context current
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress");
    if (p == nullptr) return fail(KMC_ERR_CUDA, "%s: cudaGetSymbolAddress returned a null address", who);
    if (!ctx && (get(&ctx) != CUDA_SUCCESS || !ctx))
        return fail(KMC_ERR_CUDA, "%s: no current CUDA context after cudaGetSymbolAddress", who);
    if (g_static_used == kStaticSlots) return fail(KMC_ERR_UNSUPPORTED, "%s: more than %d CUDA contexts", who, kStaticSlots);
    g_static_slots[g_static_used++] = StaticSlot{ctx, p};
    *out = p;
    return KMC_OK;
}

// kmc_finish / kmc_totals_unpack given no workspace: the static scratch kmc_pass_static left its grid in
int static_workspace(const char* who, int d, int k, void** workspace, size_t* ws_bytes) {
    if (*workspace) return KMC_OK;
    const size_t need = carve(nullptr, d, k).bytes;
    if (need > (size_t)KMC_STATIC_SCRATCH_BYTES)
        return fail(KMC_ERR_UNSUPPORTED, "%s: d=%d, k=%d need %zu bytes of workspace, above the fixed %d bytes of "
                    "the static scratch", who, d, k, need, (int)KMC_STATIC_SCRATCH_BYTES);
    if (int s = static_scratch(who, workspace)) return s;
    *ws_bytes = (size_t)KMC_STATIC_SCRATCH_BYTES;
    return KMC_OK;
}
}  // namespace

}  // namespace kmc

using namespace kmc;

extern "C" {

int kmc_version(void) { return 1; }

const char* kmc_last_error(void) { return g_err.c_str(); }

int kmc_num_sms(void) { return num_sms(); }

int64_t kmc_row_block(int64_t n_total) { return lowd_block_rows(n_total); }

size_t kmc_workspace_bytes(int d, int k) { return carve(nullptr, d, k).bytes; }

size_t kmc_far_workspace_bytes(int64_t cand_rows) { return carve_far(nullptr, cand_rows).bytes; }

int kmc_colmax(const float* X, int64_t n, int d, uint32_t* colmax, unsigned flags, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (!colmax || (n > 0 && !X)) return fail(KMC_ERR_INVALID, "kmc_colmax: null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (!(flags & KMC_PASS_ACCUMULATE)) {
        cudaError_t e = cudaMemsetAsync(colmax, 0, sizeof(uint32_t) * d, st);
        if (e != cudaSuccess) return cuda_fail(e, "kmc_colmax");
    }
    if (n == 0) return KMC_OK;
    cudaError_t e = launch_colmax(X, n, d, colmax, st);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_colmax");
    return KMC_OK;
}

}  // extern "C"

namespace {
// kmc_pass and kmc_pass_bounded: bounds == nullptr for a plain pass
int pass_impl(const char* who, const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax,
              int64_t n_total, int64_t* totals, int32_t* labels, float* best, unsigned flags, void* workspace,
              size_t ws_bytes, void* bounds, void* stream, void* loop = nullptr) {
    if (int s = check_shape(n, d, k)) return s;
    if (!C || !colmax || !totals || !workspace || (n > 0 && !X))
        return fail(KMC_ERR_INVALID, "%s: null pointer", who);
    if (n_total < n) return fail(KMC_ERR_INVALID, "%s: n_total %lld < n %lld", who, (long long)n_total, (long long)n);
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "%s: workspace of %zu bytes, need %zu", who, ws_bytes, ws.bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    const bool fused = !(flags & KMC_PASS_GENERIC) && lowd_supports(d, k);
    const bool bounded = bounds && fused && n > 0;
    BoundsState b{};
    if (bounded) b = carve_bounds(bounds, n, d, k);
    const bool clear = !(flags & KMC_PASS_ACCUMULATE);
    e = launch_prepare(C, k, d, colmax, n_total, ws.prep, ws.scale_x, ws.hc,
                       clear ? reinterpret_cast<long long*>(totals) : nullptr, clear ? ws.counters : nullptr,
                       bounded ? b.meta : nullptr, bounded ? b.cprev : nullptr, bounded ? b.hsep : nullptr,
                       (flags & KMC_PASS_LABEL32) ? 1 : 0, st, loop);
    if (e != cudaSuccess) return cuda_fail(e, who);
    if (n == 0) return KMC_OK;
    PassArgs a;
    a.X = X;
    a.n = n;
    a.n_total = n_total;
    a.d = d;
    a.k = k;
    a.C = C;
    a.hc = ws.hc;
    a.scale_x = ws.scale_x;
    a.prep = ws.prep;
    a.totals = reinterpret_cast<long long*>(totals);
    a.labels = labels;
    a.best = best;
    a.counters = ws.counters;
    a.smem_acc = 0;
    a.ctile = 0;
    a.key_keep = 0;
    a.brows = nullptr;
    a.hsep = nullptr;
    if (bounded) {
        a.brows = b.rows;
        a.hsep = b.hsep;
        a.labels = nullptr;
        a.best = nullptr;
    }
    e = cudaErrorNotSupported;
    if (fused) e = launch_pass_lowd(a, st);
    if (e == cudaErrorNotSupported) e = launch_pass_generic(a, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    return KMC_OK;
}
}  // namespace

extern "C" {

int kmc_pass(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax, int64_t n_total,
             int64_t* totals, int32_t* labels, float* best, unsigned flags, void* workspace, size_t ws_bytes,
             void* stream) {
    return pass_impl("kmc_pass", X, n, d, C, k, colmax, n_total, totals, labels, best, flags, workspace, ws_bytes,
                     nullptr, stream);
}

size_t kmc_bounds_bytes(int64_t n, int d, int k) { return bounds_bytes(n, d, k); }

int kmc_bounds_reset(void* bounds, void* stream) {
    if (!bounds) return fail(KMC_ERR_INVALID, "kmc_bounds_reset: null pointer");
    cudaError_t e = cudaMemsetAsync(bounds, 0, 16, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_bounds_reset");
    return KMC_OK;
}

int kmc_pass_bounded(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax,
                     int64_t n_total, int64_t* totals, unsigned flags, void* bounds, size_t bounds_size,
                     void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(n, d, k)) return s;
    if (!bounds) return fail(KMC_ERR_INVALID, "kmc_pass_bounded: null bounds");
    if (bounds_size < bounds_bytes(n, d, k))
        return fail(KMC_ERR_INVALID, "kmc_pass_bounded: bounds of %zu bytes, need %zu", bounds_size,
                    bounds_bytes(n, d, k));
    return pass_impl("kmc_pass_bounded", X, n, d, C, k, colmax, n_total, totals, nullptr, nullptr, flags, workspace,
                     ws_bytes, bounds, stream);
}

static_assert(sizeof(kmc_loop) == sizeof(LoopState), "kmc_loop layout");

int kmc_loop_init(kmc_loop* loop, double tol, int64_t max_steps, int64_t steps_done, double prev_inertia,
                  int have_prev, void* stream) {
    if (!loop) return fail(KMC_ERR_INVALID, "kmc_loop_init: null pointer");
    if (!(tol >= 0.0) || max_steps < 0 || steps_done < 0)
        return fail(KMC_ERR_INVALID, "kmc_loop_init: tol %g, max_steps %lld, steps_done %lld", tol,
                    (long long)max_steps, (long long)steps_done);
    cudaError_t e = launch_loop_init(loop, tol, max_steps, steps_done, prev_inertia, have_prev,
                                     static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_loop_init");
    return KMC_OK;
}

int kmc_lloyd(const float* X, int64_t n, int d, float* C0, float* C1, int k, const uint32_t* colmax, int64_t n_total,
              int64_t* totals, unsigned flags, void* bounds, size_t bounds_size, kmc_stats* stats, kmc_loop* loop,
              int steps, void* workspace, size_t ws_bytes, void* stream) {
    const char* who = "kmc_lloyd";
    if (int s = check_shape(n, d, k)) return s;
    if (!C0 || !C1 || !colmax || !totals || !stats || !loop || !workspace || (n > 0 && !X))
        return fail(KMC_ERR_INVALID, "%s: null pointer", who);
    if (steps < 0) return fail(KMC_ERR_INVALID, "%s: steps %d", who, steps);
    if (flags & (KMC_PASS_ACCUMULATE | KMC_PASS_APPROX))
        return fail(KMC_ERR_INVALID, "%s: flags 0x%x (one slice per call; the approximate pass is kmc_pass_split's)",
                    who, flags);
    if (bounds && bounds_size < bounds_bytes(n, d, k))
        return fail(KMC_ERR_INVALID, "%s: bounds of %zu bytes, need %zu", who, bounds_size, bounds_bytes(n, d, k));
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "%s: workspace of %zu bytes, need %zu", who, ws_bytes, ws.bytes);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    for (int i = 0; i < steps; i++) {
        float* Cin = (i & 1) ? C1 : C0;
        float* Cout = (i & 1) ? C0 : C1;
        if (int s = pass_impl(who, X, n, d, Cin, k, colmax, n_total, totals, nullptr, nullptr, flags, workspace,
                              ws_bytes, bounds, stream, loop))
            return s;
        cudaError_t e = launch_finish(reinterpret_cast<long long*>(totals), k, d, nullptr, 0, 1, Cout, stats, ws, st,
                                      nullptr, 1, 0, 0, loop);
        if (e != cudaSuccess) return cuda_fail(e, who);
    }
    return KMC_OK;
}

size_t kmc_split_bytes(int64_t n, int d) { return split_rows_bytes(n, d); }

size_t kmc_csplit_bytes(int d, int k) { return split_centers_bytes(d, k); }

int kmc_split_rows(const float* X, int64_t n, int d, void* split, size_t split_bytes, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (!split || (n > 0 && !X)) return fail(KMC_ERR_INVALID, "kmc_split_rows: null pointer");
    if (split_bytes < split_rows_bytes(n, d))
        return fail(KMC_ERR_INVALID, "kmc_split_rows: split of %zu bytes, need %zu", split_bytes,
                    split_rows_bytes(n, d));
    cudaError_t e = launch_split_rows(X, n, d, carve_rows(split, n, d), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_split_rows");
    return KMC_OK;
}

}  // extern "C"

// The cascade's prefix (kmc_pass_cascade): the first m columns in the caller's order, as rows split once per slice
// (msplit) and as centers (Cm, k x m, split into mcsplit by every pass).
struct Prefix {
    const float* Cm;
    int m;
    void* msplit;
    void* mcsplit;
};

// kmc_pass_split, kmc_pass_elkan and kmc_pass_cascade: elkan == nullptr for a plain tensor-core pass; else the
// per-center bounds, built by the tensor-core pass (flags & KMC_PASS_ELKAN_BUILD) or used by the bounded pass; or,
// with pre, the cascade's state (threshold and survivor bits).
static int tc_pass_impl(const char* who, const float* X, int64_t n, int d, const float* C, int k,
                        const uint32_t* colmax, int64_t n_total, int64_t* totals, int32_t* labels, float* best,
                        unsigned flags, void* split, size_t split_bytes, void* csplit, size_t csplit_bytes,
                        void* elkan, void* workspace, size_t ws_bytes, void* stream, const Prefix* pre = nullptr) {
    if (int s = check_shape(n, d, k)) return s;
    if (!C || !colmax || !totals || !workspace || !split || !csplit || (n > 0 && !X))
        return fail(KMC_ERR_INVALID, "%s: null pointer", who);
    if (n_total < n) return fail(KMC_ERR_INVALID, "%s: n_total %lld < n %lld", who, (long long)n_total, (long long)n);
    if (n > (int64_t)UINT32_MAX)
        return fail(KMC_ERR_INVALID, "%s: %lld rows in one call, at most 2^32 - 1", who, (long long)n);
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "%s: workspace of %zu bytes, need %zu", who, ws_bytes, ws.bytes);
    if (split_bytes < split_rows_bytes(n, d))
        return fail(KMC_ERR_INVALID, "%s: split of %zu bytes, need %zu", who, split_bytes, split_rows_bytes(n, d));
    if (csplit_bytes < split_centers_bytes(d, k))
        return fail(KMC_ERR_INVALID, "%s: center split of %zu bytes, need %zu", who, csplit_bytes,
                    split_centers_bytes(d, k));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    const bool clear = !(flags & KMC_PASS_ACCUMULATE);
    const int rule = (flags & KMC_PASS_LABEL32) ? 1 : 0;
    e = launch_prepare(C, k, d, colmax, n_total, ws.prep, ws.scale_x, ws.hc,
                       clear ? reinterpret_cast<long long*>(totals) : nullptr, clear ? ws.counters : nullptr, nullptr,
                       nullptr, nullptr, rule, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    if (n == 0) return KMC_OK;
    const RowSplit rs = carve_rows(split, n, d);
    const CenterSplit cs = carve_centers(csplit, d, k);
    e = launch_split_centers(C, k, d, cs, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    TcSplit ts;
    ts.n = n;
    ts.dp = split_dp(d);
    ts.kp = split_kp(k);
    ts.k = k;
    ts.xh = rs.xh;
    ts.xl = rs.xl;
    ts.ch = cs.ch;
    ts.cl = cs.cl;
    ts.hs = cs.hs;
    ts.xn = rs.xn;
    ts.cmax = reinterpret_cast<const float*>(cs.cmax_bits);
    ts.lab = rs.lab;
    ts.cands = rs.cands;
    ts.error = cs.error;
    ts.dump = nullptr;
    ts.rule = rule;
    ts.approx = (flags & KMC_PASS_APPROX) ? 1 : 0;
    ts.lb = nullptr;
    ts.xsq_lo = rs.xsq_lo;
    if (pre) {
        // The cascade (elkan: its state, kmc_cascade_bytes).  Each row's threshold from its previous label; then
        // the tensor-core pass over the prefix columns marks, per (row, center), whether a lower bound on the
        // prefix's distance -- a lower bound on the full distance too, the other columns' terms being nonnegative
        // -- is within it (that pass's own labels go to the prefix split and are not used; a barrier timeout in it
        // sets the full pass's error flag, which sends every row to the float64 decision, the marks untrusted);
        // then the marked centers are scored in full.
        const CascadeState cst = carve_cascade(elkan, n, k);
        const RowSplit prs = carve_rows(pre->msplit, n, pre->m);
        const CenterSplit pcs = carve_centers(pre->mcsplit, pre->m, k);
        e = launch_cascade_ub(X, n, d, C, k, cst, rs.lab, ws.prep, st);
        if (e == cudaSuccess) e = launch_split_centers(pre->Cm, k, pre->m, pcs, st);
        if (e == cudaSuccess) {
            TcSplit tp = ts;
            tp.dp = split_dp(pre->m);
            tp.xh = prs.xh;
            tp.xl = prs.xl;
            tp.ch = pcs.ch;
            tp.cl = pcs.cl;
            tp.hs = pcs.hs;
            tp.xn = prs.xn;
            tp.cmax = reinterpret_cast<const float*>(pcs.cmax_bits);
            tp.lab = prs.lab;
            tp.cands = prs.cands;
            tp.error = cs.error;
            tp.approx = 0;
            tp.xsq_lo = prs.xsq_lo;
            tp.mask = cst.mask;
            tp.ub = cst.ub;
            tp.plab = rs.lab;
            tp.srows = cst.srows;
            tp.nsrows = cst.nsrows;
            e = launch_assign_tc(tp, st);
        }
        if (e == cudaSuccess) e = launch_cascade(X, n, d, C, k, cst, rs.lab, rs.cands, ws.prep, ws.counters, st);
    } else if (elkan) {
        const ElkanState es = carve_elkan(elkan, n, d, k);
        if (flags & KMC_PASS_ELKAN_BUILD) {            // a full pass that also writes every bound
            ts.lb = es.lb;
            e = launch_assign_tc(ts, st);
            if (e == cudaSuccess)
                e = cudaMemcpyAsync(es.cprev, C, sizeof(float) * (size_t)k * d, cudaMemcpyDeviceToDevice, st);
        } else {                                       // the bounded pass: drift, then the rows
            e = launch_elkan_drift(C, es, k, d, st);
            // rows in the grouped order the previous pass's scatter left in rs.perm (every pass on the split ends with it)
            if (e == cudaSuccess)
                e = launch_elkan(X, n, d, C, k, es, rs.lab, rs.cands, rs.perm, ws.prep, ws.counters, st);
        }
    } else {
        e = launch_assign_tc(ts, st);
    }
    if (e != cudaSuccess) return cuda_fail(e, who);
    PassArgs a;
    a.X = X;
    a.n = n;
    a.n_total = n_total;
    a.d = d;
    a.k = k;
    a.C = C;
    a.hc = ws.hc;
    a.scale_x = ws.scale_x;
    a.prep = ws.prep;
    a.totals = reinterpret_cast<long long*>(totals);
    a.labels = labels;
    a.best = best;
    a.counters = ws.counters;
    a.smem_acc = 0;
    a.ctile = 0;
    a.key_keep = 0;
    a.brows = nullptr;
    a.hsep = nullptr;
    e = launch_accum_split(a, rs, cs, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    return KMC_OK;
}

extern "C" {

int kmc_pass_split(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax,
                   int64_t n_total, int64_t* totals, int32_t* labels, float* best, unsigned flags, void* split,
                   size_t split_bytes, void* csplit, size_t csplit_bytes, void* workspace, size_t ws_bytes,
                   void* stream) {
    return tc_pass_impl("kmc_pass_split", X, n, d, C, k, colmax, n_total, totals, labels, best,
                        flags & ~(unsigned)KMC_PASS_ELKAN_BUILD, split, split_bytes, csplit, csplit_bytes, nullptr,
                        workspace, ws_bytes, stream);
}

size_t kmc_elkan_bytes(int64_t n, int d, int k) { return elkan_bytes(n, d, k); }

int kmc_pass_elkan(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax, int64_t n_total,
                   int64_t* totals, int32_t* labels, float* best, unsigned flags, void* split, size_t split_bytes,
                   void* csplit, size_t csplit_bytes, void* elkan, size_t elkan_bytes_, void* workspace,
                   size_t ws_bytes, void* stream) {
    const char* who = "kmc_pass_elkan";
    if (int s = check_shape(n, d, k)) return s;
    if (!elkan) return fail(KMC_ERR_INVALID, "%s: null bounds", who);
    if (k % 8) return fail(KMC_ERR_UNSUPPORTED, "%s: k = %d, the bounds need k to be a multiple of 8", who, k);
    if (flags & KMC_PASS_APPROX) return fail(KMC_ERR_INVALID, "%s: the bounds are for the exact pass", who);
    if (elkan_bytes_ < elkan_bytes(n, d, k))
        return fail(KMC_ERR_INVALID, "%s: bounds of %zu bytes, need %zu", who, elkan_bytes_, elkan_bytes(n, d, k));
    return tc_pass_impl(who, X, n, d, C, k, colmax, n_total, totals, labels, best, flags, split, split_bytes, csplit,
                        csplit_bytes, elkan, workspace, ws_bytes, stream);
}

int kmc_pass_cascade(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax,
                     int64_t n_total, int64_t* totals, int32_t* labels, float* best, unsigned flags, void* split,
                     size_t split_bytes, void* csplit, size_t csplit_bytes, const float* Cm, int m, void* msplit,
                     size_t msplit_bytes, void* mcsplit, size_t mcsplit_bytes, void* cascade, size_t cascade_bytes_,
                     void* workspace, size_t ws_bytes, void* stream) {
    const char* who = "kmc_pass_cascade";
    if (int s = check_shape(n, d, k)) return s;
    if (!cascade || !Cm || !msplit || !mcsplit) return fail(KMC_ERR_INVALID, "%s: null pointer", who);
    if (m < 1 || m > d) return fail(KMC_ERR_INVALID, "%s: prefix of %d columns out of 1..%d", who, m, d);
    if (k % 8) return fail(KMC_ERR_UNSUPPORTED, "%s: k = %d, the bounds need k to be a multiple of 8", who, k);
    if (flags & (KMC_PASS_APPROX | KMC_PASS_ELKAN_BUILD))
        return fail(KMC_ERR_INVALID, "%s: flags 0x%x (the cascade is an exact pass that builds its own bounds)", who,
                    flags);
    if (cascade_bytes_ < cascade_bytes(n, k))
        return fail(KMC_ERR_INVALID, "%s: cascade state of %zu bytes, need %zu", who, cascade_bytes_,
                    cascade_bytes(n, k));
    if (msplit_bytes < split_rows_bytes(n, m))
        return fail(KMC_ERR_INVALID, "%s: prefix split of %zu bytes, need %zu", who, msplit_bytes,
                    split_rows_bytes(n, m));
    if (mcsplit_bytes < split_centers_bytes(m, k))
        return fail(KMC_ERR_INVALID, "%s: prefix center split of %zu bytes, need %zu", who, mcsplit_bytes,
                    split_centers_bytes(m, k));
    const Prefix pre{Cm, m, msplit, mcsplit};
    return tc_pass_impl(who, X, n, d, C, k, colmax, n_total, totals, labels, best, flags, split, split_bytes, csplit,
                        csplit_bytes, cascade, workspace, ws_bytes, stream, &pre);
}

size_t kmc_cascade_bytes(int64_t n, int k) { return cascade_bytes(n, k); }

int kmc_tc_dot(const float* C, int64_t n, int d, int k, void* split, size_t split_bytes, void* csplit,
               size_t csplit_bytes, float* out, int* error, void* stream) {
    const char* who = "kmc_tc_dot";
    if (int s = check_shape(n, d, k)) return s;
    if (!C || !split || !csplit || !out || !error) return fail(KMC_ERR_INVALID, "%s: null pointer", who);
    if (n > (int64_t)UINT32_MAX) return fail(KMC_ERR_INVALID, "%s: %lld rows in one call", who, (long long)n);
    if (split_bytes < split_rows_bytes(n, d) || csplit_bytes < split_centers_bytes(d, k))
        return fail(KMC_ERR_INVALID, "%s: split buffers too small", who);
    if (n == 0) return KMC_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const RowSplit rs = carve_rows(split, n, d);
    const CenterSplit cs = carve_centers(csplit, d, k);
    cudaError_t e = launch_split_centers(C, k, d, cs, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    TcSplit ts;
    ts.n = n;
    ts.dp = split_dp(d);
    ts.kp = split_kp(k);
    ts.k = k;
    ts.xh = rs.xh;
    ts.xl = rs.xl;
    ts.ch = cs.ch;
    ts.cl = cs.cl;
    ts.hs = cs.hs;
    ts.xn = rs.xn;
    ts.cmax = reinterpret_cast<const float*>(cs.cmax_bits);
    ts.lab = rs.lab;
    ts.cands = rs.cands;
    ts.error = cs.error;
    ts.dump = out;
    ts.rule = 0;
    ts.approx = 0;
    ts.lb = nullptr;
    ts.xsq_lo = rs.xsq_lo;
    e = launch_assign_tc(ts, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(error, cs.error, sizeof(int), cudaMemcpyDeviceToDevice, st);
    if (e != cudaSuccess) return cuda_fail(e, who);
    return KMC_OK;
}

size_t kmc_exchange_bytes(int k, int d) { return exchange_bytes(k, d); }

int kmc_exchange_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle) return fail(KMC_ERR_INVALID, "kmc_exchange_alloc: null pointer");
    if (bytes < (size_t)kExchangeHeader) return fail(KMC_ERR_INVALID, "kmc_exchange_alloc: %zu bytes", bytes);
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_exchange_alloc: cudaMalloc");
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_fail(e, "kmc_exchange_alloc: cudaIpcGetMemHandle");
    }
    *ptr = p;
    return KMC_OK;
}

int kmc_exchange_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(KMC_ERR_INVALID, "kmc_exchange_open: null pointer");
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_exchange_open: cudaIpcOpenMemHandle");
    return KMC_OK;
}

int kmc_exchange_close(void* ptr, int own) {
    if (!ptr) return KMC_OK;
    cudaError_t e = own ? cudaFree(ptr) : cudaIpcCloseMemHandle(ptr);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_exchange_close");
    return KMC_OK;
}

int kmc_exchange_sum(int64_t* totals, int k, int d, const uint64_t* peers, int world, int rank, uint64_t step,
                     void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(0, d, k)) return s;
    if (!totals || !peers || !workspace) return fail(KMC_ERR_INVALID, "kmc_exchange_sum: null pointer");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(KMC_ERR_INVALID, "kmc_exchange_sum: rank %d of %d (at most 64 GPUs)", rank, world);
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes)
        return fail(KMC_ERR_INVALID, "kmc_exchange_sum: workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
    cudaError_t e = launch_exchange_sum(reinterpret_cast<long long*>(totals), k, d,
                                        reinterpret_cast<const unsigned long long*>(peers), world, rank, step,
                                        ws.counters, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_exchange_sum");
    return KMC_OK;
}

int kmc_exchange_finish(int64_t* totals, int k, int d, const uint64_t* peers, int world, int rank, uint64_t step,
                        float* C_new, kmc_stats* stats, void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(0, d, k)) return s;
    if (!totals || !peers || !C_new || !stats || !workspace)
        return fail(KMC_ERR_INVALID, "kmc_exchange_finish: null pointer");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(KMC_ERR_INVALID, "kmc_exchange_finish: rank %d of %d (at most 64 GPUs)", rank, world);
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes)
        return fail(KMC_ERR_INVALID, "kmc_exchange_finish: workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
    cudaError_t e = launch_finish(reinterpret_cast<long long*>(totals), k, d, nullptr, 0, 1, C_new, stats, ws,
                                  static_cast<cudaStream_t>(stream), reinterpret_cast<const unsigned long long*>(peers),
                                  world, rank, step);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_exchange_finish");
    return KMC_OK;
}

int kmc_far_rows(const float* X, int64_t n, int d, const int32_t* labels, const float* best, int64_t row0,
                 int64_t cand_rows, uint32_t* cands, void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (cand_rows < 1) return fail(KMC_ERR_INVALID, "kmc_far_rows: cand_rows must be >= 1");
    if (!cands || !workspace || (n > 0 && (!X || !labels || !best)))
        return fail(KMC_ERR_INVALID, "kmc_far_rows: null pointer");
    if (n > 0xffffffffll) return fail(KMC_ERR_UNSUPPORTED, "kmc_far_rows: more than 2^32 rows on one GPU");
    FarWorkspace ws = carve_far(workspace, cand_rows);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "kmc_far_rows: workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
    cudaError_t e = launch_far_rows(X, n, d, labels, best, row0, cand_rows, cands, ws, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_far_rows");
    return KMC_OK;
}

int kmc_finish(int64_t* totals, int k, int d, const uint32_t* cands, int64_t cand_rows, int ranks, float* C_new,
               kmc_stats* stats, void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(0, d, k)) return s;
    if (!totals || !C_new || !stats) return fail(KMC_ERR_INVALID, "kmc_finish: null pointer");
    if (cands && (cand_rows < 1 || ranks < 1 || ranks > 64))
        return fail(KMC_ERR_INVALID, "kmc_finish: cand_rows %lld / ranks %d", (long long)cand_rows, ranks);
    if (int s = static_workspace("kmc_finish", d, k, &workspace, &ws_bytes)) return s;
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "kmc_finish: workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
    cudaError_t e = launch_finish(reinterpret_cast<long long*>(totals), k, d, cands, cand_rows, ranks, C_new, stats, ws,
                                  static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_finish");
    return KMC_OK;
}

int kmc_stats_read(const kmc_stats* stats_dev, kmc_stats* stats_host, void* stream) {
    if (!stats_dev || !stats_host) return fail(KMC_ERR_INVALID, "kmc_stats_read: null pointer");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(stats_host, stats_dev, sizeof(kmc_stats), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return cuda_fail(e, "kmc_stats_read");
    return KMC_OK;
}

int kmc_totals_unpack(const int64_t* totals, int k, int d, double* sums, int64_t* counts, double* inertia,
                      void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(0, d, k)) return s;
    if (!totals || !sums || !counts || !inertia) return fail(KMC_ERR_INVALID, "kmc_totals_unpack: null pointer");
    if (int s = static_workspace("kmc_totals_unpack", d, k, &workspace, &ws_bytes)) return s;
    Workspace ws = carve(workspace, d, k);
    if (ws_bytes < ws.bytes) return fail(KMC_ERR_INVALID, "kmc_totals_unpack: workspace of %zu bytes, need %zu", ws_bytes, ws.bytes);
    cudaError_t e = launch_unpack(reinterpret_cast<const long long*>(totals), k, d, ws.scale_x, ws.prep, ws.counters, sums, counts,
                                  inertia, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_totals_unpack");
    return KMC_OK;
}

int kmc_d64(const float* X, const float* C, int d, int64_t m, double* out, void* stream) {
    if (int s = check_shape(m, d, 1)) return s;
    if (m > 0 && (!X || !C || !out)) return fail(KMC_ERR_INVALID, "kmc_d64: null pointer");
    if (m == 0) return KMC_OK;
    cudaError_t e = launch_d64(X, C, d, m, out, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_d64");
    return KMC_OK;
}

size_t kmc_pp_workspace_bytes(int64_t m, int d, int k) { return pp_workspace_bytes(m, d, k); }

int kmc_pp_init(const float* S, int64_t m, int d, int k, int64_t first, const uint64_t* seeds, int64_t* picks,
                float* C_out, void* workspace, size_t ws_bytes, void* stream) {
    if (int s = check_shape(m, d, k)) return s;
    if (m < 1) return fail(KMC_ERR_INVALID, "kmc_pp_init: empty sample");
    if (first < 0 || first >= m) return fail(KMC_ERR_INVALID, "kmc_pp_init: first row %lld outside the sample", (long long)first);
    if (!S || !picks || !C_out || !workspace || (k > 1 && !seeds)) return fail(KMC_ERR_INVALID, "kmc_pp_init: null pointer");
    if (ws_bytes < pp_workspace_bytes(m, d, k)) return fail(KMC_ERR_INVALID, "kmc_pp_init: workspace too small");
    cudaError_t e = launch_pp_init(S, m, d, k, first, seeds, picks, C_out, workspace, ws_bytes, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_pp_init");
    return KMC_OK;
}

int kmc_gen(int kind, float* X, int64_t n, int d, int64_t row0, uint64_t seed, const float* means, const float* sds,
            int ncomp, float lo, float hi, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (n > 0 && !X) return fail(KMC_ERR_INVALID, "kmc_gen: null pointer");
    if (kind < 0 || kind > 2) return fail(KMC_ERR_INVALID, "kmc_gen: unknown kind %d", kind);
    if (kind > 0 && (!means || !sds || ncomp < 1)) return fail(KMC_ERR_INVALID, "kmc_gen: mixture needs means, sds, ncomp");
    cudaError_t e = launch_gen(kind, X, n, d, row0, seed, means, sds, ncomp, lo, hi, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_gen");
    return KMC_OK;
}

int kmc_colsums(const float* X, int64_t n, int d, const uint32_t* colmax, int64_t n_total, int64_t* sums, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (!colmax || !sums || (n > 0 && !X)) return fail(KMC_ERR_INVALID, "kmc_colsums: null pointer");
    cudaError_t e = launch_colsums(X, n, d, colmax, n_total, reinterpret_cast<long long*>(sums), static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_colsums");
    return KMC_OK;
}

int kmc_standardize(float* X, int64_t n, int d, const int64_t* sums, const uint32_t* colmax, int64_t n_total,
                    double* mean_std, void* stream) {
    if (int s = check_shape(n, d, 1)) return s;
    if (!colmax || !sums || !mean_std || (n > 0 && !X)) return fail(KMC_ERR_INVALID, "kmc_standardize: null pointer");
    if (n_total < 1) return fail(KMC_ERR_INVALID, "kmc_standardize: n_total must be >= 1");
    cudaError_t e = launch_standardize(X, n, d, reinterpret_cast<const long long*>(sums), colmax, n_total, mean_std,
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return cuda_fail(e, "kmc_standardize");
    return KMC_OK;
}


int kmc_pass_static(const float* X, int64_t n, int d, const float* C, int k, const uint32_t* colmax, int64_t n_total,
                    int64_t* totals, int32_t* labels, float* best, unsigned flags, void* stream) {
    if (int s = check_shape(n, d, k)) return s;
    const size_t need = carve(nullptr, d, k).bytes;
    if (need > (size_t)KMC_STATIC_SCRATCH_BYTES)
        return fail(KMC_ERR_UNSUPPORTED,
                    "kmc_pass_static: d=%d, k=%d need %zu bytes of scratch, above the fixed %d bytes; "
                    "use kmc_pass with a caller workspace", d, k, need, (int)KMC_STATIC_SCRATCH_BYTES);
    void* ws = nullptr;
    if (int s = static_scratch("kmc_pass_static", &ws)) return s;
    return kmc_pass(X, n, d, C, k, colmax, n_total, totals, labels, best, flags, ws, (size_t)KMC_STATIC_SCRATCH_BYTES,
                    stream);
}

}  // extern "C"
