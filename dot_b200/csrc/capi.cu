// extern "C" boundary of dot_b200 (declared in include/dot_b200.h): argument
// checks, dispatch to the kernel families, error state, launch accounting.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"

namespace dotb {

size_t bs_fwd_ws(int64_t B, int64_t L1, int64_t L2);
size_t bs_bwd_ws(int64_t B, int64_t L1, int64_t L2);
int bs_fwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2,
           float tau, float* out, float* row_stats, float* col_stats, void* ws, cudaStream_t st);
int bs_bwd(const void* sim, int dtype, const int32_t* lengths, int64_t B, int64_t L1, int64_t L2, float tau,
           const float* row_stats, const float* col_stats, const float* gout, void* gsim, int gdtype,
           float* gtau, void* ws, cudaStream_t st);

// ---------------------------------------------------------------------------
// error state
// ---------------------------------------------------------------------------
static thread_local std::string t_err;

void set_error(const std::string& msg) { t_err = msg; }
void clear_error() { t_err.clear(); }
int fail(int code, const std::string& msg) {
    set_error(msg);
    return code;
}
int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
        return fail(DOT_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
    return DOT_OK;
}

// ---------------------------------------------------------------------------
// launch accounting / event timing
// ---------------------------------------------------------------------------
namespace {
struct Prof {
    std::mutex mu;
    bool timing = false;
    int64_t launches[DOT_K_NCLASS] = {};
    struct Pair {
        int k;
        cudaEvent_t a, b;
    };
    std::vector<Pair> pairs;
    std::vector<cudaEvent_t> pool;
    cudaEvent_t pending[DOT_K_NCLASS] = {};
};
Prof& prof() {
    static Prof p;
    return p;
}
cudaEvent_t take_event(Prof& p) {
    if (!p.pool.empty()) {
        cudaEvent_t e = p.pool.back();
        p.pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}
}  // namespace

void prof_pre(int k, cudaStream_t s, int count) {
    Prof& p = prof();
    std::lock_guard<std::mutex> g(p.mu);
    p.launches[k] += count;
    if (p.timing) {
        cudaEvent_t a = take_event(p);
        cudaEventRecord(a, s);
        p.pending[k] = a;
    }
}

void prof_post(int k, cudaStream_t s) {
    Prof& p = prof();
    std::lock_guard<std::mutex> g(p.mu);
    if (p.timing && p.pending[k] != nullptr) {
        cudaEvent_t b = take_event(p);
        cudaEventRecord(b, s);
        p.pairs.push_back({k, p.pending[k], b});
        p.pending[k] = nullptr;
    }
}

}  // namespace dotb

using namespace dotb;

namespace {

bool bad_float(float x) { return !std::isfinite(x); }

int check_dims(int64_t B, int64_t n, int64_t m) {
    if (B < 0 || n < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    return DOT_OK;
}

}  // namespace

extern "C" {

const char* dot_last_error(void) { return t_err.c_str(); }

int dot_abi_version(void) { return DOT_B200_ABI_VERSION; }

size_t dot_sinkhorn_fwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int n_iters, float tol,
                                        int want_cost) {
    if (B <= 0 || n <= 0 || m <= 0) return 0;
    size_t a = sk_stream_fwd_ws(B, n, m, n_iters, tol, want_cost != 0);
    size_t b = sk_resident_supported(n, m) ? sk_resident_fwd_ws(B, n, m, want_cost != 0) : 0;
    return a > b ? a : b;
}

int dot_sinkhorn_fwd(const float* X, float score_sign, const float* log_a, const float* log_b,
                     int64_t B, int64_t n, int64_t m, float tau, int n_iters, float tol, int out_mode,
                     float* out, float* cost, float* pot_u, float* pot_v, int32_t* status,
                     void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (out_mode != 0 && out_mode != 1) return fail(DOT_ERR_INVALID, "out_mode must be 0 or 1");
    if (cost != nullptr && out_mode != 0) return fail(DOT_ERR_INVALID, "cost requires out_mode 0");
    if (bad_float(tol) || tol < 0.0f) return fail(DOT_ERR_INVALID, "tol must be finite and >= 0");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !out || !pot_u || !pot_v || !status) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_sinkhorn_fwd_workspace_bytes(B, n, m, n_iters, tol, cost != nullptr);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    SkFwdArgs a{};
    a.X = X;
    a.sign = score_sign;
    a.tau = tau;
    a.kinv = score_sign * (1.0f / tau);
    a.B = B;
    a.n = n;
    a.m = m;
    a.n_iters = n_iters;
    a.tol = tol;
    a.out_mode = out_mode;
    a.out = out;
    a.cost = cost;
    a.u2 = pot_u;
    a.v2 = pot_v;
    a.status = status;
    // Uniform default marginals: -log(n) in fp32 (src/sinkhorn/torch_cuda.cpp:33-43).
    a.la_def = -logf(float(n));
    a.lb_def = -logf(float(m));
    a.la = log_a;
    a.lb = log_b;
    if (tol == 0.0f && sk_resident_supported(n, m)) return sk_resident_fwd(a, workspace, st);
    if (tol == 0.0f && sk_cluster_preferred(B, n, m, X)) {
        rc = sk_cluster_fwd(a, st);
        if (rc != DOT_ERR_UNSUPPORTED) return rc;
        clear_error();
    }
    return sk_stream_fwd(a, workspace, st);
}

int dot_sinkhorn_fwd_hist(const float* X, float score_sign, const float* log_a, const float* log_b, int64_t B,
                          int64_t n, int64_t m, float tau, int n_iters, float tol, float* out, float* cost,
                          float* pot_u, float* pot_v, float* u_hist, float* v_hist, int32_t* status, void* workspace,
                          size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (bad_float(tol) || tol < 0.0f) return fail(DOT_ERR_INVALID, "tol must be finite and >= 0");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !out || !pot_u || !pot_v || !status) return fail(DOT_ERR_INVALID, "null tensor pointer");
    if (n_iters > 0 && (!u_hist || !v_hist)) return fail(DOT_ERR_INVALID, "null history pointer");
    const size_t need = sk_stream_fwd_ws(B, n, m, n_iters, tol, cost != nullptr);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    SkFwdArgs a{};
    a.X = X;
    a.sign = score_sign;
    a.tau = tau;
    a.kinv = score_sign * (1.0f / tau);
    a.B = B;
    a.n = n;
    a.m = m;
    a.n_iters = n_iters;
    a.tol = tol;
    a.out_mode = 0;
    a.out = out;
    a.cost = cost;
    a.u2 = pot_u;
    a.v2 = pot_v;
    a.status = status;
    a.la_def = -logf(float(n));
    a.lb_def = -logf(float(m));
    a.la = log_a;
    a.lb = log_b;
    a.u_hist = u_hist;
    a.v_hist = v_hist;
    return sk_stream_fwd(a, workspace, static_cast<cudaStream_t>(stream));
}

size_t dot_sinkhorn_bwd_unrolled_workspace_bytes(int64_t B, int64_t n, int64_t m) {
    if (B <= 0 || n <= 0 || m <= 0) return 0;
    return sk_unrolled_bwd_ws(B, n, m);
}

int dot_sinkhorn_bwd_unrolled(const float* X, float score_sign, const float* P, const float* u_hist,
                              const float* v_hist, const float* grad_P, const float* grad_cost, int64_t B, int64_t n,
                              int64_t m, float tau, int n_iters, float* grad_X, float* grad_tau, void* workspace,
                              size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !P || !grad_X) return fail(DOT_ERR_INVALID, "null tensor pointer");
    if (n_iters > 0 && (!u_hist || !v_hist)) return fail(DOT_ERR_INVALID, "null history pointer");
    const size_t need = sk_unrolled_bwd_ws(B, n, m);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    SkBwdArgs a{};
    a.X = X;
    a.sign = score_sign;
    a.tau = tau;
    a.P = P;
    a.gP = grad_P;
    a.gcost = grad_cost;
    a.B = B;
    a.n = n;
    a.m = m;
    a.bwd_iters = n_iters;
    a.gX = grad_X;
    a.gtau = grad_tau;
    return sk_unrolled_bwd(a, u_hist, v_hist, workspace, static_cast<cudaStream_t>(stream));
}

size_t dot_sinkhorn_bwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int bwd_iters) {
    (void)bwd_iters;
    if (B <= 0 || n <= 0 || m <= 0) return 0;
    // the streaming size covers the resident path and its unaligned fallback
    size_t a = sk_stream_bwd_ws(B, n, m);
    size_t b = sk_resident_supported(n, m) ? sk_resident_bwd_ws(B, n, m) : 0;
    return a > b ? a : b;
}

int dot_sinkhorn_bwd(const float* X, float score_sign, const float* P, const float* pot_u,
                     const float* pot_v, const float* grad_P, const float* grad_cost, int64_t B,
                     int64_t n, int64_t m, float tau, int bwd_iters, float* grad_X, float* grad_tau,
                     void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (bwd_iters < 0) return fail(DOT_ERR_INVALID, "backward_iters must be >= 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !P || !grad_X) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_sinkhorn_bwd_workspace_bytes(B, n, m, bwd_iters);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    SkBwdArgs a{};
    a.X = X;
    a.sign = score_sign;
    a.tau = tau;
    a.P = P;
    a.u2 = pot_u;
    a.v2 = pot_v;
    a.gP = grad_P;
    a.gcost = grad_cost;
    a.B = B;
    a.n = n;
    a.m = m;
    a.bwd_iters = bwd_iters;
    a.gX = grad_X;
    a.gtau = grad_tau;
    if (sk_resident_supported(n, m)) return sk_resident_bwd(a, workspace, st);
    if (sk_cluster_preferred(B, n, m, P) && workspace != nullptr) {
        rc = sk_cluster_bwd(a, static_cast<int32_t*>(workspace), st);
        if (rc != DOT_ERR_UNSUPPORTED) return rc;
        clear_error();
    }
    return sk_stream_bwd(a, workspace, st);
}

size_t dot_sinkhorn_rows_colpairs_workspace_bytes(int64_t B, int64_t n, int64_t m) {
    if (B <= 0 || n <= 0 || m <= 0) return 0;
    const size_t a = sk_split_colpairs_ws(B, n, m);
    const size_t b = (m >= 8192 && m <= 65536 && (m % 32) == 0) ? sk_wide_ws(B, n, m) : 0;
    return a > b ? a : b;
}

int dot_sinkhorn_rows_colpairs(const float* X, float score_sign, const float* log_a, int64_t B, int64_t n, int64_t m,
                               int64_t n_total, float tau, const float* pot_v, float* pot_u, float* pairs,
                               int32_t* status, void* workspace, size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (n_total < n) return fail(DOT_ERR_INVALID, "n_total must be >= the shard's row count");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !pot_v || !pot_u || !pairs || !status) return fail(DOT_ERR_INVALID, "null tensor pointer");
    if ((reinterpret_cast<uintptr_t>(pairs) & 7u) != 0) return fail(DOT_ERR_INVALID, "pairs must be 8-byte aligned");
    const size_t need = dot_sinkhorn_rows_colpairs_workspace_bytes(B, n, m);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const float kinv = score_sign * (1.0f / tau);
    const float la_def = -logf(float(n_total));
    if (sk_wide_supported(B, n, m, X))
        return sk_wide_rows_pairs(X, kinv, log_a, la_def, B, n, m, pot_v, pot_u, reinterpret_cast<float2*>(pairs),
                                  status, workspace, st);
    rc = sk_split_rows(X, kinv, log_a, la_def, B, n, m, pot_v, pot_u, st);
    if (rc != DOT_OK) return rc;
    return sk_split_colpairs(X, kinv, pot_u, B, n, m, reinterpret_cast<float2*>(pairs), workspace, st);
}

int dot_sinkhorn_col_merge(const float* pairs, int parts, const float* log_b, int64_t B, int64_t m, float* pot_v,
                           void* stream) {
    clear_error();
    if (B < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    if (parts < 1) return fail(DOT_ERR_INVALID, "parts must be >= 1");
    if (B == 0 || m == 0) return DOT_OK;
    if (!pairs || !pot_v) return fail(DOT_ERR_INVALID, "null tensor pointer");
    if ((reinterpret_cast<uintptr_t>(pairs) & 7u) != 0) return fail(DOT_ERR_INVALID, "pairs must be 8-byte aligned");
    return sk_split_pair_merge(reinterpret_cast<const float2*>(pairs), parts, log_b, -logf(float(m)), B, m, pot_v,
                               static_cast<cudaStream_t>(stream));
}

size_t dot_sinkhorn_plan_workspace_bytes(int64_t B, int64_t n, int64_t m) {
    (void)m;
    if (B <= 0 || n <= 0) return 0;
    return sk_split_plan_ws(B, n);
}

int dot_sinkhorn_plan(const float* X, float score_sign, const float* pot_u, const float* pot_v, int64_t B, int64_t n,
                      int64_t m, float tau, int out_mode, float* out, float* cost, void* workspace,
                      size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, n, m);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (out_mode != 0 && out_mode != 1) return fail(DOT_ERR_INVALID, "out_mode must be 0 or 1");
    if (cost != nullptr && out_mode != 0) return fail(DOT_ERR_INVALID, "cost requires out_mode 0");
    if (B == 0 || n == 0 || m == 0) return DOT_OK;
    if (!X || !pot_u || !pot_v || !out) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = cost ? sk_split_plan_ws(B, n) : 0;
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    return sk_split_plan(X, score_sign * (1.0f / tau), pot_u, pot_v, B, n, m, out_mode, out, cost, workspace,
                         static_cast<cudaStream_t>(stream));
}

size_t dot_bidir_fwd_workspace_bytes(int64_t B, int64_t L1, int64_t L2) {
    if (B <= 0 || L1 <= 0 || L2 <= 0) return 0;
    return bs_fwd_ws(B, L1, L2);
}

int dot_bidir_fwd(const void* sim, int sim_dtype, const int32_t* lengths, int64_t B, int64_t L1,
                  int64_t L2, float tau, float* out, float* row_stats, float* col_stats, void* workspace,
                  size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, L1, L2);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (sim_dtype != DOT_F32 && sim_dtype != DOT_BF16)
        return fail(DOT_ERR_UNSUPPORTED, "sim dtype must be float32 or bfloat16");
    if (B == 0 || L1 == 0 || L2 == 0) return DOT_OK;
    if (!sim || !lengths || !out || !row_stats || !col_stats) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_bidir_fwd_workspace_bytes(B, L1, L2);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    return bs_fwd(sim, sim_dtype, lengths, B, L1, L2, tau, out, row_stats, col_stats, workspace,
                  static_cast<cudaStream_t>(stream));
}

size_t dot_bidir_bwd_workspace_bytes(int64_t B, int64_t L1, int64_t L2) {
    if (B <= 0 || L1 <= 0 || L2 <= 0) return 0;
    return bs_bwd_ws(B, L1, L2);
}

int dot_bidir_bwd(const void* sim, int sim_dtype, const int32_t* lengths, int64_t B, int64_t L1,
                  int64_t L2, float tau, const float* row_stats, const float* col_stats,
                  const float* grad_out, void* grad_sim, int grad_dtype, float* grad_tau, void* workspace,
                  size_t workspace_bytes, void* stream) {
    clear_error();
    int rc = check_dims(B, L1, L2);
    if (rc) return rc;
    if (!(tau > 0.0f) || bad_float(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (sim_dtype != DOT_F32 && sim_dtype != DOT_BF16)
        return fail(DOT_ERR_UNSUPPORTED, "sim dtype must be float32 or bfloat16");
    if (grad_dtype != DOT_F32 && grad_dtype != DOT_BF16)
        return fail(DOT_ERR_UNSUPPORTED, "grad dtype must be float32 or bfloat16");
    if (B == 0 || L1 == 0 || L2 == 0) return DOT_OK;
    if (!sim || !lengths || !row_stats || !col_stats || !grad_out || !grad_sim)
        return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_bidir_bwd_workspace_bytes(B, L1, L2);
    if (need > 0 && (workspace == nullptr || workspace_bytes < need))
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    return bs_bwd(sim, sim_dtype, lengths, B, L1, L2, tau, row_stats, col_stats, grad_out, grad_sim, grad_dtype,
                  grad_tau, workspace, static_cast<cudaStream_t>(stream));
}

int dot_prof_begin(int time_events) {
    clear_error();
    Prof& p = prof();
    std::lock_guard<std::mutex> g(p.mu);
    for (int k = 0; k < DOT_K_NCLASS; ++k) p.launches[k] = 0;
    for (auto& pr : p.pairs) {
        p.pool.push_back(pr.a);
        p.pool.push_back(pr.b);
    }
    p.pairs.clear();
    p.timing = time_events != 0;
    return DOT_OK;
}

int dot_prof_end(int64_t* launches, double* ms) {
    clear_error();
    Prof& p = prof();
    std::lock_guard<std::mutex> g(p.mu);
    double acc[DOT_K_NCLASS] = {};
    for (auto& pr : p.pairs) {
        if (cudaEventSynchronize(pr.b) != cudaSuccess) return fail(DOT_ERR_CUDA, "event synchronize failed");
        float t = 0.0f;
        cudaEventElapsedTime(&t, pr.a, pr.b);
        acc[pr.k] += t;
        p.pool.push_back(pr.a);
        p.pool.push_back(pr.b);
    }
    p.pairs.clear();
    p.timing = false;
    for (int k = 0; k < DOT_K_NCLASS; ++k) {
        if (launches) launches[k] = p.launches[k];
        if (ms) ms[k] = acc[k];
    }
    return DOT_OK;
}

}  // extern "C"
