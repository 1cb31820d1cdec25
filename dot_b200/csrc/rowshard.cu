// Row-sharded Sinkhorn forward with the per-iteration exchange owned by the
// library: one process per GPU, each holding a contiguous block of rows of
// every problem; the column half-step's (max, sum) pairs are all-gathered
// over NCCL and merged in rank order, so every rank computes the same v.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the
// process has already loaded, e.g. PyTorch's), so the library has no link-time
// NCCL dependency and callers that never shard rows need no NCCL at all.  The
// reference has no multi-GPU path; the per-rank arithmetic is that of
// dot_sinkhorn_rows_colpairs / dot_sinkhorn_col_merge / dot_sinkhorn_plan.
#include <dlfcn.h>
#include <nccl.h>

#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"
#include "sinkhorn.h"

namespace dotb {
namespace {

struct Nccl {
    bool ok = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int*) = nullptr;
    ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
};

template <typename F>
bool sym(void* h, const char* name, F& fn) {
    fn = reinterpret_cast<F>(dlsym(h, name));
    return fn != nullptr;
}

const Nccl& nccl() {
    static Nccl n;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) h = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (h == nullptr) {
            n.why = "libnccl.so.2 could not be loaded";
            return;
        }
        n.ok = sym(h, "ncclGetUniqueId", n.get_unique_id) && sym(h, "ncclCommInitRank", n.comm_init_rank) &&
               sym(h, "ncclCommDestroy", n.comm_destroy) && sym(h, "ncclCommCount", n.comm_count) &&
               sym(h, "ncclCommUserRank", n.comm_user_rank) && sym(h, "ncclAllGather", n.all_gather) &&
               sym(h, "ncclAllReduce", n.all_reduce) && sym(h, "ncclGetErrorString", n.error_string);
        if (!n.ok) n.why = "libnccl.so.2 lacks a required entry point";
    });
    return n;
}

// Pairs of a shard that holds no rows: (max -FLT_MAX, sum 0), the identity of
// the merge.
__global__ void rs_empty_pairs_kernel(float2* pairs, int64_t count) {
    const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (i < count) pairs[i] = make_float2(kNegBig, 0.0f);
}

int nccl_fail(const Nccl& n, ncclResult_t r, const char* what) {
    return fail(DOT_ERR_CUDA, std::string(what) + ": " + (n.error_string ? n.error_string(r) : "NCCL error"));
}

struct RowshardWs {
    float2* gathered;   // [nranks][B][m] pairs, this rank's slot written in place
    char* step;         // dot_sinkhorn_rows_colpairs workspace
    char* plan;         // dot_sinkhorn_plan workspace
};

RowshardWs carve_rowshard(Carve& c, int64_t B, int64_t n, int64_t m, int nranks) {
    RowshardWs w{};
    w.gathered = c.take<float2>(size_t(nranks) * size_t(B * m));
    w.step = c.take<char>(dot_sinkhorn_rows_colpairs_workspace_bytes(B, n, m));
    w.plan = c.take<char>(dot_sinkhorn_plan_workspace_bytes(B, n, m));
    return w;
}

}  // namespace
}  // namespace dotb

using namespace dotb;

extern "C" {

int dot_nccl_unique_id(void* id_out) {
    clear_error();
    if (id_out == nullptr) return fail(DOT_ERR_INVALID, "null id pointer");
    const Nccl& n = nccl();
    if (!n.ok) return fail(DOT_ERR_UNSUPPORTED, n.why);
    ncclUniqueId id;
    const ncclResult_t r = n.get_unique_id(&id);
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof(id));
    return DOT_OK;
}

int dot_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank) {
    clear_error();
    if (comm_out == nullptr || id == nullptr) return fail(DOT_ERR_INVALID, "null pointer");
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(DOT_ERR_INVALID, "rank must be in [0, nranks)");
    const Nccl& n = nccl();
    if (!n.ok) return fail(DOT_ERR_UNSUPPORTED, n.why);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = n.comm_init_rank(&comm, nranks, uid, rank);
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommInitRank");
    *comm_out = comm;
    return DOT_OK;
}

int dot_nccl_comm_destroy(void* comm) {
    clear_error();
    if (comm == nullptr) return DOT_OK;
    const Nccl& n = nccl();
    if (!n.ok) return fail(DOT_ERR_UNSUPPORTED, n.why);
    const ncclResult_t r = n.comm_destroy(static_cast<ncclComm_t>(comm));
    if (r != ncclSuccess) return nccl_fail(n, r, "ncclCommDestroy");
    return DOT_OK;
}

size_t dot_sinkhorn_fwd_rowshard_workspace_bytes(int64_t B, int64_t n, int64_t m, int nranks) {
    if (B <= 0 || n < 0 || m <= 0 || nranks < 1) return 0;
    Carve c(nullptr);
    carve_rowshard(c, B, n > 0 ? n : 1, m, nranks);
    return c.size();
}

int dot_sinkhorn_fwd_rowshard(const float* X, float score_sign, const float* log_a, const float* log_b, int64_t B,
                              int64_t n, int64_t m, int64_t n_total, float tau, int n_iters, void* nccl_comm,
                              float* out, float* cost, float* pot_u, float* pot_v, int32_t* status, void* workspace,
                              size_t workspace_bytes, void* stream) {
    clear_error();
    if (B < 0 || n < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    if (!(tau > 0.0f) || !std::isfinite(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (score_sign != 1.0f && score_sign != -1.0f) return fail(DOT_ERR_INVALID, "score_sign must be +1 or -1");
    if (n_total < n || n_total < 1) return fail(DOT_ERR_INVALID, "n_total must be >= the shard's row count and >= 1");
    if (cost != nullptr && out == nullptr) return fail(DOT_ERR_INVALID, "cost requires the plan output");
    int nranks = 1, rank = 0;
    const Nccl* nc = nullptr;
    if (nccl_comm != nullptr) {
        nc = &nccl();
        if (!nc->ok) return fail(DOT_ERR_UNSUPPORTED, nc->why);
        ncclResult_t r = nc->comm_count(static_cast<ncclComm_t>(nccl_comm), &nranks);
        if (r == ncclSuccess) r = nc->comm_user_rank(static_cast<ncclComm_t>(nccl_comm), &rank);
        if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclCommCount/UserRank");
    }
    if (B == 0 || m == 0) return DOT_OK;
    if (!pot_u || !pot_v || !status || (n > 0 && !X)) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_sinkhorn_fwd_rowshard_workspace_bytes(B, n, m, nranks);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Carve c(workspace);
    const RowshardWs w = carve_rowshard(c, B, n > 0 ? n : 1, m, nranks);
    const size_t pair_floats = size_t(B * m) * 2;
    float* mine = reinterpret_cast<float*>(w.gathered) + size_t(rank) * pair_floats;
    const size_t step_bytes = dot_sinkhorn_rows_colpairs_workspace_bytes(B, n, m);

    cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    cudaMemsetAsync(pot_v, 0, sizeof(float) * size_t(B * m), st);
    if (n > 0) cudaMemsetAsync(pot_u, 0, sizeof(float) * size_t(B * n), st);
    // A shard without rows contributes empty pairs (max -FLT_MAX, sum 0).
    if (n == 0)
        rs_empty_pairs_kernel<<<unsigned(ceil_div(B * m, 256)), 256, 0, st>>>(reinterpret_cast<float2*>(mine),
                                                                             B * m);
    for (int it = 0; it < n_iters; ++it) {
        if (n > 0) {
            const int rc = dot_sinkhorn_rows_colpairs(X, score_sign, log_a, B, n, m, n_total, tau, pot_v, pot_u, mine,
                                                      status, w.step, step_bytes, stream);
            if (rc != DOT_OK) return rc;
        }
        if (nranks > 1) {
            // in place: this rank's pairs already sit in its slot of the gather buffer
            ProfScope ps(DOT_K_SK_EXCHANGE, st);
            const ncclResult_t r = nc->all_gather(mine, w.gathered, pair_floats, ncclFloat32,
                                                  static_cast<ncclComm_t>(nccl_comm), st);
            if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclAllGather (column pairs)");
        }
        const int rc = dot_sinkhorn_col_merge(reinterpret_cast<const float*>(w.gathered), nranks, log_b, B, m, pot_v,
                                              stream);
        if (rc != DOT_OK) return rc;
    }
    if (out != nullptr) {
        if (n > 0) {
            const int rc = dot_sinkhorn_plan(X, score_sign, pot_u, pot_v, B, n, m, tau, 0, out, cost, w.plan,
                                             dot_sinkhorn_plan_workspace_bytes(B, n, m), stream);
            if (rc != DOT_OK) return rc;
        } else if (cost != nullptr) {
            cudaMemsetAsync(cost, 0, sizeof(float) * size_t(B), st);
        }
        if (cost != nullptr && nranks > 1) {
            const ncclResult_t r =
                nc->all_reduce(cost, cost, size_t(B), ncclFloat32, ncclSum, static_cast<ncclComm_t>(nccl_comm), st);
            if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclAllReduce (cost)");
        }
    }
    return check_launch("sinkhorn row-sharded forward");
}

size_t dot_sinkhorn_points_fwd_rowshard_workspace_bytes(int64_t B, int64_t n, int64_t m, int d, int nranks) {
    if (B <= 0 || n < 0 || m <= 0 || d < 1 || d > 4 || nranks < 1) return 0;
    Carve c(nullptr);
    c.take<float2>(size_t(nranks) * size_t(B * m));
    c.take<char>(skp_shard_ws(B, n, m, d));
    return c.size();
}

int dot_sinkhorn_points_fwd_rowshard(const float* x, const float* y, const float* log_a, const float* log_b,
                                     int64_t B, int64_t n, int64_t m, int d, int64_t n_total, float cost_scale,
                                     float tau, int n_iters, void* nccl_comm, float* plan, float* cost,
                                     float* pot_u, float* pot_v, int32_t* status, void* workspace,
                                     size_t workspace_bytes, void* stream) {
    clear_error();
    if (B < 0 || n < 0 || m < 0) return fail(DOT_ERR_INVALID, "negative dimension");
    if (d < 1) return fail(DOT_ERR_INVALID, "point dimension must be >= 1");
    if (d > 4) return fail(DOT_ERR_UNSUPPORTED, "row-sharded point clouds take up to 4 coordinates");
    if (!(tau > 0.0f) || !std::isfinite(tau)) return fail(DOT_ERR_INVALID, "tau must be > 0");
    if (!std::isfinite(cost_scale)) return fail(DOT_ERR_INVALID, "cost_scale must be finite");
    if (n_iters < 0) return fail(DOT_ERR_INVALID, "n_iters must be >= 0");
    if (n_total < n || n_total < 1) return fail(DOT_ERR_INVALID, "n_total must be >= the shard's row count and >= 1");
    int nranks = 1, rank = 0;
    const Nccl* nc = nullptr;
    if (nccl_comm != nullptr) {
        nc = &nccl();
        if (!nc->ok) return fail(DOT_ERR_UNSUPPORTED, nc->why);
        ncclResult_t r = nc->comm_count(static_cast<ncclComm_t>(nccl_comm), &nranks);
        if (r == ncclSuccess) r = nc->comm_user_rank(static_cast<ncclComm_t>(nccl_comm), &rank);
        if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclCommCount/UserRank");
    }
    if (B == 0 || m == 0) return DOT_OK;
    if (!y || !pot_v || !status || (n > 0 && (!x || !pot_u))) return fail(DOT_ERR_INVALID, "null tensor pointer");
    const size_t need = dot_sinkhorn_points_fwd_rowshard_workspace_bytes(B, n, m, d, nranks);
    if (workspace == nullptr || workspace_bytes < need)
        return fail(DOT_ERR_WORKSPACE, "workspace too small: need " + std::to_string(need) + " bytes");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    Carve c(workspace);
    float2* gathered = c.take<float2>(size_t(nranks) * size_t(B * m));
    void* sws = c.take<char>(skp_shard_ws(B, n, m, d));
    float2* mine = gathered + size_t(rank) * size_t(B * m);
    const float kinv = -(1.0f / tau);
    const float la_def = -logf(float(n_total)), lb_def = -logf(float(m));   // uniform marginals of the whole problem

    cudaMemsetAsync(status, 0, sizeof(int32_t), st);
    int rc = skp_shard_begin(x, y, B, n, m, d, pot_u, pot_v, sws, st);
    for (int it = 0; it < n_iters && rc == DOT_OK; ++it) {
        rc = skp_shard_rows_pairs(x, y, log_a, la_def, B, n, m, d, cost_scale * kinv, pot_u, mine, sws, st);
        if (rc != DOT_OK) break;
        if (nranks > 1) {
            // in place: this rank's pairs already sit in its slot of the gather buffer
            ProfScope ps(DOT_K_SK_EXCHANGE, st);
            const ncclResult_t r = nc->all_gather(mine, gathered, size_t(B * m) * 2, ncclFloat32,
                                                  static_cast<ncclComm_t>(nccl_comm), st);
            if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclAllGather (column pairs)");
        }
        rc = skp_shard_col_merge(gathered, nranks, log_b, lb_def, B, n, m, d, pot_v, sws, st);
    }
    if (rc != DOT_OK) return rc;
    if (plan != nullptr || cost != nullptr) {
        rc = skp_shard_plan(x, y, B, n, m, d, cost_scale, kinv, pot_u, pot_v, plan, cost, sws, st);
        if (rc != DOT_OK) return rc;
        if (cost != nullptr && nranks > 1) {
            const ncclResult_t r =
                nc->all_reduce(cost, cost, size_t(B), ncclFloat32, ncclSum, static_cast<ncclComm_t>(nccl_comm), st);
            if (r != ncclSuccess) return nccl_fail(*nc, r, "ncclAllReduce (cost)");
        }
    }
    return check_launch("point-cloud row-sharded forward");
}

}  // extern "C"
