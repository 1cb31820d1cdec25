// Internal interface between the C-ABI layer (capi.cu) and the Sinkhorn
// kernel families (streaming: sinkhorn_stream.cu, on-chip resident:
// sinkhorn_resident.cu).
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace dotb {

struct SkFwdArgs {
    const float* X;
    float kinv;        // sign * (1/tau): K = X * kinv
    float sign;
    float tau;
    const float* la;   // natural-log marginals [B,n] / [B,m] or nullptr (uniform)
    const float* lb;
    float la_def;      // -log(n), -log(m) in fp32
    float lb_def;
    int64_t B, n, m;
    int n_iters;
    float tol;
    int out_mode;      // 0 plan, 1 log-plan
    float* out;
    float* cost;       // nullptr = not requested
    float* u2;         // [B,n] dual potentials u, v (natural log; output)
    float* v2;         // [B,m]
    int32_t* status;   // device int32[4]
    float* u_hist;     // [n_iters,B,n] u after each iteration, or nullptr
    float* v_hist;     // [n_iters,B,m]
};

struct SkBwdArgs {
    const float* X;
    float sign;
    float tau;
    const float* P;
    const float* u2;   // may be nullptr
    const float* v2;
    const float* gP;   // may be nullptr
    const float* gcost;
    int64_t B, n, m;
    int bwd_iters;
    float* gX;
    float* gtau;       // may be nullptr
};

// Fused single-pass iteration kernels (sinkhorn_fused.cu) for m <= 1024,
// m % 4 == 0, 16-byte aligned data.
// Persistent balanced schedule: the B*nblk row blocks are split into G equal
// contiguous ranges, one per CTA (G = CTAs resident at once).
struct FusedPlan {
    int nseg = 1;              // segment slots per problem in the partial buffers (= maxseg)
    int G = 1;                 // CTAs
    int64_t nblk = 1;          // row blocks per problem
    int64_t total_blocks = 1;  // B * nblk
    int maxseg = 1;            // most CTAs whose ranges touch one problem
    int stages = 2;            // bulk-copy pipeline depth
};
bool sk_fused_shape_ok(int64_t B, int64_t n, int64_t m);
bool sk_fused_supported(int64_t B, int64_t n, int64_t m, const void* data);
// fwd: the plan of the forward iterations (their full-width kernel holds
// fewer CTAs per SM than the adjoint's)
FusedPlan sk_fused_plan(int64_t B, int64_t n, int64_t m, bool fwd = false);
// first: launched without programmatic dependency (the previous stream work
// writes what the kernel reads before its dependency wait); last: plain
// copies (earlier iterations copy with L2 evict_first).
int sk_fused_fwd_iter(const SkFwdArgs& a, const FusedPlan& p, float2* part, int32_t* cnt, float* delta,
                      int iter, bool first, bool last, cudaStream_t st);
// Invariants of the adjoint system (row and column sums of P G and P) in one
// sweep over P and X; part [B, p.maxseg, m] float2, cnt [B] zero.
int sk_fused_bwd_prep(const SkBwdArgs& a, const FusedPlan& p, float2* rinv, float2* cinv, float2* part,
                      int32_t* cnt, cudaStream_t st);
int sk_fused_bwd_iter(const SkBwdArgs& a, const FusedPlan& p, const float2* rinv, const float2* cinv,
                      float* lam, float* mu, float* part, int32_t* cnt, int32_t* err, bool first, bool last,
                      cudaStream_t st);

// Fused single-pass forward iterations for mid-width rows, 1024 < m <= 8192,
// m % 4 == 0 (sinkhorn_fused.cu: the whole CTA shares every row); the plan
// and partial buffers are as for sk_fused_*.
bool sk_mid_shape_ok(int64_t B, int64_t n, int64_t m);
bool sk_mid_supported(int64_t B, int64_t n, int64_t m, const void* data);
FusedPlan sk_mid_plan(int64_t B, int64_t n, int64_t m, bool fwd);
int sk_mid_fwd_iter(const SkFwdArgs& a, const FusedPlan& p, float2* part, int32_t* cnt, float* delta, int iter,
                    bool first, bool last, cudaStream_t st);
int sk_mid_bwd_iter(const SkBwdArgs& a, const FusedPlan& p, const float2* rinv, const float2* cinv, float* lam,
                    float* mu, float* part, int32_t* cnt, int32_t* err, bool first, bool last, cudaStream_t st);

size_t sk_stream_fwd_ws(int64_t B, int64_t n, int64_t m, int n_iters, float tol, bool want_cost);
int sk_stream_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st);
size_t sk_stream_bwd_ws(int64_t B, int64_t n, int64_t m);
int sk_stream_bwd(const SkBwdArgs& a, void* ws, cudaStream_t st);

// Fused single-pass iterations for wide rows on thread-block clusters
// (sinkhorn_wide.cu): 8192 <= m <= 65536, m % 32 == 0, tol == 0.
bool sk_wide_supported(int64_t B, int64_t n, int64_t m, const void* X);
size_t sk_wide_ws(int64_t B, int64_t n, int64_t m);
int sk_wide_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st);
// Row shard: u for the shard's rows from the given v, and the shard's column
// (max, sum) pairs [B, m] over those rows with the new u, in one pass.  A
// bounded wait that expires ORs kErrBarrierTimeout (0x100) into *err.
int sk_wide_rows_pairs(const float* X, float kinv, const float* la, float la_def, int64_t B, int64_t n, int64_t m,
                       const float* v2, float* u2, float2* pairs, int32_t* err, void* ws, cudaStream_t st);

// Row shards of the point-cloud solver (sinkhorn_points.cu): this rank holds
// the points x [B,n,d] of its rows (n may be 0) and all of y [B,m,d], d <= 4.
// begin packs both clouds and zeroes the potentials; rows_pairs runs the row
// half-step (u of the shard's rows from v) and the column half-step over the
// shard's rows, leaving one (max, sum) pair per column in pairs [B,m];
// col_merge merges the gathered pairs [nranks][B][m] in rank order into v;
// plan writes the shard's plan rows (plan may be null) and cost sums over
// its rows.  All share one workspace of skp_shard_ws bytes.
size_t skp_shard_ws(int64_t B, int64_t n, int64_t m, int d);
int skp_shard_begin(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d, float* pot_u,
                    float* pot_v, void* ws, cudaStream_t st);
int skp_shard_rows_pairs(const float* x, const float* y, const float* la, float la_def, int64_t B, int64_t n,
                         int64_t m, int d, float kfold, float* pot_u, float2* pairs, void* ws, cudaStream_t st);
int skp_shard_col_merge(const float2* gathered, int nranks, const float* lb, float lb_def, int64_t B, int64_t n,
                        int64_t m, int d, float* pot_v, void* ws, cudaStream_t st);
int skp_shard_plan(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d, float cost_scale,
                   float kinv, const float* pot_u, const float* pot_v, float* plan, float* cost, void* ws,
                   cudaStream_t st);

// Unrolled backward through a recorded forward (sinkhorn_unrolled.cu):
// a.bwd_iters = the number of recorded iterations to differentiate through.
size_t sk_unrolled_bwd_ws(int64_t B, int64_t n, int64_t m);
int sk_unrolled_bwd(const SkBwdArgs& a, const float* u_hist, const float* v_hist, void* ws, cudaStream_t st);

// Split half-steps for row-sharded problems (sinkhorn_stream.cu).
int sk_split_rows(const float* X, float kinv, const float* la, float la_def, int64_t B, int64_t n, int64_t m,
                  const float* v2, float* u2, cudaStream_t st);
size_t sk_split_colpairs_ws(int64_t B, int64_t n, int64_t m);
int sk_split_colpairs(const float* X, float kinv, const float* u2, int64_t B, int64_t n, int64_t m, float2* pairs,
                      void* ws, cudaStream_t st);
int sk_split_pair_merge(const float2* pairs, int parts, const float* lb, float lb_def, int64_t B, int64_t m,
                        float* v2, cudaStream_t st);
size_t sk_split_plan_ws(int64_t B, int64_t n);
int sk_split_plan(const float* X, float kinv, const float* u2, const float* v2, int64_t B, int64_t n, int64_t m,
                  int out_mode, float* out, float* cost, void* ws, cudaStream_t st);

// On-chip resident solvers (one CTA per problem).  *_supported() tells whether
// a shape has a resident configuration; the entry points then need the same
// workspace as reported by *_ws().
bool sk_resident_supported(int64_t n, int64_t m);
size_t sk_resident_fwd_ws(int64_t B, int64_t n, int64_t m, bool want_cost);
int sk_resident_fwd(const SkFwdArgs& a, void* ws, cudaStream_t st);
size_t sk_resident_bwd_ws(int64_t B, int64_t n, int64_t m);
int sk_resident_bwd(const SkBwdArgs& a, void* ws, cudaStream_t st);

// Cluster-resident solvers (sinkhorn_cluster.cu): one thread-block cluster per
// problem, the problem's rows spread over the cluster's shared memory, all
// iterations on chip; m % 4 == 0, m <= 1024, tol == 0.  The entry points
// return DOT_ERR_UNSUPPORTED (having launched nothing) when the device cannot
// hold a cluster of the configuration; the caller then streams.  No workspace
// beyond the backward's error word.
bool sk_cluster_supported(int64_t B, int64_t n, int64_t m, const void* data);
// Problems of this shape the device solves at once on clusters (0: none fits).
int sk_cluster_capacity(int64_t n, int64_t m);
// The cluster path is taken for batches of at most kClusterWaves waves of
// clusters.  Measured on 512 x 512, 200 fwd + 200 adjoint iterations: one
// wave (B <= 8) 1.23 ms per fwd+bwd step against 3.9-4.7 ms streaming (the
// streaming kernels leave most of the GPU idle); B = 256 (19 waves) 21.6 ms
// against 20.3 ms streaming, whose per-iteration cost is amortised over the
// batch; the per-problem costs cross near B = 200.
bool sk_cluster_preferred(int64_t B, int64_t n, int64_t m, const void* data);
int sk_cluster_fwd(const SkFwdArgs& a, cudaStream_t st);
int sk_cluster_bwd(const SkBwdArgs& a, int32_t* err, cudaStream_t st);

}  // namespace dotb
