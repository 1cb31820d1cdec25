/*
 * dot_b200 C-ABI: the drop-in boundary for dot's two operator hot paths on
 * NVIDIA B200 (sm_100a).
 *
 * Every entry point is extern "C", takes plain device pointers, int64 shapes,
 * float parameters and a cudaStream_t passed as void*, and returns an int
 * status (DOT_OK = 0, negative on error; dot_last_error() gives the text of
 * the calling thread's last error).  Kernels are enqueued on the given stream
 * and the calls return without synchronising.  No entry point allocates device
 * memory: scratch space is passed in as `workspace`, sized by the matching
 * *_workspace_bytes() query (callers allocate it, e.g. from torch's caching
 * allocator).  All tensors are dense, row-major, contiguous.
 *
 * Each function names the reference interface it replaces (paths relative to
 * the caseysm/dot project root).  The reference exposes its ops through
 * TORCH_LIBRARY schemas; this boundary carries the same arguments as raw
 * pointers, folds the cost negation (log_alpha = -C) into a sign argument,
 * and returns the dual potentials so the backward pass need not re-run the
 * forward (the reference re-runs it, src/sinkhorn/torch_cuda.cpp:842-853).
 */
#ifndef DOT_B200_H_
#define DOT_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define DOT_B200_ABI_VERSION 1

#if defined(__GNUC__)
#define DOT_API __attribute__((visibility("default")))
#else
#define DOT_API
#endif

enum dot_status {
    DOT_OK = 0,
    DOT_ERR_INVALID = -1,     /* bad argument (shape, pointer, parameter)      */
    DOT_ERR_CUDA = -2,        /* a CUDA runtime call or kernel launch failed    */
    DOT_ERR_WORKSPACE = -3,   /* workspace missing or smaller than required     */
    DOT_ERR_UNSUPPORTED = -4  /* valid request this build does not implement    */
};

enum dot_dtype { DOT_F32 = 0, DOT_BF16 = 1, DOT_F16 = 2 };

/* Text of the calling thread's last error ("" if none). */
DOT_API const char* dot_last_error(void);

/* DOT_B200_ABI_VERSION of the loaded library. */
DOT_API int dot_abi_version(void);

/* ------------------------------------------------------------------------ */
/* Sinkhorn (log-domain, dual potentials)                                    */
/* ------------------------------------------------------------------------ */

/* Bytes of workspace dot_sinkhorn_fwd needs for this problem. */
DOT_API size_t dot_sinkhorn_fwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int n_iters,
                                        float tol, int want_cost);

/*
 * Sinkhorn forward on X [B,n,m]: K = score_sign * X / tau (score_sign = -1
 * when X is a cost matrix, +1 when X holds log-scores log_alpha).  Starting
 * from u = v = 0, each iteration sets
 *     u_i = log_a_i - LSE_j(K_ij + v_j),   then   v_j = log_b_j - LSE_i(K_ij + u_i),
 * for n_iters iterations, or, when tol > 0, until the first iteration whose
 * max_i |u_i - u_i(prev)| over the whole batch is below tol.  Then
 *     out = exp(K + u_i + v_j)   (out_mode 0, exp clamped as the reference's
 *                                 safe_exp)   or   K + u_i + v_j  (out_mode 1),
 * and, if cost != NULL, cost_b = sum_ij out_ij * X_ij (out_mode 0 only).
 *
 * log_a [B,n], log_b [B,m]: natural-log marginals; NULL = uniform (-log n,
 * -log m).  pot_u [B,n], pot_v [B,m]: receive the final dual potentials u, v
 * (natural log, as the reference's log_u / log_v); pass them to
 * dot_sinkhorn_bwd.
 * status (device int32[4]): {n_iters_used, converged, -, -}, written on the
 * stream.
 *
 * Replaces: sinkhorn_dual_forward (src/sinkhorn/registry.cpp:38-45,
 * CUDA impl src/sinkhorn/torch_cuda.cpp:266-557, vanilla method :147-264),
 * sinkhorn and sinkhorn_log (registry.cpp:31,34; torch_cuda.cpp:599-715),
 * plus the Python-side cost reduction (P*C).sum (dot/sinkhorn.py:1703).
 */
DOT_API int dot_sinkhorn_fwd(const float* X, float score_sign, const float* log_a,
                     const float* log_b, int64_t B, int64_t n, int64_t m, float tau,
                     int n_iters, float tol, int out_mode, float* out, float* cost,
                     float* pot_u, float* pot_v, int32_t* status, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * dot_sinkhorn_fwd without a workspace argument: the same computation, with
 * its scratch space taken from a fixed 16 MiB array in device memory that the
 * library itself holds (a static __device__ array), so this call never
 * allocates.  It is for callers that cannot call cudaMalloc: plugins running
 * inside a host application that owns all device memory and forbids further
 * allocations, and foreign-language bindings (cgo, JNI, ctypes) that receive
 * device pointers from elsewhere but have no device allocator of their own.
 *
 * Limits and rules:
 *  * Problems whose scratch need (dot_sinkhorn_fwd_workspace_bytes) exceeds
 *    16 MiB are rejected with DOT_ERR_WORKSPACE and a message giving the need
 *    (e.g. B=256 x 512 x 512 and B=4096 x 128 x 128 fit).
 *  * The first call on a device looks up the array's device address with that
 *    device current and caches it; make that first call before any stream
 *    capture begins.  The cache is never invalidated: after cudaDeviceReset,
 *    or anything else that destroys and re-creates the device's primary
 *    context, the cached address is stale -- do not call this entry point
 *    again in that process.
 *  * All calls share the one array per device, and it keeps the last call's
 *    contents (the call clears what must start at zero itself).  Calls that
 *    overlap on the GPU -- on different streams, or from several host threads
 *    -- race on it; serialise them (one stream, or your own ordering).
 *  * Every GPU that loads the library holds the 16 MiB until process exit.
 * This entry point has no counterpart in the reference.
 */
DOT_API int dot_sinkhorn_fwd_noalloc(const float* X, float score_sign, const float* log_a,
                                     const float* log_b, int64_t B, int64_t n, int64_t m, float tau,
                                     int n_iters, float tol, int out_mode, float* out, float* cost,
                                     float* pot_u, float* pot_v, int32_t* status, void* stream);

/* Bytes of workspace dot_sinkhorn_bwd needs for this problem. */
DOT_API size_t dot_sinkhorn_bwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int bwd_iters);

/*
 * Implicit-function backward of dot_sinkhorn_fwd for the loss
 *     L = sum_b grad_cost_b * cost_b + sum_ij grad_P_ij * P_ij,
 * i.e. G = grad_P + grad_cost_b * X.  Runs bwd_iters Gauss-Seidel sweeps of
 *     lambda_i = (sum_k P_ik G_ik - sum_k P_ik mu_k) / max(sum_k P_ik, 1e-12)
 *     mu_k     = (sum_i P_ik G_ik - sum_i P_ik lambda_i) / max(sum_i P_ik, 1e-12)
 * from lambda = mu = 0, then with g = P (G - lambda_i - mu_k) / tau (the
 * gradient with respect to log_alpha = score_sign * X):
 *     grad_X   = score_sign * g + grad_cost_b * P
 *     grad_tau_b = -sum_ij g_ij * log_alpha_ij / tau          (if grad_tau)
 * P is the forward plan (out_mode 0); pot_u / pot_v are the forward's
 * potentials (may be NULL).  grad_P [B,n,m] and grad_cost [B] may be NULL
 * (zero).
 *
 * Replaces: sinkhorn_with_grads_implicit (src/sinkhorn/registry.cpp:56; CUDA
 * impl src/sinkhorn/torch_cuda.cpp:803-871, kernels.cu:965-1098,1682-1726)
 * together with the autograd terms of the Python cost (dot/sinkhorn.py:1703)
 * and the negation log_alpha = -C (dot/sinkhorn.py:1346).
 */
DOT_API int dot_sinkhorn_bwd(const float* X, float score_sign, const float* P,
                     const float* pot_u, const float* pot_v, const float* grad_P,
                     const float* grad_cost, int64_t B, int64_t n, int64_t m, float tau,
                     int bwd_iters, float* grad_X, float* grad_tau, void* workspace,
                     size_t workspace_bytes, void* stream);

/*
 * Forward for the unrolled backward: dot_sinkhorn_fwd (plan, out_mode 0)
 * that also records the potentials after every iteration, u_hist
 * [n_iters,B,n] and v_hist [n_iters,B,m].  Workspace as
 * dot_sinkhorn_fwd_workspace_bytes.  With tol > 0, iterations after the stop
 * repeat the final potentials; status[0] gives the count to differentiate.
 * Replaces: sinkhorn_dual_forward_with_intermediates_cuda, reached through
 * sinkhorn_with_grads_unrolled (src/sinkhorn/registry.cpp:52;
 * torch_cuda.cpp:717-801, kernels.cu:1445-1507).
 */
DOT_API int dot_sinkhorn_fwd_hist(const float* X, float score_sign, const float* log_a, const float* log_b,
                                  int64_t B, int64_t n, int64_t m, float tau, int n_iters, float tol, float* out,
                                  float* cost, float* pot_u, float* pot_v, float* u_hist, float* v_hist,
                                  int32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/*
 * Unrolled backward: differentiates through the first n_iters recorded
 * iterations.  Same upstream gradients and outputs as dot_sinkhorn_bwd
 * (grad_P and/or grad_cost; grad_X, grad_tau).
 * Replaces: the backward half of sinkhorn_with_grads_unrolled
 * (src/sinkhorn/registry.cpp:52; torch_cuda.cpp:785; kernels.cu:844-961,1622-1680).
 */
DOT_API size_t dot_sinkhorn_bwd_unrolled_workspace_bytes(int64_t B, int64_t n, int64_t m);
DOT_API int dot_sinkhorn_bwd_unrolled(const float* X, float score_sign, const float* P, const float* u_hist,
                                      const float* v_hist, const float* grad_P, const float* grad_cost, int64_t B,
                                      int64_t n, int64_t m, float tau, int n_iters, float* grad_X, float* grad_tau,
                                      void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Sinkhorn half-steps for problems whose rows are sharded across GPUs       */
/* ------------------------------------------------------------------------ */
/*
 * One forward iteration of dot_sinkhorn_fwd split at its only exchange point,
 * for a shard holding rows [r0, r0 + n) of each problem's n_total x m matrix.
 * Per iteration every shard runs
 *     dot_sinkhorn_rows_colpairs   u_i = log_a_i - LSE_j(K_ij + v_j) for its rows, then
 *                                  its column pairs (max_j, sum_j) of LSE_i(K_ij + u_i)
 *     gather of every shard's pairs in shard order (caller, e.g. NCCL all-gather)
 *     dot_sinkhorn_col_merge       v_j = log_b_j - LSE over the gathered pairs
 * and finally dot_sinkhorn_plan for its rows (plus a sum of the per-shard
 * costs).  Same arithmetic as the reference's row/column update kernels
 * (src/sinkhorn/kernels.cu:503-545, 629-753 -- its split-column phase1/phase2
 * merge is the same max-then-rescaled-sum combine) and materialisation
 * (kernels.cu:755-775); the reference itself has no multi-GPU path.
 *
 * dot_sinkhorn_rows_colpairs: pairs [B,m,2]; for wide rows (8192 <= m <=
 * 65536, m % 32 == 0) a single pass over the shard on thread-block clusters
 * (the matrix is read once per iteration instead of twice).  status is a
 * device int32 error word: a bounded wait inside the kernels that expires
 * ORs 0x100 into it (zero it before the first iteration, read it after the
 * last).  dot_sinkhorn_col_merge merges [parts,B,m,2] in part order and
 * writes v (log_b NULL: -log(m)); every shard computes the same v bit for bit.
 */
DOT_API size_t dot_sinkhorn_rows_colpairs_workspace_bytes(int64_t B, int64_t n, int64_t m);
DOT_API int dot_sinkhorn_rows_colpairs(const float* X, float score_sign, const float* log_a, int64_t B, int64_t n,
                                       int64_t m, int64_t n_total, float tau, const float* pot_v, float* pot_u,
                                       float* pairs, int32_t* status, void* workspace, size_t workspace_bytes,
                                       void* stream);
DOT_API int dot_sinkhorn_col_merge(const float* pairs, int parts, const float* log_b, int64_t B, int64_t m,
                                   float* pot_v, void* stream);
DOT_API size_t dot_sinkhorn_plan_workspace_bytes(int64_t B, int64_t n, int64_t m);
DOT_API int dot_sinkhorn_plan(const float* X, float score_sign, const float* pot_u, const float* pot_v, int64_t B,
                              int64_t n, int64_t m, float tau, int out_mode, float* out, float* cost,
                              void* workspace, size_t workspace_bytes, void* stream);

/*
 * The whole row-sharded forward in one call, with the exchange done by the
 * library: n_iters iterations of dot_sinkhorn_rows_colpairs on this rank's
 * rows, an NCCL all-gather of every rank's column pairs (in place, rank
 * order) and dot_sinkhorn_col_merge; then, if out != NULL, the plan rows
 * (dot_sinkhorn_plan) and, if cost != NULL, the global cost sum_ij P_ij X_ij
 * (an NCCL all-reduce of the per-rank sums).  nccl_comm is an ncclComm_t
 * whose rank order is the row order of the shards (NULL: a single shard, no
 * collective).  X [B,n,m] holds this rank's rows of each [B,n_total,m]
 * problem (n may be 0); log_a [B,n] this rank's rows of the row marginals and
 * log_b [B,m] the column marginals (NULL: uniform over n_total / m).  pot_u
 * [B,n], pot_v [B,m] receive the potentials (pot_v identical on every rank);
 * status is one device int32 word: 0, or 0x100 if a bounded wait expired.
 * Every rank of the communicator must make the same call (same B, m, n_total,
 * tau, n_iters, and out/cost both given or both NULL).  No counterpart in the
 * reference (it has no multi-GPU path); the per-rank arithmetic is that of the
 * reference's row/column updates and materialisation (kernels.cu:503-775).
 */
DOT_API size_t dot_sinkhorn_fwd_rowshard_workspace_bytes(int64_t B, int64_t n, int64_t m, int nranks);
DOT_API int dot_sinkhorn_fwd_rowshard(const float* X, float score_sign, const float* log_a, const float* log_b,
                                      int64_t B, int64_t n, int64_t m, int64_t n_total, float tau, int n_iters,
                                      void* nccl_comm, float* out, float* cost, float* pot_u, float* pot_v,
                                      int32_t* status, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* Sinkhorn on point clouds (squared-distance cost built in the sweeps)     */
/* ------------------------------------------------------------------------ */

/*
 * C [B,n,m] from two point clouds x [B,n,d] and y [B,m,d] (fp32, row-major):
 *     s = (x_i0 - y_j0)^2, then s = fma(x_ik - y_jk, x_ik - y_jk, s) for
 *     k = 1..d-1 (each difference rounded), C_ij = s * cost_scale rounded.
 * These are exactly the entries dot_sinkhorn_points_fwd builds internally.
 * Replaces the cost construction the reference leaves to its callers
 * (torch.cdist(x, y) ** 2 before sinkhorn(); e.g. the squared-distance costs
 * of its benchmarks); no op of the reference corresponds.
 */
DOT_API int dot_sq_dist(const float* x, const float* y, int64_t B, int64_t n, int64_t m, int d,
                        float cost_scale, float* C, void* stream);

/* Bytes of workspace dot_sinkhorn_points_fwd needs (want_plan / want_cost:
 * whether plan / cost will be non-NULL). */
DOT_API size_t dot_sinkhorn_points_fwd_workspace_bytes(int64_t B, int64_t n, int64_t m, int d,
                                                       int n_iters, float tol, int want_plan,
                                                       int want_cost);

/*
 * dot_sinkhorn_fwd with X = dot_sq_dist(x, y, cost_scale) and score_sign = -1
 * (out_mode 0), without the matrix: for 1 <= d <= 4 and tol == 0 (any n, m)
 * every half-step builds the cost entries it needs from the points, so no
 * B x n x m array is read or written in the iterations; other requests
 * (d > 4, tol > 0) materialise C in the workspace and run the matrix solvers.
 * plan [B,n,m] may be NULL (potentials and cost only: the point kernels then
 * write no B x n x m array at all); cost [B] may be NULL.  log_a, log_b,
 * pot_u, pot_v and status as dot_sinkhorn_fwd.  Results agree with
 * dot_sinkhorn_fwd on the materialised matrix within rounding (the point
 * kernels form K + v with one rounding and merge the log-sum-exps in another
 * order).
 * Extension with no counterpart in the reference (its sinkhorn() takes a
 * materialised cost, dot/sinkhorn.py:1284-1714).
 */
DOT_API int dot_sinkhorn_points_fwd(const float* x, const float* y, int64_t B, int64_t n, int64_t m,
                                    int d, float cost_scale, const float* log_a, const float* log_b,
                                    float tau, int n_iters, float tol, float* plan, float* cost,
                                    float* pot_u, float* pot_v, int32_t* status, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Bytes of workspace dot_sinkhorn_points_fwd_rowshard needs on a rank holding
 * n of the rows (0 for d > 4, which it does not take). */
DOT_API size_t dot_sinkhorn_points_fwd_rowshard_workspace_bytes(int64_t B, int64_t n, int64_t m, int d,
                                                                int nranks);

/*
 * dot_sinkhorn_points_fwd for one problem batch whose rows are split over the
 * ranks of nccl_comm (NULL: one rank): this rank holds the points x [B,n,d]
 * of its n of the n_total rows (n may be 0; which rows does not matter to the
 * arithmetic) and their log_a [B,n] (or NULL: uniform -log n_total), and all
 * of y [B,m,d] and log_b [B,m].  Each iteration runs the row half-step on the shard's points,
 * the column half-step over the shard's rows -- one (max, sum) pair per
 * column -- and one in-place NCCL all-gather of the pairs, merged in rank
 * order, so every rank ends with the same v.  plan [B,n,m] (this rank's rows)
 * and cost [B] (all-reduced over the ranks) may be NULL.  1 <= d <= 4
 * (DOT_ERR_UNSUPPORTED otherwise).  status is one device int32 word, 0.
 * Collective: every rank calls it with the same B, m, d, tau, n_iters and
 * the same requests for cost.  Extension with no counterpart in the
 * reference (it has no multi-GPU path).
 */
DOT_API int dot_sinkhorn_points_fwd_rowshard(const float* x, const float* y, const float* log_a,
                                             const float* log_b, int64_t B, int64_t n, int64_t m, int d,
                                             int64_t n_total, float cost_scale, float tau, int n_iters,
                                             void* nccl_comm, float* plan, float* cost, float* pot_u,
                                             float* pot_v, int32_t* status, void* workspace,
                                             size_t workspace_bytes, void* stream);

/*
 * NCCL communicator for dot_sinkhorn_fwd_rowshard, for callers that have
 * none: rank 0 creates a 128-byte id, the caller hands it to every rank (any
 * channel), and each rank calls dot_nccl_comm_init with its CUDA device
 * current (collective: it returns once all nranks have joined).  NCCL is
 * loaded at run time (the process's copy of libnccl.so.2 if one is loaded);
 * without it these return DOT_ERR_UNSUPPORTED.
 */
DOT_API int dot_nccl_unique_id(void* id_out);
DOT_API int dot_nccl_comm_init(void** comm_out, int nranks, const void* id, int rank);
DOT_API int dot_nccl_comm_destroy(void* comm);

/* ------------------------------------------------------------------------ */
/* Bidirectional softmax                                                     */
/* ------------------------------------------------------------------------ */

DOT_API size_t dot_bidir_fwd_workspace_bytes(int64_t B, int64_t L1, int64_t L2);

/*
 * out_ij = sqrt(1e-9 + softmax_j(sim_i. / tau)_ij * softmax_i(sim_.j / tau)_ij)
 * inside each batch's window i < lengths[b,0], j < lengths[b,1] (softmaxes
 * taken over the window), and 0 outside.  sim [B,L1,L2] is DOT_F32 or
 * DOT_BF16 (read natively, computed in fp32); lengths is a device int32
 * [B,2].  row_stats [B,L1,2] and col_stats [B,L2,2] receive (max, 1/sum) of
 * the row and column softmaxes; the backward recomputes both softmaxes from
 * them instead of storing two full-size buffers.
 *
 * Replaces: bidirectional_softmax (src/bidirectional_softmax/registry.cpp:31;
 * CUDA impl torch_cuda.cpp:42-76, kernels.cu:90-242,417-448).
 */
DOT_API int dot_bidir_fwd(const void* sim, int sim_dtype, const int32_t* lengths, int64_t B,
                  int64_t L1, int64_t L2, float tau, float* out, float* row_stats,
                  float* col_stats, void* workspace, size_t workspace_bytes, void* stream);

DOT_API size_t dot_bidir_bwd_workspace_bytes(int64_t B, int64_t L1, int64_t L2);

/*
 * Backward of dot_bidir_fwd for upstream grad_out [B,L1,L2] (fp32):
 *     d = grad_out * 0.5 / out (where out > 1e-9), d_row = d * col, d_col = d * row
 *     grad_sim = (d_row - sum_j d_row*row) * row / tau + (d_col - sum_i d_col*col) * col / tau
 * inside the window (0 outside); grad_sim is written as grad_dtype (DOT_F32 or
 * DOT_BF16, rounded to nearest even).  grad_tau_b = -sum grad_sim * sim / tau
 * over the window (if grad_tau != NULL).
 *
 * Replaces: bidirectional_softmax_backward (src/bidirectional_softmax/
 * registry.cpp:34; CUDA impl torch_cuda.cpp:78-143, kernels.cu:249-411,450-501).
 */
DOT_API int dot_bidir_bwd(const void* sim, int sim_dtype, const int32_t* lengths, int64_t B,
                  int64_t L1, int64_t L2, float tau, const float* row_stats,
                  const float* col_stats, const float* grad_out, void* grad_sim,
                  int grad_dtype, float* grad_tau, void* workspace, size_t workspace_bytes,
                  void* stream);

/* ------------------------------------------------------------------------ */
/* Instrumentation (no counterpart in the reference)                         */
/* ------------------------------------------------------------------------ */

/* Kernel classes counted and (optionally) timed by the library. */
enum dot_kclass {
    DOT_K_SK_FWD_ITER = 0,   /* Sinkhorn forward iteration kernels          */
    DOT_K_SK_FWD_EPI = 1,    /* plan / cost epilogue                         */
    DOT_K_SK_BWD_ITER = 2,   /* adjoint iteration kernels                    */
    DOT_K_SK_BWD_EPI = 3,    /* adjoint setup and gradient epilogue          */
    DOT_K_SK_RESIDENT = 4,   /* on-chip resident solver kernels              */
    DOT_K_BS_FWD = 5,        /* bidirectional softmax forward                */
    DOT_K_BS_BWD = 6,        /* bidirectional softmax backward               */
    DOT_K_SK_EXCHANGE = 7,   /* row-shard column exchange: pair merges and   */
                             /* the all-gather between the shards            */
    DOT_K_NCLASS = 8
};

/* Start counting launches per class; with time_events != 0 also bracket each
 * launch with CUDA events on its stream. */
DOT_API int dot_prof_begin(int time_events);

/* Stop; per class write launch counts and (if timed) summed kernel time in
 * milliseconds (arrays of DOT_K_NCLASS entries; either may be NULL).
 * Synchronises the recorded events. */
DOT_API int dot_prof_end(int64_t* launches, double* ms);

#ifdef __cplusplus
}
#endif

#endif /* DOT_B200_H_ */
