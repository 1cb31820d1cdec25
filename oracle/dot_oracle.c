/*
 * CPU oracle for the dot hot paths -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in plain C, the reference implementation's CPU
 * algorithms for the two operator hot paths:
 *   - log-domain Sinkhorn forward (primal log-P form, compensated sums) and
 *     its implicit-function (Gauss-Seidel adjoint) backward;
 *   - bidirectional softmax forward and backward.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it, and only as a checker or a timed CPU baseline. The product path
 * (dot_b200) never calls into it; there is no CPU fallback.
 *
 * Every function cites the reference file:line it follows (paths are
 * relative to the caseysm/dot project root). Arithmetic is fp32 throughout,
 * in the same operation order as the reference, so that the oracle agrees
 * with the reference's own CPU build to the last bit or within a few ulp.
 * Build with -ffp-contract=off (no FMA contraction), as oracle/Makefile does.
 *
 * Parity pin: tests/test_oracle_golden.py checks this oracle against golden
 * vectors produced by the reference's own Python API (tests/golden/), and,
 * when oracle/_ref/libdotref.so is present, against the reference's CPU
 * kernels compiled from their sources.
 */
#include <float.h>
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* exp with the reference's clamp: 0 below -88, argument capped at +88.
 * src/sinkhorn/kernels_cpu.cpp:18-22, src/bidirectional_softmax/kernels_cpu.cpp:31-35 */
static float orc_exp88(float x) {
    if (x < -88.0f) return 0.0f;
    if (x > 88.0f) x = 88.0f;
    return expf(x);
}

/* log-sum-exp of n values spaced `stride` apart: max pass, then a
 * compensated (Kahan) sum of exp(x - max).  -FLT_MAX for an all -FLT_MAX or
 * all-underflowing input.  src/sinkhorn/kernels_cpu.cpp:24-58 */
static float orc_lse(const float *x, int64_t n, int64_t stride) {
    float hi = -FLT_MAX;
    for (int64_t k = 0; k < n; ++k) {
        float val = x[k * stride];
        if (hi < val) hi = val;
    }
    if (hi == -FLT_MAX) return -FLT_MAX;
    float acc = 0.0f, lost = 0.0f;
    for (int64_t k = 0; k < n; ++k) {
        float term = orc_exp88(x[k * stride] - hi) - lost;
        float next = acc + term;
        lost = (next - acc) - term;
        acc = next;
    }
    if (acc == 0.0f) return -FLT_MAX;
    return hi + logf(acc);
}

/* Primal Sinkhorn: X = log_alpha / tau; T times (row normalisation to log_a,
 * then column normalisation to log_b); out = exp(X) or X.
 * Default marginals are -log(n) / -log(m) in fp32.
 * src/sinkhorn/kernels_cpu.cpp:60-107 (called from torch_cpu.cpp:23-66). */
void orc_sinkhorn_forward(const float *log_alpha, float *out,
                          const float *log_a, const float *log_b,
                          int64_t B, int64_t n, int64_t m, float tau,
                          int n_iters, int return_log) {
    if (!(tau > 0.0f)) return;
    const int64_t nm = n * m;
    const float def_a = -logf((float)n);
    const float def_b = -logf((float)m);
    for (int64_t b = 0; b < B; ++b) {
        const float *src = log_alpha + b * nm;
        float *x = out + b * nm;
        for (int64_t e = 0; e < nm; ++e) x[e] = src[e] / tau;
        for (int it = 0; it < n_iters; ++it) {
            for (int64_t i = 0; i < n; ++i) {
                float *row = x + i * m;
                float shift = orc_lse(row, m, 1) -
                              (log_a ? log_a[b * n + i] : def_a);
                for (int64_t j = 0; j < m; ++j) row[j] -= shift;
            }
            for (int64_t j = 0; j < m; ++j) {
                float shift = orc_lse(x + j, n, m) -
                              (log_b ? log_b[b * m + j] : def_b);
                for (int64_t i = 0; i < n; ++i) x[i * m + j] -= shift;
            }
        }
        if (!return_log)
            for (int64_t e = 0; e < nm; ++e) x[e] = orc_exp88(x[e]);
    }
}

/* Primal Sinkhorn storing every half-step for the unrolled backward:
 * log_X [B, T+1, n, m] (X_0 = log_alpha / tau, X_{t+1} after the column
 * normalisation of iteration t) and log_Y [B, T, n, m] (after the row
 * normalisation of iteration t); P = exp(X_T).
 * src/sinkhorn/kernels_cpu.cpp:108-165 */
void orc_sinkhorn_forward_hist(const float *log_alpha, float *P, float *log_X,
                               float *log_Y, const float *log_a,
                               const float *log_b, int64_t B, int64_t n,
                               int64_t m, float tau, int n_iters) {
    if (!(tau > 0.0f)) return;
    const int64_t nm = n * m;
    const float def_a = -logf((float)n);
    const float def_b = -logf((float)m);
    for (int64_t b = 0; b < B; ++b) {
        float *Xb = log_X + b * (int64_t)(n_iters + 1) * nm;
        float *Yb = log_Y + b * (int64_t)n_iters * nm;
        for (int64_t e = 0; e < nm; ++e) Xb[e] = log_alpha[b * nm + e] / tau;
        for (int t = 0; t < n_iters; ++t) {
            float *Y = Yb + t * nm;
            float *X1 = Xb + (t + 1) * nm;
            memcpy(Y, Xb + t * nm, sizeof(float) * (size_t)nm);
            for (int64_t i = 0; i < n; ++i) {
                float *row = Y + i * m;
                float shift = orc_lse(row, m, 1) - (log_a ? log_a[b * n + i] : def_a);
                for (int64_t j = 0; j < m; ++j) row[j] -= shift;
            }
            memcpy(X1, Y, sizeof(float) * (size_t)nm);
            for (int64_t j = 0; j < m; ++j) {
                float shift = orc_lse(X1 + j, n, m) - (log_b ? log_b[b * m + j] : def_b);
                for (int64_t i = 0; i < n; ++i) X1[i * m + j] -= shift;
            }
        }
        const float *XT = Xb + (int64_t)n_iters * nm;
        for (int64_t e = 0; e < nm; ++e) P[b * nm + e] = orc_exp88(XT[e]);
    }
}

/* Unrolled backward through the stored half-steps: Gamma = grad_P * P; for
 * t = T-1 .. 0, column step Gamma_Y = Gamma - exp(X_{t+1}) * colsum(Gamma),
 * row step Gamma = Gamma_Y - exp(Y_t) * rowsum(Gamma_Y); then
 * grad = Gamma / tau, grad_tau = -sum(Gamma * log_alpha) / tau^2.
 * src/sinkhorn/kernels_cpu.cpp:169-245 */
void orc_sinkhorn_backward_unrolled(const float *log_alpha, const float *P,
                                    const float *grad_P, const float *log_X,
                                    const float *log_Y, float *grad,
                                    float *grad_tau, int64_t B, int64_t n,
                                    int64_t m, float tau, int n_iters) {
    const int64_t nm = n * m;
    float *Gm = (float *)malloc(sizeof(float) * (size_t)nm);
    float *GY = (float *)malloc(sizeof(float) * (size_t)nm);
    for (int64_t b = 0; b < B; ++b) {
        const float *Xb = log_X + b * (int64_t)(n_iters + 1) * nm;
        const float *Yb = log_Y + b * (int64_t)n_iters * nm;
        for (int64_t e = 0; e < nm; ++e) Gm[e] = grad_P[b * nm + e] * P[b * nm + e];
        for (int t = n_iters - 1; t >= 0; --t) {
            const float *X1 = Xb + (int64_t)(t + 1) * nm;
            const float *Y = Yb + (int64_t)t * nm;
            for (int64_t k = 0; k < m; ++k) {
                float s = 0.0f;
                for (int64_t i = 0; i < n; ++i) s += Gm[i * m + k];
                for (int64_t i = 0; i < n; ++i) GY[i * m + k] = Gm[i * m + k] - orc_exp88(X1[i * m + k]) * s;
            }
            for (int64_t i = 0; i < n; ++i) {
                float ti = 0.0f;
                for (int64_t k = 0; k < m; ++k) ti += GY[i * m + k];
                for (int64_t k = 0; k < m; ++k) Gm[i * m + k] = GY[i * m + k] - orc_exp88(Y[i * m + k]) * ti;
            }
        }
        float acc = 0.0f;
        for (int64_t e = 0; e < nm; ++e) {
            grad[b * nm + e] = Gm[e] / tau;
            acc += Gm[e] * log_alpha[b * nm + e];
        }
        grad_tau[b] = -acc / (tau * tau);
    }
    free(Gm);
    free(GY);
}

/* Dual-potential Sinkhorn as the reference's CUDA path runs it:
 * u_i = log_a_i - LSE_j(K_ij + v_j), then v_j = log_b_j - LSE_i(K_ij + u_i),
 * K = log_alpha / tau, u = v = 0 at start, log floor max(sum, 1e-12);
 * with tol > 0 it stops after the first iteration whose max|u - u_prev|
 * over the whole batch is below tol.  Writes u [B,n], v [B,m] and returns the
 * number of iterations run (*converged set accordingly).
 * src/sinkhorn/torch_cuda.cpp:147-264, src/sinkhorn/kernels.cu:503-545,629-671 */
int orc_sinkhorn_dual(const float *log_alpha, const float *log_a,
                      const float *log_b, int64_t B, int64_t n, int64_t m,
                      float tau, int n_iters, float tol, float *u, float *v,
                      int *converged) {
    const int64_t nm = n * m;
    const float def_a = -logf((float)n);
    const float def_b = -logf((float)m);
    float *K = (float *)malloc(sizeof(float) * (size_t)(B * nm));
    float *t = (float *)malloc(sizeof(float) * (size_t)(n > m ? n : m));
    float *u_prev = (float *)malloc(sizeof(float) * (size_t)(B * n));
    for (int64_t e = 0; e < B * nm; ++e) K[e] = log_alpha[e] * (1.0f / tau);
    memset(u, 0, sizeof(float) * (size_t)(B * n));
    memset(v, 0, sizeof(float) * (size_t)(B * m));
    int used = 0;
    *converged = 0;
    for (int it = 0; it < n_iters; ++it) {
        memcpy(u_prev, u, sizeof(float) * (size_t)(B * n));
        for (int64_t b = 0; b < B; ++b) {
            const float *Kb = K + b * nm;
            for (int64_t i = 0; i < n; ++i) {
                float hi = -FLT_MAX, s = 0.0f;
                for (int64_t j = 0; j < m; ++j) {
                    t[j] = Kb[i * m + j] + v[b * m + j];
                    if (hi < t[j]) hi = t[j];
                }
                for (int64_t j = 0; j < m; ++j) s += orc_exp88(t[j] - hi);
                u[b * n + i] = (log_a ? log_a[b * n + i] : def_a) -
                               (hi + logf(s > 1.0e-12f ? s : 1.0e-12f));
            }
            for (int64_t j = 0; j < m; ++j) {
                float hi = -FLT_MAX, s = 0.0f;
                for (int64_t i = 0; i < n; ++i) {
                    t[i] = Kb[i * m + j] + u[b * n + i];
                    if (hi < t[i]) hi = t[i];
                }
                for (int64_t i = 0; i < n; ++i) s += orc_exp88(t[i] - hi);
                v[b * m + j] = (log_b ? log_b[b * m + j] : def_b) -
                               (hi + logf(s > 1.0e-12f ? s : 1.0e-12f));
            }
        }
        used = it + 1;
        if (tol > 0.0f) {
            float delta = 0.0f;
            for (int64_t e = 0; e < B * n; ++e) {
                float d = fabsf(u[e] - u_prev[e]);
                if (d > delta) delta = d;
            }
            if (delta < tol) {
                *converged = 1;
                break;
            }
        }
    }
    free(K);
    free(t);
    free(u_prev);
    return used;
}

/* Implicit backward: Gauss-Seidel solve of the adjoint system
 *   lambda_i = (sum_k P_ik G_ik - sum_k P_ik mu_k) / max(sum_k P_ik, 1e-12)
 *   mu_k     = (sum_i P_ik G_ik - sum_i P_ik lambda_i) / max(sum_i P_ik, 1e-12)
 * for up to max_iters sweeps (stopping early when the largest change drops
 * below tol; tol = 0 never stops early, which is what the reference's CUDA
 * path does), then grad = P (G - lambda_i - mu_k) / tau and
 * grad_tau_b = -sum(grad * log_alpha) / tau.
 * src/sinkhorn/kernels_cpu.cpp:247-327 (CUDA: kernels.cu:965-1098,1682-1726). */
void orc_sinkhorn_backward_implicit(const float *log_alpha, const float *P,
                                    const float *G, float *grad,
                                    float *grad_tau, int64_t B, int64_t n,
                                    int64_t m, float tau, int max_iters,
                                    float tol) {
    const int64_t nm = n * m;
    float *lam = (float *)malloc(sizeof(float) * (size_t)n);
    float *mu = (float *)malloc(sizeof(float) * (size_t)m);
    for (int64_t b = 0; b < B; ++b) {
        const float *Pb = P + b * nm;
        const float *Gb = G + b * nm;
        float *gb = grad + b * nm;
        memset(lam, 0, sizeof(float) * (size_t)n);
        memset(mu, 0, sizeof(float) * (size_t)m);
        for (int it = 0; it < max_iters; ++it) {
            float change = 0.0f;
            for (int64_t i = 0; i < n; ++i) {
                float pg = 0.0f, pm = 0.0f, ps = 0.0f;
                for (int64_t k = 0; k < m; ++k) {
                    float p = Pb[i * m + k];
                    pg += p * Gb[i * m + k];
                    pm += p * mu[k];
                    ps += p;
                }
                float nl = (pg - pm) / (ps > 1.0e-12f ? ps : 1.0e-12f);
                float d = fabsf(nl - lam[i]);
                if (change < d) change = d;
                lam[i] = nl;
            }
            for (int64_t k = 0; k < m; ++k) {
                float pg = 0.0f, pl = 0.0f, ps = 0.0f;
                for (int64_t i = 0; i < n; ++i) {
                    float p = Pb[i * m + k];
                    pg += p * Gb[i * m + k];
                    pl += p * lam[i];
                    ps += p;
                }
                float nm_ = (pg - pl) / (ps > 1.0e-12f ? ps : 1.0e-12f);
                float d = fabsf(nm_ - mu[k]);
                if (change < d) change = d;
                mu[k] = nm_;
            }
            if (change < tol) break;
        }
        for (int64_t i = 0; i < n; ++i)
            for (int64_t k = 0; k < m; ++k) {
                float centred = Gb[i * m + k] - lam[i] - mu[k];
                gb[i * m + k] = Pb[i * m + k] * centred / tau;
            }
        if (grad_tau) {
            float acc = 0.0f;
            for (int64_t e = 0; e < nm; ++e) acc += gb[e] * log_alpha[b * nm + e];
            grad_tau[b] = -acc / tau;
        }
    }
    free(lam);
    free(mu);
}

/* Bidirectional softmax forward over each batch's valid window
 * [0,L1) x [0,L2): row softmax and column softmax of sim/T (max, clamped
 * exp, 1/sum normalisation when the sum is positive), then
 * out = sqrt(1e-9 + row * col) inside the window and 0 outside.
 * row_sm / col_sm may be NULL (scratch is then allocated here).
 * src/bidirectional_softmax/kernels_cpu.cpp:41-143 */
void orc_bidir_forward(const float *sim, float *out, float *row_sm,
                       float *col_sm, const int32_t *lengths, int64_t B,
                       int64_t L1max, int64_t L2max, float T) {
    const int64_t ms = L1max * L2max;
    const float invT = 1.0f / T;
    float *rs_own = row_sm ? NULL : (float *)malloc(sizeof(float) * (size_t)ms);
    float *cs_own = col_sm ? NULL : (float *)malloc(sizeof(float) * (size_t)ms);
    for (int64_t b = 0; b < B; ++b) {
        const float *S = sim + b * ms;
        float *O = out + b * ms;
        float *R = row_sm ? row_sm + b * ms : rs_own;
        float *Cc = col_sm ? col_sm + b * ms : cs_own;
        const int64_t L1 = lengths[2 * b], L2 = lengths[2 * b + 1];
        memset(R, 0, sizeof(float) * (size_t)ms);
        memset(Cc, 0, sizeof(float) * (size_t)ms);
        for (int64_t i = 0; i < L1; ++i) {
            float hi = -1e30f, s = 0.0f;
            for (int64_t j = 0; j < L2; ++j) {
                float val = S[i * L2max + j] * invT;
                if (val > hi) hi = val;
            }
            for (int64_t j = 0; j < L2; ++j) {
                float e = orc_exp88(S[i * L2max + j] * invT - hi);
                R[i * L2max + j] = e;
                s += e;
            }
            if (s > 0.0f) {
                float inv = 1.0f / s;
                for (int64_t j = 0; j < L2; ++j) R[i * L2max + j] *= inv;
            }
        }
        for (int64_t j = 0; j < L2; ++j) {
            float hi = -1e30f, s = 0.0f;
            for (int64_t i = 0; i < L1; ++i) {
                float val = S[i * L2max + j] * invT;
                if (val > hi) hi = val;
            }
            for (int64_t i = 0; i < L1; ++i) {
                float e = orc_exp88(S[i * L2max + j] * invT - hi);
                Cc[i * L2max + j] = e;
                s += e;
            }
            if (s > 0.0f) {
                float inv = 1.0f / s;
                for (int64_t i = 0; i < L1; ++i) Cc[i * L2max + j] *= inv;
            }
        }
        for (int64_t i = 0; i < L1max; ++i)
            for (int64_t j = 0; j < L2max; ++j) {
                int64_t e = i * L2max + j;
                O[e] = (i < L1 && j < L2) ? sqrtf(1e-9f + R[e] * Cc[e]) : 0.0f;
            }
    }
    free(rs_own);
    free(cs_own);
}

/* Bidirectional softmax backward:
 *   d = g * 0.5 / out where out > 1e-9 (else 0), d_row = d * col, d_col = d * row,
 *   grad += (d_row - sum_j d_row*row) * row / T      (row softmax)
 *   grad += (d_col - sum_i d_col*col) * col / T      (column softmax)
 *   grad_T_b = -sum grad * sim / T over the window.
 * src/bidirectional_softmax/kernels_cpu.cpp:149-232 */
void orc_bidir_backward(const float *sim, const float *out, const float *g,
                        const float *row_sm, const float *col_sm, float *grad,
                        float *grad_T, const int32_t *lengths, int64_t B,
                        int64_t L1max, int64_t L2max, float T) {
    const int64_t ms = L1max * L2max;
    const float invT = 1.0f / T;
    float *dp = (float *)malloc(sizeof(float) * (size_t)ms);
    float *dr = (float *)malloc(sizeof(float) * (size_t)ms);
    float *dc = (float *)malloc(sizeof(float) * (size_t)ms);
    for (int64_t b = 0; b < B; ++b) {
        const float *S = sim + b * ms, *O = out + b * ms, *Gr = g + b * ms;
        const float *R = row_sm + b * ms, *Cc = col_sm + b * ms;
        float *D = grad + b * ms;
        const int64_t L1 = lengths[2 * b], L2 = lengths[2 * b + 1];
        memset(D, 0, sizeof(float) * (size_t)ms);
        memset(dp, 0, sizeof(float) * (size_t)ms);
        memset(dr, 0, sizeof(float) * (size_t)ms);
        memset(dc, 0, sizeof(float) * (size_t)ms);
        for (int64_t i = 0; i < L1; ++i)
            for (int64_t j = 0; j < L2; ++j) {
                int64_t e = i * L2max + j;
                if (O[e] > 1e-9f) dp[e] = Gr[e] * 0.5f / O[e];
            }
        for (int64_t i = 0; i < L1; ++i)
            for (int64_t j = 0; j < L2; ++j) {
                int64_t e = i * L2max + j;
                dr[e] = dp[e] * Cc[e];
                dc[e] = dp[e] * R[e];
            }
        for (int64_t i = 0; i < L1; ++i) {
            float acc = 0.0f;
            for (int64_t j = 0; j < L2; ++j) acc += dr[i * L2max + j] * R[i * L2max + j];
            for (int64_t j = 0; j < L2; ++j) {
                int64_t e = i * L2max + j;
                D[e] += (dr[e] - acc) * R[e] * invT;
            }
        }
        for (int64_t j = 0; j < L2; ++j) {
            float acc = 0.0f;
            for (int64_t i = 0; i < L1; ++i) acc += dc[i * L2max + j] * Cc[i * L2max + j];
            for (int64_t i = 0; i < L1; ++i) {
                int64_t e = i * L2max + j;
                D[e] += (dc[e] - acc) * Cc[e] * invT;
            }
        }
        if (grad_T) {
            float acc = 0.0f;
            for (int64_t i = 0; i < L1; ++i)
                for (int64_t j = 0; j < L2; ++j)
                    acc -= D[i * L2max + j] * S[i * L2max + j] * invT;
            grad_T[b] = acc;
        }
    }
    free(dp);
    free(dr);
    free(dc);
}

/*
 * Squared-distance cost of two point clouds, for the point-cloud solver
 * (dot_sinkhorn_points_fwd), which has no counterpart in the reference: its
 * callers build such costs with torch.cdist(x, y) ** 2 and pass the matrix to
 * sinkhorn() (dot/sinkhorn.py:1284).  x [B,n,d], y [B,m,d], C [B,n,m]:
 *     s = (x_0 - y_0)^2,  s = fmaf(x_k - y_k, x_k - y_k, s) for k >= 1,
 *     C = s * scale,
 * every operation rounded once to fp32 (C99 fmaf is the correctly rounded
 * fused multiply-add), the operation sequence the GPU kernels perform.
 */
void orc_sq_dist(const float *x, const float *y, float *C, int64_t B, int64_t n,
                 int64_t m, int d, float scale) {
    for (int64_t b = 0; b < B; ++b)
        for (int64_t i = 0; i < n; ++i) {
            const float *xi = x + (b * n + i) * d;
            float *ci = C + (b * n + i) * m;
            for (int64_t j = 0; j < m; ++j) {
                const float *yj = y + (b * m + j) * d;
                float t = xi[0] - yj[0];
                float s = t * t;
                for (int k = 1; k < d; ++k) {
                    t = xi[k] - yj[k];
                    s = fmaf(t, t, s);
                }
                ci[j] = s * scale;
            }
        }
}
