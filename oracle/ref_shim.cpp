// C-ABI shim over the reference's own CPU kernels -- TEST INFRASTRUCTURE ONLY.
//
// oracle/Makefile compiles this file together with the reference's CPU
// sources where they lie (src/sinkhorn/kernels_cpu.cpp and
// src/bidirectional_softmax/kernels_cpu.cpp of caseysm/dot) into
// oracle/_ref/libdotref.so.  Nothing of the reference is copied into this
// repository; the shim only gives the reference's C++ entry points plain
// extern "C" names so that ctypes can call them.  It is used to pin the C
// restatement in oracle/dot_oracle.c and as the timed CPU baseline
// (bench.py --impl reference).
#include <cstdint>

#include "sinkhorn/kernels_cpu.h"
#include "bidirectional_softmax/kernels_cpu.h"

extern "C" {

// src/sinkhorn/kernels_cpu.h: sinkhorn_forward_cpu
void ref_sinkhorn_forward(const float* log_alpha, float* out, const float* log_a,
                          const float* log_b, int B, int n, int m, float tau,
                          int n_iters, int return_log) {
    dot::sinkhorn::sinkhorn_forward_cpu(log_alpha, out, log_a, log_b, B, n, m, tau,
                                        n_iters, return_log != 0);
}

// src/sinkhorn/kernels_cpu.h: sinkhorn_backward_implicit_cpu
void ref_sinkhorn_backward_implicit(const float* log_alpha, const float* P,
                                    const float* grad_P, float* grad_log_alpha,
                                    float* grad_tau, int B, int n, int m, float tau,
                                    int max_iters, float tol) {
    dot::sinkhorn::sinkhorn_backward_implicit_cpu(log_alpha, P, grad_P, nullptr, nullptr,
                                                  grad_log_alpha, grad_tau, B, n, m, tau,
                                                  max_iters, tol);
}

// src/sinkhorn/kernels_cpu.h: sinkhorn_forward_with_intermediates_cpu
void ref_sinkhorn_forward_hist(const float* log_alpha, float* P, float* log_X, float* log_Y,
                               const float* log_a, const float* log_b, int B, int n, int m,
                               float tau, int n_iters) {
    dot::sinkhorn::sinkhorn_forward_with_intermediates_cpu(log_alpha, P, log_X, log_Y, log_a, log_b,
                                                           B, n, m, tau, n_iters);
}

// src/sinkhorn/kernels_cpu.h: sinkhorn_backward_unrolled_cpu
void ref_sinkhorn_backward_unrolled(const float* log_alpha, const float* P, const float* grad_P,
                                    const float* log_X, const float* log_Y, float* grad,
                                    float* grad_tau, int B, int n, int m, float tau, int n_iters) {
    dot::sinkhorn::sinkhorn_backward_unrolled_cpu(log_alpha, P, grad_P, log_X, log_Y, nullptr, nullptr,
                                                  grad, grad_tau, B, n, m, tau, n_iters);
}

// src/bidirectional_softmax/kernels_cpu.h: bidirectional_softmax_forward_cpu
void ref_bidir_forward(const float* sim, float* out, float* row_sm, float* col_sm,
                       const int32_t* lengths, int B, int L1, int L2, float T) {
    dot::bidirectional_softmax::bidirectional_softmax_forward_cpu(
        sim, out, row_sm, col_sm, reinterpret_cast<const int*>(lengths), B, L1, L2, T);
}

// src/bidirectional_softmax/kernels_cpu.h: bidirectional_softmax_backward_cpu
void ref_bidir_backward(const float* sim, const float* out, const float* g,
                        const float* row_sm, const float* col_sm, float* grad,
                        float* grad_T, const int32_t* lengths, int B, int L1, int L2,
                        float T) {
    dot::bidirectional_softmax::bidirectional_softmax_backward_cpu(
        sim, out, g, row_sm, col_sm, grad, grad_T, reinterpret_cast<const int*>(lengths),
        B, L1, L2, T);
}

}  // extern "C"
