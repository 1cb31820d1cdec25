"""CPU oracle for the dot hot paths -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg (and ``bench.py --impl reference``) may import this module, and only as a
checker or as the timed CPU baseline.  The product package ``dot_b200`` never
imports it: there is no CPU fallback.

Two interchangeable backends expose the same functions:

* ``restated`` -- ``oracle/_build/liboracle.so``, the C restatement in
  ``oracle/dot_oracle.c`` of the reference's CPU algorithms;
* ``reference`` -- ``oracle/_ref/libdotref.so``, the reference's own CPU
  kernels (``src/sinkhorn/kernels_cpu.cpp``,
  ``src/bidirectional_softmax/kernels_cpu.cpp``) compiled from their sources
  by ``oracle/Makefile``.

On top of the kernels, :func:`sinkhorn_api` and :func:`bidir_api` compose the
reference's public-API behaviour for the CPU path (``dot/sinkhorn.py:1284-1714``
and ``dot/bidirectional_softmax.py:19-106``): ``log_alpha = -C``, marginal
logs, ``cost = sum(P * C)``, and the autograd chain of ``cost``/``P`` back to
``C`` and ``reg``.
"""

from __future__ import annotations

import ctypes
import math
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATHS = {
    "restated": os.path.join(_HERE, "_build", "liboracle.so"),
    "reference": os.path.join(_HERE, "_ref", "libdotref.so"),
}
_PREFIX = {"restated": "orc_", "reference": "ref_"}
_libs: dict[str, ctypes.CDLL] = {}

_fp = ctypes.POINTER(ctypes.c_float)
_ip = ctypes.POINTER(ctypes.c_int32)


def available(kind: str = "restated") -> bool:
    return os.path.exists(_LIB_PATHS[kind])


def build() -> None:
    """Compile the oracle libraries (``make -C oracle``)."""
    import subprocess

    subprocess.run(["make", "-s", "-C", _HERE], check=True)


def _lib(kind: str) -> ctypes.CDLL:
    if kind not in _libs:
        path = _LIB_PATHS[kind]
        if not os.path.exists(path):
            raise FileNotFoundError(f"oracle library missing: {path} (run make -C oracle)")
        lib = ctypes.CDLL(path)
        p = _PREFIX[kind]
        i64 = ctypes.c_int64 if kind == "restated" else ctypes.c_int
        f = getattr(lib, p + "sinkhorn_forward")
        f.argtypes = [_fp, _fp, _fp, _fp, i64, i64, i64, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        f.restype = None
        f = getattr(lib, p + "sinkhorn_backward_implicit")
        f.argtypes = [_fp, _fp, _fp, _fp, _fp, i64, i64, i64, ctypes.c_float, ctypes.c_int, ctypes.c_float]
        f.restype = None
        f = getattr(lib, p + "bidir_forward")
        f.argtypes = [_fp, _fp, _fp, _fp, _ip, i64, i64, i64, ctypes.c_float]
        f.restype = None
        f = getattr(lib, p + "bidir_backward")
        f.argtypes = [_fp, _fp, _fp, _fp, _fp, _fp, _fp, _ip, i64, i64, i64, ctypes.c_float]
        f.restype = None
        f = getattr(lib, p + "sinkhorn_forward_hist")
        f.argtypes = [_fp, _fp, _fp, _fp, _fp, _fp, i64, i64, i64, ctypes.c_float, ctypes.c_int]
        f.restype = None
        f = getattr(lib, p + "sinkhorn_backward_unrolled")
        f.argtypes = [_fp, _fp, _fp, _fp, _fp, _fp, _fp, i64, i64, i64, ctypes.c_float, ctypes.c_int]
        f.restype = None
        if kind == "restated":
            f = lib.orc_sq_dist
            f.argtypes = [_fp, _fp, _fp, i64, i64, i64, ctypes.c_int, ctypes.c_float]
            f.restype = None
            f = lib.orc_sinkhorn_dual
            f.argtypes = [_fp, _fp, _fp, i64, i64, i64, ctypes.c_float, ctypes.c_int,
                          ctypes.c_float, _fp, _fp, ctypes.POINTER(ctypes.c_int)]
            f.restype = ctypes.c_int
        _libs[kind] = lib
    return _libs[kind]


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _ptr(a: np.ndarray | None):
    if a is None:
        return None
    return a.ctypes.data_as(_fp)


# ----------------------------------------------------------------------------
# kernel-level functions (same meaning as the reference's CPU kernels)
# ----------------------------------------------------------------------------

def sinkhorn_forward(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None,
                     return_log: bool = False, kind: str = "restated") -> np.ndarray:
    """Primal Sinkhorn plan (or log-plan) of ``log_alpha`` [B,n,m].

    Reference: ``src/sinkhorn/kernels_cpu.cpp:60-107`` via ``torch_cpu.cpp:23-66``.
    """
    la = _f32(log_alpha)
    B, n, m = la.shape
    out = np.empty_like(la)
    la_a = None if log_a is None else _f32(log_a)
    la_b = None if log_b is None else _f32(log_b)
    fn = getattr(_lib(kind), _PREFIX[kind] + "sinkhorn_forward")
    fn(_ptr(la), _ptr(out), _ptr(la_a), _ptr(la_b), B, n, m, float(tau), int(n_iters), int(bool(return_log)))
    return out


def sinkhorn_backward_implicit(log_alpha, P, grad_P, tau: float, max_iters: int,
                               tol: float = 0.0, kind: str = "restated"):
    """Implicit backward: returns ``(grad_log_alpha [B,n,m], grad_tau [B])``.

    ``tol=0`` runs exactly ``max_iters`` Gauss-Seidel sweeps, as the
    reference's CUDA path does (``kernels.cu:1715-1718``); the reference's CPU
    op passes ``tol=1e-6`` (``torch_cpu.cpp:324``).
    Reference: ``src/sinkhorn/kernels_cpu.cpp:247-327``.
    """
    la, p, g = _f32(log_alpha), _f32(P), _f32(grad_P)
    B, n, m = la.shape
    grad = np.empty_like(la)
    gtau = np.empty((B,), np.float32)
    fn = getattr(_lib(kind), _PREFIX[kind] + "sinkhorn_backward_implicit")
    fn(_ptr(la), _ptr(p), _ptr(g), _ptr(grad), _ptr(gtau), B, n, m, float(tau), int(max_iters), float(tol))
    return grad, gtau


def sinkhorn_forward_hist(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None,
                          kind: str = "restated"):
    """Primal Sinkhorn keeping every half-step: returns ``(P, log_X [B,T+1,n,m],
    log_Y [B,T,n,m])``.  Reference: ``src/sinkhorn/kernels_cpu.cpp:108-165``."""
    la = _f32(log_alpha)
    B, n, m = la.shape
    T = int(n_iters)
    P = np.empty_like(la)
    X = np.empty((B, T + 1, n, m), np.float32)
    Y = np.empty((B, max(T, 1), n, m), np.float32)
    la_a = None if log_a is None else _f32(log_a)
    la_b = None if log_b is None else _f32(log_b)
    fn = getattr(_lib(kind), _PREFIX[kind] + "sinkhorn_forward_hist")
    fn(_ptr(la), _ptr(P), _ptr(X), _ptr(Y), _ptr(la_a), _ptr(la_b), B, n, m, float(tau), T)
    return P, X, Y


def sinkhorn_backward_unrolled(log_alpha, P, grad_P, log_X, log_Y, tau: float, n_iters: int,
                               kind: str = "restated"):
    """Unrolled backward: returns ``(grad_log_alpha [B,n,m], grad_tau [B])``.
    Reference: ``src/sinkhorn/kernels_cpu.cpp:169-245``."""
    la, p, g = _f32(log_alpha), _f32(P), _f32(grad_P)
    X, Y = _f32(log_X), _f32(log_Y)
    B, n, m = la.shape
    grad = np.empty_like(la)
    gtau = np.empty((B,), np.float32)
    fn = getattr(_lib(kind), _PREFIX[kind] + "sinkhorn_backward_unrolled")
    fn(_ptr(la), _ptr(p), _ptr(g), _ptr(X), _ptr(Y), _ptr(grad), _ptr(gtau), B, n, m, float(tau), int(n_iters))
    return grad, gtau


def sinkhorn_dual(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None, tol: float = 0.0):
    """Dual-potential iteration as the reference's CUDA path runs it.

    Returns ``(u [B,n], v [B,m], n_iters_used, converged)``; the plan is
    ``exp(log_alpha/tau + u_i + v_j)``.  Reference: ``src/sinkhorn/torch_cuda.cpp:147-264``.
    """
    la = _f32(log_alpha)
    B, n, m = la.shape
    u = np.empty((B, n), np.float32)
    v = np.empty((B, m), np.float32)
    conv = ctypes.c_int(0)
    la_a = None if log_a is None else _f32(log_a)
    la_b = None if log_b is None else _f32(log_b)
    used = _lib("restated").orc_sinkhorn_dual(_ptr(la), _ptr(la_a), _ptr(la_b), B, n, m, float(tau),
                                             int(n_iters), float(tol), _ptr(u), _ptr(v), ctypes.byref(conv))
    return u, v, int(used), bool(conv.value)


def sinkhorn_dual_fp64(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None) -> np.ndarray:
    """The dual-potential iteration of :func:`sinkhorn_dual` (the reference's
    CUDA path, ``src/sinkhorn/torch_cuda.cpp:147-264``, row then column update
    from ``u = v = 0``, default marginals ``-log n`` / ``-log m``) evaluated in
    float64 from the fp32 input, as a rounding-free yardstick for problems
    whose fp32 sums are long (m in the tens of thousands), where the
    reference's own two fp32 formulations already differ at the 1e-5 level.
    Returns the plan [B,n,m] (float64)."""
    K = _f32(log_alpha).astype(np.float64) / float(tau)
    B, n, m = K.shape
    la = np.full((B, n), -math.log(n)) if log_a is None else np.asarray(log_a, np.float64)
    lb = np.full((B, m), -math.log(m)) if log_b is None else np.asarray(log_b, np.float64)
    u = np.zeros((B, n))
    v = np.zeros((B, m))
    for _ in range(int(n_iters)):
        t = K + v[:, None, :]
        mx = t.max(axis=2, keepdims=True)
        u = la - (mx[..., 0] + np.log(np.exp(t - mx).sum(axis=2)))
        t = K + u[:, :, None]
        mx = t.max(axis=1, keepdims=True)
        v = lb - (mx[:, 0] + np.log(np.exp(t - mx).sum(axis=1)))
    return np.exp(K + u[:, :, None] + v[:, None, :])


def sinkhorn_implicit_fp64(log_alpha, P, G, tau: float, n_iters: int):
    """The reference's implicit backward (Gauss-Seidel adjoint of
    ``src/sinkhorn/kernels_cpu.cpp:247-327`` run for ``n_iters`` sweeps, no
    early stop, then grad = P (G - lambda - mu) / tau and grad_tau =
    -sum(grad * log_alpha) / tau) evaluated in float64, as a rounding-free
    yardstick for quantities whose fp32 sums cancel (the temperature gradient
    of a batch).  Returns (grad [B,n,m], grad_tau [B]) in float64."""
    la = np.asarray(log_alpha, np.float64)
    P = np.asarray(P, np.float64)
    G = np.asarray(G, np.float64)
    B, n, m = P.shape
    rPG, rP = (P * G).sum(2), np.maximum(P.sum(2), 1e-12)
    cPG, cP = (P * G).sum(1), np.maximum(P.sum(1), 1e-12)
    lam = np.zeros((B, n))
    mu = np.zeros((B, m))
    for _ in range(int(n_iters)):
        lam = (rPG - (P * mu[:, None, :]).sum(2)) / rP
        mu = (cPG - (P * lam[:, :, None]).sum(1)) / cP
    grad = P * (G - lam[:, :, None] - mu[:, None, :]) / float(tau)
    return grad, -(grad * la).sum((1, 2)) / float(tau)


def bidir_forward(sim, tau: float, lengths, kind: str = "restated"):
    """Returns ``(out, row_softmax, col_softmax)``, all [B,L1,L2] fp32.

    Reference: ``src/bidirectional_softmax/kernels_cpu.cpp:41-143``.
    """
    s = _f32(sim)
    B, L1, L2 = s.shape
    ln = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    out, rs, cs = np.empty_like(s), np.empty_like(s), np.empty_like(s)
    fn = getattr(_lib(kind), _PREFIX[kind] + "bidir_forward")
    fn(_ptr(s), _ptr(out), _ptr(rs), _ptr(cs), ln.ctypes.data_as(_ip), B, L1, L2, float(tau))
    return out, rs, cs


def bidir_backward(sim, out, grad_out, row_sm, col_sm, tau: float, lengths, kind: str = "restated"):
    """Returns ``(grad_sim [B,L1,L2], grad_tau [B])``.

    Reference: ``src/bidirectional_softmax/kernels_cpu.cpp:149-232``.
    """
    s, o, g, rs, cs = (_f32(x) for x in (sim, out, grad_out, row_sm, col_sm))
    B, L1, L2 = s.shape
    ln = np.ascontiguousarray(np.asarray(lengths, dtype=np.int32))
    grad = np.empty_like(s)
    gT = np.empty((B,), np.float32)
    fn = getattr(_lib(kind), _PREFIX[kind] + "bidir_backward")
    fn(_ptr(s), _ptr(o), _ptr(g), _ptr(rs), _ptr(cs), _ptr(grad), _ptr(gT), ln.ctypes.data_as(_ip),
       B, L1, L2, float(tau))
    return grad, gT


# ----------------------------------------------------------------------------
# API-level composition (what dot.sinkhorn / dot.bidirectional_softmax return
# on the reference's CPU path, including the autograd chain)
# ----------------------------------------------------------------------------

def _log_marginal(x, B: int, size: int):
    """``torch.log`` of a marginal, as ``dot/sinkhorn.py:1348-1349`` takes it
    (numpy's fp32 log can differ from ATen's by an ulp)."""
    if x is None:
        return None
    import torch

    x = np.asarray(x, dtype=np.float32)
    if x.ndim == 1:
        x = np.broadcast_to(x[None, :], (B, size))
    return torch.log(torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32))).numpy()


def sinkhorn_api(C, reg: float, n_iters: int, a=None, b=None, backward_iters: int | None = None,
                 g_cost=None, grad_P=None, bwd_tol: float = 0.0, kind: str = "restated",
                 with_grad: bool = True, backward_mode: str = "implicit"):
    """``dot.sinkhorn(C, reg, n_iters, a=a, b=b)`` on the reference's CPU path.

    Returns a dict with ``P`` [B,n,m], ``cost`` [B] and, when ``with_grad``,
    ``dC`` [B,n,m] and ``dreg`` (scalar) for the loss
    ``sum_b g_cost[b] * cost[b] + sum(grad_P * P)`` (``g_cost`` defaults to ones,
    i.e. ``cost.sum()``).

    Mirrors ``dot/sinkhorn.py``: ``log_alpha = -C`` (:1346), marginal logs
    (:1347-1350), ``_SinkhornImplicitFunction`` (:99-152) whose backward runs the
    implicit op (``torch_cpu.cpp:261-328``), and ``cost = (P*C).sum((-2,-1))``
    (:1703) whose autograd gives ``grad_P += g*C`` and ``dC += g*P``; the
    negation gives ``dC -= grad_log_alpha``.  ``bwd_tol`` is the adjoint
    early-exit threshold: the reference CPU op uses 1e-6, its CUDA op runs all
    ``backward_iters`` sweeps (``bwd_tol=0``).  ``backward_mode='unrolled'``
    follows ``_SinkhornUnrolledFunction`` (:45-96): the backward differentiates
    through the ``n_iters`` stored iterations (``torch_cpu.cpp:188-259``).
    """
    C = _f32(C)
    B, n, m = C.shape
    log_alpha = -C
    la = _log_marginal(a, B, n)
    lb = _log_marginal(b, B, m)
    P = sinkhorn_forward(log_alpha, reg, n_iters, la, lb, kind=kind)
    cost = (P.astype(np.float64) * C.astype(np.float64)).sum(axis=(1, 2)).astype(np.float32)
    out = {"P": P, "cost": cost}
    if not with_grad:
        return out
    g = np.ones((B,), np.float32) if g_cost is None else np.asarray(g_cost, np.float32).reshape(B)
    G = (g[:, None, None] * C).astype(np.float32)
    if grad_P is not None:
        G = (G + _f32(grad_P)).astype(np.float32)
    if backward_mode == "unrolled":
        _, X, Y = sinkhorn_forward_hist(log_alpha, reg, n_iters, la, lb, kind=kind)
        gla, gtau = sinkhorn_backward_unrolled(log_alpha, P, G, X, Y, reg, n_iters, kind=kind)
    else:
        bi = n_iters if backward_iters is None else backward_iters
        gla, gtau = sinkhorn_backward_implicit(log_alpha, P, G, reg, bi, tol=bwd_tol, kind=kind)
    dC = (g[:, None, None] * P - gla).astype(np.float32)
    out.update(dC=dC, dreg=np.float32(gtau.sum(dtype=np.float64)), grad_log_alpha=gla, grad_tau=gtau)
    return out


def sq_dist(x, y, cost_scale: float = 1.0) -> np.ndarray:
    """Squared-distance cost of point clouds x [B,n,d], y [B,m,d] with the
    operation sequence of the GPU point-cloud solver (``orc_sq_dist``)."""
    x, y = _f32(x), _f32(y)
    B, n, d = x.shape
    m = y.shape[1]
    C = np.empty((B, n, m), np.float32)
    _lib("restated").orc_sq_dist(_ptr(x), _ptr(y), _ptr(C), B, n, m, d, cost_scale)
    return C


def sinkhorn_points_api(x, y, reg: float, n_iters: int, a=None, b=None, cost_scale: float = 1.0,
                        with_grad: bool = True, backward_iters: int | None = None) -> dict:
    """``sinkhorn(sq_dist(x, y), reg, n_iters, a, b)`` on the reference's CPU
    path (``sinkhorn_api``) plus the gradients of ``cost.sum()`` with respect
    to the points, chained through ``dC`` in float64:
    ``dx_i = 2 s sum_j dC_ij (x_i - y_j)``, ``dy_j = 2 s sum_i dC_ij (y_j - x_i)``."""
    x, y = _f32(x), _f32(y)
    C = sq_dist(x, y, cost_scale)
    out = sinkhorn_api(C, reg, n_iters, a, b, backward_iters=backward_iters, with_grad=with_grad)
    out["C"] = C
    if with_grad:
        dC = out["dC"].astype(np.float64)
        xd, yd = x.astype(np.float64), y.astype(np.float64)
        out["dx"] = (2.0 * cost_scale * (xd * dC.sum(axis=2)[..., None] - dC @ yd)).astype(np.float32)
        out["dy"] = (2.0 * cost_scale * (yd * dC.sum(axis=1)[..., None] -
                                         np.swapaxes(dC, 1, 2) @ xd)).astype(np.float32)
    return out


def bidir_api(sim, tau: float, lengths=None, grad_out=None, kind: str = "restated"):
    """``dot.bidirectional_softmax(sim, tau, lengths)`` forward (+ backward for
    ``grad_out``) on the reference's CPU path.  ``sim`` is upcast to fp32 as the
    reference does (``src/bidirectional_softmax/torch_cpu.cpp:41``)."""
    s = _f32(sim)
    B, L1, L2 = s.shape
    if lengths is None:
        lengths = np.tile(np.array([[L1, L2]], np.int32), (B, 1))
    out, rs, cs = bidir_forward(s, tau, lengths, kind=kind)
    res = {"out": out}
    if grad_out is not None:
        grad, gT = bidir_backward(s, out, grad_out, rs, cs, tau, lengths, kind=kind)
        res.update(grad=grad, grad_tau=gT)
    return res


# ----------------------------------------------------------------------------
# multi-threaded CPU timing (the reference's ops are single-threaded loops;
# a batch is split over threads, each running the unmodified op on its slice)
# ----------------------------------------------------------------------------

def sinkhorn_fwd_bwd_threaded(C, reg: float, n_iters: int, a=None, b=None, threads: int = 1,
                              kind: str = "reference", bwd_tol: float = 1e-6):
    """Reference CPU fwd+bwd, one problem slice per thread (ctypes drops the GIL).

    Each slice runs exactly what the reference's CPU path runs for
    ``dot.sinkhorn(C).cost.sum().backward()``: the forward op, then the backward
    op, which re-runs the forward before the implicit solve
    (``torch_cpu.cpp:300-326``).
    """
    C = _f32(C)
    B = C.shape[0]
    threads = max(1, min(int(threads), B))
    bounds = [(k * B // threads, (k + 1) * B // threads) for k in range(threads)]
    a = None if a is None else np.asarray(a, np.float32)
    b = None if b is None else np.asarray(b, np.float32)

    def work(lo_hi):
        lo, hi = lo_hi
        Cs = C[lo:hi]
        la = None if a is None else a[lo:hi]
        lb = None if b is None else b[lo:hi]
        log_alpha = -Cs
        lga = _log_marginal(la, hi - lo, Cs.shape[1])
        lgb = _log_marginal(lb, hi - lo, Cs.shape[2])
        P = sinkhorn_forward(log_alpha, reg, n_iters, lga, lgb, kind=kind)
        P2 = sinkhorn_forward(log_alpha, reg, n_iters, lga, lgb, kind=kind)
        G = Cs
        gla, _ = sinkhorn_backward_implicit(log_alpha, P2, G, reg, n_iters, tol=bwd_tol, kind=kind)
        return float((P * Cs).sum()), gla

    with ThreadPoolExecutor(max_workers=threads) as ex:
        res = list(ex.map(work, bounds))
    return res


def default_log_marginal(size: int) -> float:
    """``-log(float(size))`` in fp32, the reference's default (``torch_cuda.cpp:33-43``)."""
    return float(np.float32(-math.log(float(np.float32(size)))))
