"""Low-level operators on the C-ABI, mirroring the reference's op set.

The reference registers these through ``TORCH_LIBRARY_FRAGMENT(dot)``
(``src/sinkhorn/registry.cpp:21-57``, ``src/bidirectional_softmax/registry.cpp:17-35``)
and its Python layer calls them as ``dot._ops.<name>``.  Here each op is a
plain Python function over the C-ABI (``include/dot_b200.h``) with the same
name, argument meaning and return layout, except where noted:

* ``bidirectional_softmax`` returns ``[out, row_stats, col_stats]`` where
  the stats are [B,L1,2] / [B,L2,2] (max, 1/sum) instead of the reference's
  two full-size softmax buffers; ``bidirectional_softmax_backward`` takes the
  stats back.
* ``sinkhorn_dual_forward`` implements ``method=0`` (vanilla) and
  ``schedule=0``; other methods raise ``NotImplementedError``.
* ``sinkhorn_spectral_preflight`` raises ``NotImplementedError``.

All ops run on CUDA tensors only and enqueue on the current stream.
"""

from __future__ import annotations

import math
from typing import Optional

import torch

from . import _lib


def _need_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"dot_b200: {name} must be a CUDA tensor (dot_b200 has no CPU implementation)")


def _f32c(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.float32).contiguous()


def _check_marg(x: Optional[torch.Tensor], B: int, size: int, name: str, dev) -> Optional[torch.Tensor]:
    if x is None:
        return None
    if x.dim() != 2 or x.size(0) != B or x.size(1) != size:
        raise ValueError(f"{name} must have shape [B, {'n' if name == 'log_a' else 'm'}]")
    return _f32c(x.to(dev))


def sinkhorn_forward_raw(X: torch.Tensor, score_sign: float, tau: float, n_iters: int,
                         log_a: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                         tol: float = 0.0, return_log: bool = False, want_cost: bool = False):
    """One call of ``dot_sinkhorn_fwd``.

    Returns ``(out, cost_or_None, u, v, status)`` with ``status`` a device
    int32[4] tensor ``{n_iters_used, converged, ...}``.
    """
    _need_cuda(X, "input")
    if X.dim() != 3:
        raise ValueError("log_alpha must be 3D [B, n, m]")
    if not tau > 0.0:
        raise ValueError("tau must be > 0")
    if n_iters < 0:
        raise ValueError("n_iters must be >= 0")
    X = _f32c(X)
    B, n, m = X.shape
    dev = X.device
    la = _check_marg(log_a, B, n, "log_a", dev)
    lb = _check_marg(log_b, B, m, "log_b", dev)
    out = torch.empty((B, n, m), dtype=torch.float32, device=dev)
    cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
    u = torch.empty((B, n), dtype=torch.float32, device=dev)
    v = torch.empty((B, m), dtype=torch.float32, device=dev)
    status = torch.zeros((4,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    nbytes = lib.dot_sinkhorn_fwd_workspace_bytes(B, n, m, int(n_iters), float(tol), 1 if want_cost else 0)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_sinkhorn_fwd(_lib.ptr(X), float(score_sign), _lib.ptr(la), _lib.ptr(lb), B, n, m, float(tau),
                              int(n_iters), float(tol), 1 if return_log else 0, _lib.ptr(out), _lib.ptr(cost),
                              _lib.ptr(u), _lib.ptr(v), _lib.ptr(status), _lib.ptr(ws), nbytes,
                              _lib.stream_of(X))
    _lib.check(rc, "dot_sinkhorn_fwd")
    return out, cost, u, v, status


def sinkhorn_forward_hist_raw(X: torch.Tensor, score_sign: float, tau: float, n_iters: int,
                              log_a: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                              tol: float = 0.0, want_cost: bool = False):
    """One call of ``dot_sinkhorn_fwd_hist``: the forward that records the
    potentials after every iteration for the unrolled backward.

    Returns ``(P, cost_or_None, u, v, status, u_hist [T,B,n], v_hist [T,B,m])``.
    """
    _need_cuda(X, "input")
    if X.dim() != 3:
        raise ValueError("log_alpha must be 3D [B, n, m]")
    if not tau > 0.0:
        raise ValueError("tau must be > 0")
    if n_iters < 0:
        raise ValueError("n_iters must be >= 0")
    X = _f32c(X)
    B, n, m = X.shape
    dev = X.device
    la = _check_marg(log_a, B, n, "log_a", dev)
    lb = _check_marg(log_b, B, m, "log_b", dev)
    out = torch.empty((B, n, m), dtype=torch.float32, device=dev)
    cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
    u = torch.empty((B, n), dtype=torch.float32, device=dev)
    v = torch.empty((B, m), dtype=torch.float32, device=dev)
    uh = torch.empty((max(int(n_iters), 1), B, n), dtype=torch.float32, device=dev)
    vh = torch.empty((max(int(n_iters), 1), B, m), dtype=torch.float32, device=dev)
    status = torch.zeros((4,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    nbytes = lib.dot_sinkhorn_fwd_workspace_bytes(B, n, m, int(n_iters), float(tol), 1 if want_cost else 0)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_sinkhorn_fwd_hist(_lib.ptr(X), float(score_sign), _lib.ptr(la), _lib.ptr(lb), B, n, m, float(tau),
                                   int(n_iters), float(tol), _lib.ptr(out), _lib.ptr(cost), _lib.ptr(u), _lib.ptr(v),
                                   _lib.ptr(uh), _lib.ptr(vh), _lib.ptr(status), _lib.ptr(ws), nbytes,
                                   _lib.stream_of(X))
    _lib.check(rc, "dot_sinkhorn_fwd_hist")
    return out, cost, u, v, status, uh, vh


def sinkhorn_backward_unrolled_raw(X: torch.Tensor, score_sign: float, P: torch.Tensor, u_hist: torch.Tensor,
                                   v_hist: torch.Tensor, grad_P: Optional[torch.Tensor],
                                   grad_cost: Optional[torch.Tensor], tau: float, n_iters: int,
                                   want_grad_tau: bool = False):
    """One call of ``dot_sinkhorn_bwd_unrolled``; returns ``(grad_X, grad_tau_or_None)``."""
    X = _f32c(X)
    B, n, m = X.shape
    dev = X.device
    gP = None if grad_P is None else _f32c(grad_P)
    gc = None if grad_cost is None else _f32c(grad_cost.reshape(B))
    gX = torch.empty((B, n, m), dtype=torch.float32, device=dev)
    gtau = torch.empty((B,), dtype=torch.float32, device=dev) if want_grad_tau else None
    lib = _lib.load()
    nbytes = lib.dot_sinkhorn_bwd_unrolled_workspace_bytes(B, n, m)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_sinkhorn_bwd_unrolled(_lib.ptr(X), float(score_sign), _lib.ptr(P.contiguous()),
                                       _lib.ptr(u_hist), _lib.ptr(v_hist), _lib.ptr(gP), _lib.ptr(gc), B, n, m,
                                       float(tau), int(n_iters), _lib.ptr(gX), _lib.ptr(gtau), _lib.ptr(ws), nbytes,
                                       _lib.stream_of(X))
    _lib.check(rc, "dot_sinkhorn_bwd_unrolled")
    return gX, gtau


def sinkhorn_backward_raw(X: torch.Tensor, score_sign: float, P: torch.Tensor, u: Optional[torch.Tensor],
                          v: Optional[torch.Tensor], grad_P: Optional[torch.Tensor],
                          grad_cost: Optional[torch.Tensor], tau: float, bwd_iters: int,
                          want_grad_tau: bool = False):
    """One call of ``dot_sinkhorn_bwd``; returns ``(grad_X, grad_tau_or_None)``."""
    X = _f32c(X)
    B, n, m = X.shape
    dev = X.device
    gP = None if grad_P is None else _f32c(grad_P)
    gc = None if grad_cost is None else _f32c(grad_cost.reshape(B))
    gX = torch.empty((B, n, m), dtype=torch.float32, device=dev)
    gtau = torch.empty((B,), dtype=torch.float32, device=dev) if want_grad_tau else None
    lib = _lib.load()
    nbytes = lib.dot_sinkhorn_bwd_workspace_bytes(B, n, m, int(bwd_iters))
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_sinkhorn_bwd(_lib.ptr(X), float(score_sign), _lib.ptr(P.contiguous()), _lib.ptr(u), _lib.ptr(v),
                              _lib.ptr(gP), _lib.ptr(gc), B, n, m, float(tau), int(bwd_iters), _lib.ptr(gX),
                              _lib.ptr(gtau), _lib.ptr(ws), nbytes, _lib.stream_of(X))
    _lib.check(rc, "dot_sinkhorn_bwd")
    return gX, gtau


def sq_dist(x: torch.Tensor, y: torch.Tensor, cost_scale: float = 1.0) -> torch.Tensor:
    """``dot_sq_dist``: C [B,n,m] = cost_scale * |x_i - y_j|^2 from x [B,n,d],
    y [B,m,d], with the entry arithmetic the point-cloud solver uses."""
    _need_cuda(x, "x")
    _need_cuda(y, "y")
    if x.dim() != 3 or y.dim() != 3 or x.size(0) != y.size(0) or x.size(2) != y.size(2):
        raise ValueError("x and y must be [B, n, d] and [B, m, d]")
    x, y = _f32c(x), _f32c(y)
    B, n, d = x.shape
    m = y.size(1)
    C = torch.empty((B, n, m), dtype=torch.float32, device=x.device)
    rc = _lib.load().dot_sq_dist(_lib.ptr(x), _lib.ptr(y), B, n, m, d, float(cost_scale), _lib.ptr(C),
                                 _lib.stream_of(x))
    _lib.check(rc, "dot_sq_dist")
    return C


def sinkhorn_points_forward_raw(x: torch.Tensor, y: torch.Tensor, cost_scale: float, tau: float, n_iters: int,
                                log_a: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                                tol: float = 0.0, want_plan: bool = True, want_cost: bool = True):
    """One call of ``dot_sinkhorn_points_fwd`` (cost = cost_scale * squared
    distances of the clouds x [B,n,d], y [B,m,d], built inside the solver).

    Returns ``(plan_or_None, cost_or_None, u, v, status)``.
    """
    _need_cuda(x, "x")
    _need_cuda(y, "y")
    if x.dim() != 3 or y.dim() != 3 or x.size(0) != y.size(0) or x.size(2) != y.size(2):
        raise ValueError("x and y must be [B, n, d] and [B, m, d]")
    if not tau > 0.0:
        raise ValueError("tau must be > 0")
    if n_iters < 0:
        raise ValueError("n_iters must be >= 0")
    x, y = _f32c(x), _f32c(y)
    B, n, d = x.shape
    m = y.size(1)
    dev = x.device
    la = _check_marg(log_a, B, n, "log_a", dev)
    lb = _check_marg(log_b, B, m, "log_b", dev)
    plan = torch.empty((B, n, m), dtype=torch.float32, device=dev) if want_plan else None
    cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
    u = torch.empty((B, n), dtype=torch.float32, device=dev)
    v = torch.empty((B, m), dtype=torch.float32, device=dev)
    status = torch.zeros((4,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    nbytes = lib.dot_sinkhorn_points_fwd_workspace_bytes(B, n, m, d, int(n_iters), float(tol), 1 if want_plan else 0,
                                                         1 if want_cost else 0)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_sinkhorn_points_fwd(_lib.ptr(x), _lib.ptr(y), B, n, m, d, float(cost_scale), _lib.ptr(la),
                                     _lib.ptr(lb), float(tau), int(n_iters), float(tol), _lib.ptr(plan),
                                     _lib.ptr(cost), _lib.ptr(u), _lib.ptr(v), _lib.ptr(status), _lib.ptr(ws),
                                     nbytes, _lib.stream_of(x))
    _lib.check(rc, "dot_sinkhorn_points_fwd")
    return plan, cost, u, v, status


# ---- reference-named ops ------------------------------------------------------

def sinkhorn(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None) -> torch.Tensor:
    """Plan of ``log_alpha`` after ``n_iters`` iterations (``registry.cpp:31``)."""
    return sinkhorn_forward_raw(log_alpha, 1.0, float(tau), int(n_iters), log_a, log_b)[0]


def sinkhorn_log(log_alpha, tau: float, n_iters: int, log_a=None, log_b=None) -> torch.Tensor:
    """Log-plan of ``log_alpha`` (``registry.cpp:34``)."""
    return sinkhorn_forward_raw(log_alpha, 1.0, float(tau), int(n_iters), log_a, log_b, return_log=True)[0]


def sinkhorn_dual_forward(log_alpha, tau: float, n_iters: int, tol: float = 0.0, log_a=None, log_b=None,
                          return_log: bool = False, method: int = 0, omega: float = 1.5, anderson_k: int = 5,
                          mixing_beta: float = 1.0, lr: float = 1.0, beta1: float = 0.9, beta2: float = 0.999,
                          eps_adam: float = 1e-8, bias_correction: bool = True, reg_start: float = -1.0,
                          schedule: int = 0):
    """``[P_or_logP, n_iters_used, converged]`` (``registry.cpp:38-45``).

    ``n_iters_used``/``converged`` are int64 CPU tensors as in the reference
    (``torch_cuda.cpp:261-263``); reading them synchronises the stream.
    """
    if method != 0 or schedule != 0:
        raise NotImplementedError("dot_b200 implements the vanilla Sinkhorn method (method=0, schedule=0) only")
    if anderson_k < 1:
        raise ValueError("anderson_k must be >= 1")
    out, _, _, _, status = sinkhorn_forward_raw(log_alpha, 1.0, float(tau), int(n_iters), log_a, log_b,
                                                tol=float(tol), return_log=return_log)
    st = status.cpu().to(torch.int64)
    return [out, st[0].clone(), st[1].clone()]


def sinkhorn_with_grads_implicit(log_alpha, grad_P, tau: float, n_iters: int, backward_iters: int,
                                 log_a=None, log_b=None):
    """``[P, grad_log_alpha, grad_tau]`` (``registry.cpp:56``)."""
    P, _, u, v, _ = sinkhorn_forward_raw(log_alpha, 1.0, float(tau), int(n_iters), log_a, log_b)
    g, gt = sinkhorn_backward_raw(log_alpha, 1.0, P, u, v, grad_P, None, float(tau), int(backward_iters),
                                  want_grad_tau=True)
    return [P, g, gt]


def sinkhorn_with_grads_unrolled(log_alpha, grad_P, tau: float, n_iters: int, log_a=None, log_b=None):
    """``[P, grad_log_alpha, grad_tau]`` through ``n_iters`` unrolled iterations (``registry.cpp:52``)."""
    P, _, _, _, _, uh, vh = sinkhorn_forward_hist_raw(log_alpha, 1.0, float(tau), int(n_iters), log_a, log_b)
    g, gt = sinkhorn_backward_unrolled_raw(log_alpha, 1.0, P, uh, vh, grad_P, None, float(tau), int(n_iters),
                                           want_grad_tau=True)
    return [P, g, gt]


def sinkhorn_spectral_preflight(*args, **kwargs):
    raise NotImplementedError("dot_b200: spectral preflight (n_iters='auto') is not implemented")


def _bs_dtype(t: torch.Tensor) -> tuple[torch.Tensor, int]:
    if t.dtype == torch.bfloat16:
        return t.contiguous(), _lib.DOT_BF16
    return _f32c(t), _lib.DOT_F32


def _bs_lengths(lengths: torch.Tensor, B: int, dev) -> torch.Tensor:
    if lengths.dim() != 2 or lengths.size(1) != 2 or lengths.size(0) != B:
        raise ValueError("lengths must be [B, 2]")
    if lengths.dtype != torch.int32:
        raise ValueError("lengths must be int32")
    return lengths.to(dev).contiguous()


def bidirectional_softmax(sim: torch.Tensor, tau: float, lengths: torch.Tensor):
    """``[out, row_stats, col_stats]`` (``src/bidirectional_softmax/registry.cpp:31``)."""
    _need_cuda(sim, "sim")
    if sim.dim() != 3:
        raise ValueError("sim_matrix must be 3D [B, L1, L2]")
    if not tau > 0.0:
        raise ValueError("tau must be > 0")
    s, dt = _bs_dtype(sim)
    B, L1, L2 = s.shape
    dev = s.device
    ln = _bs_lengths(lengths, B, dev)
    out = torch.empty((B, L1, L2), dtype=torch.float32, device=dev)
    rs = torch.empty((B, L1, 2), dtype=torch.float32, device=dev)
    cs = torch.empty((B, L2, 2), dtype=torch.float32, device=dev)
    lib = _lib.load()
    nbytes = lib.dot_bidir_fwd_workspace_bytes(B, L1, L2)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_bidir_fwd(_lib.ptr(s), dt, _lib.ptr(ln), B, L1, L2, float(tau), _lib.ptr(out), _lib.ptr(rs),
                           _lib.ptr(cs), _lib.ptr(ws), nbytes, _lib.stream_of(s))
    _lib.check(rc, "dot_bidir_fwd")
    return [out, rs, cs]


def bidirectional_softmax_backward(sim: torch.Tensor, output: torch.Tensor, grad_output: torch.Tensor,
                                   row_stats: torch.Tensor, col_stats: torch.Tensor, tau: float,
                                   lengths: torch.Tensor, grad_dtype: Optional[torch.dtype] = None,
                                   want_grad_tau: bool = True):
    """``[grad_sim, grad_tau]`` (``src/bidirectional_softmax/registry.cpp:34``).

    ``output`` is accepted for signature parity and not read: the kernels
    recompute it from ``sim`` and the stats.  ``grad_sim`` is float32, or
    bfloat16 when ``grad_dtype=torch.bfloat16``.  ``want_grad_tau=False``
    skips the temperature gradient (returned as None).
    """
    _need_cuda(sim, "sim")
    s, dt = _bs_dtype(sim)
    B, L1, L2 = s.shape
    dev = s.device
    ln = _bs_lengths(lengths, B, dev)
    g = _f32c(grad_output)
    gdt = torch.bfloat16 if grad_dtype == torch.bfloat16 else torch.float32
    gsim = torch.empty((B, L1, L2), dtype=gdt, device=dev)
    gtau = torch.empty((B,), dtype=torch.float32, device=dev) if want_grad_tau else None
    lib = _lib.load()
    nbytes = lib.dot_bidir_bwd_workspace_bytes(B, L1, L2)
    ws = _lib.workspace(nbytes, dev)
    rc = lib.dot_bidir_bwd(_lib.ptr(s), dt, _lib.ptr(ln), B, L1, L2, float(tau), _lib.ptr(row_stats.contiguous()),
                           _lib.ptr(col_stats.contiguous()), _lib.ptr(g), _lib.ptr(gsim),
                           _lib.DOT_BF16 if gdt == torch.bfloat16 else _lib.DOT_F32, _lib.ptr(gtau),
                           _lib.ptr(ws), nbytes, _lib.stream_of(s))
    _lib.check(rc, "dot_bidir_bwd")
    return [gsim, gtau]


def default_log_marginal(size: int) -> float:
    """``-log(float(size))`` in fp32 (``src/sinkhorn/torch_cuda.cpp:33-43``)."""
    return float(torch.tensor(-math.log(float(size)), dtype=torch.float32))
