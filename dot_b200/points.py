"""Sinkhorn on point clouds with the squared-distance cost built in the solver.

``sinkhorn_points(x, y, reg, n_iters)`` returns what
``dot.sinkhorn(cost_scale * cdist(x, y) ** 2, reg, n_iters, tol=0)`` returns,
without a cost matrix in memory: for low-dimensional clouds (d <= 4, any n
and m, ``tol=0``) every half-step rebuilds the entries it needs from the
points, so the iterations read no B x n x m array and the solver is bound by
the exponential unit instead of HBM.  Other requests (d > 4, ``tol > 0``)
materialise the cost once (``dot_sq_dist``) and run the matrix solvers.

The reference has no such entry point: its callers build the cost with
``torch.cdist`` and pass the matrix to ``sinkhorn`` (``dot/sinkhorn.py:1284``).
The cost entries here are ``s = (x_0 - y_0)^2``, then
``s = fma(x_k - y_k, x_k - y_k, s)``, times ``cost_scale`` (``ops.sq_dist``
gives the same matrix bit for bit).

Gradients: the backward materialises the cost once, runs the implicit
(adjoint) backward of the matrix path for ``dL/dC`` and chains it into the
points, ``dL/dx_i = 2 s sum_j dC_ij (x_i - y_j)`` and
``dL/dy_j = 2 s sum_i dC_ij (y_j - x_i)``.
"""

from __future__ import annotations

from typing import Optional

import torch

from . import ops
from .sinkhorn import SinkhornResult, _check_cuda, _prepare_marginals, _tau_value


class _SinkhornPointsFn(torch.autograd.Function):

    @staticmethod
    def forward(ctx, x, y, reg, cost_scale: float, n_iters: int, backward_iters: int, log_a, log_b, tol: float,
                want_plan: bool):
        tau = _tau_value(reg)
        P, cost, u, v, status = ops.sinkhorn_points_forward_raw(x, y, cost_scale, tau, n_iters, log_a, log_b,
                                                                tol=tol, want_plan=want_plan, want_cost=True)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(x, y, P, u, v)
        ctx.tau = tau
        ctx.cost_scale = cost_scale
        ctx.backward_iters = backward_iters
        ctx.reg_is_tensor = torch.is_tensor(reg)
        ctx.reg_meta = (reg.dtype, reg.device) if torch.is_tensor(reg) else None
        ctx.mark_non_differentiable(status)
        if P is None:
            P = cost.new_zeros(0)
            ctx.mark_non_differentiable(P)
        return P, cost, status

    @staticmethod
    def backward(ctx, grad_P, grad_cost, _grad_status):
        x, y, P, u, v = ctx.saved_tensors
        if grad_P is not None and grad_P.numel() == 0:
            grad_P = None
        need_x, need_y = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        need_tau = ctx.reg_is_tensor and ctx.needs_input_grad[2]
        if (grad_P is None and grad_cost is None) or not (need_x or need_y or need_tau):
            return (None,) * 10
        xf, yf = x.to(torch.float32), y.to(torch.float32)
        C = ops.sq_dist(xf, yf, ctx.cost_scale)
        gC, gtau = ops.sinkhorn_backward_raw(C, -1.0, P, u, v, grad_P, grad_cost, ctx.tau, ctx.backward_iters,
                                             want_grad_tau=need_tau)
        del C
        two_s = 2.0 * ctx.cost_scale
        gx = gy = None
        if need_x:
            gx = two_s * (xf * gC.sum(dim=2, keepdim=True) - torch.bmm(gC, yf))
            gx = gx.to(x.dtype)
        if need_y:
            gy = two_s * (yf * gC.sum(dim=1).unsqueeze(-1) - torch.bmm(gC.transpose(1, 2), xf))
            gy = gy.to(y.dtype)
        greg = None
        if need_tau:
            dt, dev = ctx.reg_meta
            greg = gtau.sum().to(device=dev, dtype=dt)
        return gx, gy, greg, None, None, None, None, None, None, None


def sinkhorn_points(
    x: torch.Tensor,
    y: torch.Tensor,
    reg: float | torch.Tensor = 1.0,
    n_iters: int = 20,
    a: Optional[torch.Tensor] = None,
    b: Optional[torch.Tensor] = None,
    *,
    cost_scale: float = 1.0,
    backward_iters: Optional[int] = None,
    return_plan: bool = True,
    tol: float = 0.0,
) -> SinkhornResult:
    """Entropic OT between point clouds ``x`` [B,n,d] (or [n,d]) and ``y``
    [B,m,d] (or [m,d]) under the cost ``cost_scale * |x_i - y_j|^2``.

    Same result as ``sinkhorn(ops.sq_dist(x, y, cost_scale), reg, n_iters, a,
    b, tol=tol)`` within rounding; ``return_plan=False`` skips the plan
    (``transport_plan`` is then ``None`` unless a gradient needs it) and, for
    d <= 4 and ``tol=0``, writes no B x n x m array at all.  The implicit backward gives gradients for
    ``x``, ``y`` and a tensor ``reg``.
    """
    _check_cuda(x, "x")
    _check_cuda(y, "y")
    if n_iters < 0:
        raise ValueError("n_iters must be >= 0")
    unbatched = x.dim() == 2
    if unbatched != (y.dim() == 2):
        raise ValueError("x and y must both be batched or both unbatched")
    xb = x.unsqueeze(0) if unbatched else x
    yb = y.unsqueeze(0) if unbatched else y
    if xb.dim() != 3 or yb.dim() != 3 or xb.size(0) != yb.size(0) or xb.size(2) != yb.size(2):
        raise ValueError("x and y must be (B, n, d) and (B, m, d)")
    B, n, _ = xb.shape
    m = yb.size(1)
    a, b = _prepare_marginals([(a, B, n, "a"), (b, B, m, "b")], xb.device, torch.float32)
    log_a = torch.log(a) if a is not None else None
    log_b = torch.log(b) if b is not None else None
    tau = _tau_value(reg)
    if not tau > 0:
        raise ValueError("tau must be > 0")
    if tol < 0:
        raise ValueError("tol must be >= 0")
    if backward_iters is None:
        backward_iters = n_iters
    grad_wanted = torch.is_grad_enabled() and (
        xb.requires_grad or yb.requires_grad or (torch.is_tensor(reg) and reg.requires_grad))
    want_plan = bool(return_plan or grad_wanted)
    P, cost, status = _SinkhornPointsFn.apply(xb, yb, reg, float(cost_scale), int(n_iters), int(backward_iters),
                                              log_a, log_b, float(tol), want_plan)
    if tol > 0:
        st = status.cpu()
        n_used, converged = int(st[0]), bool(st[1])
    else:
        n_used, converged = int(n_iters), True
    if not return_plan:
        P = None
    if unbatched:
        P = P.squeeze(0) if P is not None else None
        cost = cost.squeeze(0)
    return SinkhornResult(transport_plan=P, cost=cost, converged=converged, n_iters_used=n_used)
