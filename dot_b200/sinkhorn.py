"""Sinkhorn optimal transport: the drop-in for ``dot.sinkhorn`` and friends.

Public surface and behaviour follow the reference's ``dot/sinkhorn.py``:
``sinkhorn`` (:1284-1714), ``sinkhorn_from_scores`` (:1717-1860),
``Sinkhorn`` (:1863-1906), ``SinkhornFromScores`` (:1909-1954),
``SinkhornResult`` (:22-34), ``_prepare_marginal`` (:1259-1281).

Differences in mechanism (same results):

* one autograd Function returns both the plan and ``cost = sum(P * C)``; its
  backward receives both upstream gradients and runs one fused implicit
  backward (``G = grad_P + grad_cost * C``, ``dC = grad_cost * P - grad_log_alpha``),
  where the reference builds the cost with ATen outside its op (:1703) and
  lets autograd chain ``MulBackward``/``NegBackward``;
* the forward's dual potentials are saved for the backward, which therefore
  does not re-run the forward (the reference runs it three times per
  fwd+bwd: :1468-1508, ``src/sinkhorn/torch_cuda.cpp:842-853``);
* the ``tol`` early stop is decided on the device (no per-iteration host
  sync); ``n_iters_used`` is read back once, and only when ``tol > 0``.

Scope: the vanilla method with the implicit backward (default) or the
unrolled backward (``backward_mode='unrolled'``: differentiation through the
recorded iterations).  The reference's own CUDA dispatch turns some other
method requests into vanilla (:1371-1391); those are honoured.  Other
methods, schedules and ``n_iters='auto'`` raise ``NotImplementedError``.  Inputs must be CUDA
tensors: there is no CPU implementation.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Literal, Optional

import torch
import torch.nn as nn

from . import ops


@dataclass
class SinkhornResult:
    """Result from Sinkhorn computation.

    Attributes:
        transport_plan: Transport plan P of shape (B, n, m)
        cost: Transport cost sum(P * C) of shape (B,)
        converged: Whether the algorithm converged
        n_iters_used: Iterations run
    """
    transport_plan: torch.Tensor
    cost: Optional[torch.Tensor] = None
    converged: bool = True
    n_iters_used: Optional[int] = None


def _tau_value(reg) -> float:
    if torch.is_tensor(reg):
        if reg.numel() != 1:
            raise ValueError("reg/tau tensor must be scalar")
        return float(reg.detach().item())
    return float(reg)


class _SinkhornFn(torch.autograd.Function):
    """Forward: plan (+ cost); backward: fused implicit-function gradient."""

    @staticmethod
    def forward(ctx, X, reg, sign: float, n_iters: int, backward_iters: int, log_a, log_b, tol: float,
                want_cost: bool):
        tau = _tau_value(reg)
        P, cost, u, v, status = ops.sinkhorn_forward_raw(X, sign, tau, n_iters, log_a, log_b, tol=tol,
                                                         want_cost=want_cost)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(X, P, u, v)
        ctx.tau = tau
        ctx.sign = sign
        ctx.backward_iters = backward_iters
        ctx.reg_is_tensor = torch.is_tensor(reg)
        ctx.reg_meta = (reg.dtype, reg.device) if torch.is_tensor(reg) else None
        ctx.mark_non_differentiable(status)
        if cost is None:
            cost = P.new_zeros(0)
            ctx.mark_non_differentiable(cost)
        return P, cost, status

    @staticmethod
    def backward(ctx, grad_P, grad_cost, _grad_status):
        X, P, u, v = ctx.saved_tensors
        if grad_cost is not None and grad_cost.numel() == 0:
            grad_cost = None
        need_x = ctx.needs_input_grad[0]
        need_tau = ctx.reg_is_tensor and ctx.needs_input_grad[1]
        if (grad_P is None and grad_cost is None) or not (need_x or need_tau):
            return (None,) * 9
        gX, gtau = ops.sinkhorn_backward_raw(X, ctx.sign, P, u, v, grad_P, grad_cost, ctx.tau,
                                             ctx.backward_iters, want_grad_tau=need_tau)
        greg = None
        if need_tau:
            dt, dev = ctx.reg_meta
            greg = gtau.sum().to(device=dev, dtype=dt)
        return (gX if need_x else None), greg, None, None, None, None, None, None, None


class _SinkhornUnrolledFn(torch.autograd.Function):
    """Forward: plan (+ cost) with the potentials of every iteration recorded;
    backward: differentiation through the recorded iterations
    (``_SinkhornCudaDualUnrolledFunction``, ``dot/sinkhorn.py:243-311``, whose
    backward reruns the forward; here the recorded potentials are reused)."""

    @staticmethod
    def forward(ctx, X, reg, sign: float, n_iters: int, log_a, log_b, tol: float, want_cost: bool):
        tau = _tau_value(reg)
        P, cost, _u, _v, status, uh, vh = ops.sinkhorn_forward_hist_raw(X, sign, tau, n_iters, log_a, log_b,
                                                                         tol=tol, want_cost=want_cost)
        ctx.set_materialize_grads(False)
        ctx.save_for_backward(X, P, uh, vh, status)
        ctx.tau = tau
        ctx.sign = sign
        ctx.n_iters = n_iters
        ctx.tol = tol
        ctx.reg_is_tensor = torch.is_tensor(reg)
        ctx.reg_meta = (reg.dtype, reg.device) if torch.is_tensor(reg) else None
        ctx.mark_non_differentiable(status)
        if cost is None:
            cost = P.new_zeros(0)
            ctx.mark_non_differentiable(cost)
        return P, cost, status

    @staticmethod
    def backward(ctx, grad_P, grad_cost, _grad_status):
        X, P, uh, vh, status = ctx.saved_tensors
        if grad_cost is not None and grad_cost.numel() == 0:
            grad_cost = None
        need_x = ctx.needs_input_grad[0]
        need_tau = ctx.reg_is_tensor and ctx.needs_input_grad[1]
        if (grad_P is None and grad_cost is None) or not (need_x or need_tau):
            return (None,) * 8
        # with tol > 0 only the iterations actually run are differentiated
        # (the reference reruns the forward with n_iters_used, dot/sinkhorn.py:301)
        used = int(status[0].item()) if ctx.tol > 0 else ctx.n_iters
        gX, gtau = ops.sinkhorn_backward_unrolled_raw(X, ctx.sign, P, uh, vh, grad_P, grad_cost, ctx.tau, used,
                                                      want_grad_tau=need_tau)
        greg = None
        if need_tau:
            dt, dev = ctx.reg_meta
            greg = gtau.sum().to(device=dev, dtype=dt)
        return (gX if need_x else None), greg, None, None, None, None, None, None


def _prepare_marginal(marginal, batch: int, size: int, name: str, device, dtype):
    """Validate a marginal and broadcast it to [batch, size] (``dot/sinkhorn.py:1259-1281``)."""
    return _prepare_marginals([(marginal, batch, size, name)], device, dtype)[0]


def _prepare_marginals(specs, device, dtype):
    """``_prepare_marginal`` for several marginals ``(marginal, batch, size,
    name)`` with one host synchronisation: the reference's checks (shape,
    strictly positive, rows summing to 1 within atol = rtol = 1e-4, in that
    order per marginal, marginals in the order given) evaluated on the device
    and read back together.  Same results and errors as checking each in turn."""
    out, flags, names = [], [], []

    def raise_pending():   # the value errors of the marginals checked so far, in order
        if not flags:
            return
        for name, (nonpos, offsum) in zip(names, torch.stack(flags).tolist()):
            if nonpos:
                raise ValueError(f"{name} must be strictly positive")
            if offsum:
                raise ValueError(f"{name} must sum to 1 along the last dimension")

    for marginal, batch, size, name in specs:
        if marginal is None:
            out.append(None)
            continue
        if marginal.dim() == 1:
            marginal = marginal.unsqueeze(0).expand(batch, -1)
        if marginal.shape != (batch, size):
            raise_pending()
            raise ValueError(f"{name} must have shape ({batch}, {size}) or ({size},)")
        nonpos = (marginal <= 0).any().to(device)
        marginal = marginal.to(device=device, dtype=dtype)
        sums = marginal.sum(dim=-1)
        # torch.allclose(sums, 1, atol=1e-4, rtol=1e-4): |sums - 1| <= 1e-4 + 1e-4 * 1 (NaN fails)
        offsum = ~((sums - 1).abs() <= 2e-4).all()
        flags.append(torch.stack([nonpos, offsum]))
        names.append(name)
        out.append(marginal)
    raise_pending()
    return out


def _resolve_iters(n_iters, max_iter):
    if max_iter is not None:
        if n_iters is not None and n_iters != 20 and n_iters != max_iter:
            raise ValueError("pass either n_iters or its alias max_iter, not both")
        n_iters = max_iter
    if n_iters is None:
        n_iters = 20
    if isinstance(n_iters, str):
        if n_iters != "auto":
            raise ValueError("n_iters must be an int or 'auto'")
        raise NotImplementedError("dot_b200: n_iters='auto' (spectral preflight) is not implemented")
    return int(n_iters)


def _effective_method(method: str, tau: float, omega, schedule, reg_start, lr, beta1, beta2, eps_adam,
                      bias_correction, n: int, m: int):
    """The reference's CUDA dispatch (``dot/sinkhorn.py:1362-1391``): requests it
    serves with the vanilla kernels become 'vanilla'; anything else is out of scope."""
    if method == "auto":
        method = "newton" if (n <= 100 and m <= 100) else "vanilla"
    if method == "momentum" and omega is None:
        method = "vanilla"
    elif method == "anderson" and schedule is None and tau >= 0.05:
        method = "vanilla"
    elif method == "adam" and schedule is None:
        is_default_adam = (lr == 1.0 and beta1 == 0.9 and beta2 == 0.999 and eps_adam == 1e-8
                           and bias_correction)
        if tau >= 0.05 or is_default_adam:
            method = "vanilla"
    if method != "vanilla" or schedule is not None:
        raise NotImplementedError(
            f"dot_b200 implements the vanilla Sinkhorn method only (got method={method!r}, schedule={schedule!r})")
    return method


def _check_cuda(t: torch.Tensor, what: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"dot_b200: {what} must be a CUDA tensor (dot_b200 runs on NVIDIA GPUs only)")


def sinkhorn(
    cost_matrix: torch.Tensor,
    reg: float | torch.Tensor = 1.0,
    n_iters: int | Literal["auto"] = 20,
    backward_mode: Literal["unrolled", "implicit"] = "implicit",
    backward_iters: Optional[int] = None,
    a: Optional[torch.Tensor] = None,
    b: Optional[torch.Tensor] = None,
    method: str = "vanilla",
    omega: Optional[float] = None,
    anderson_k: int = 5,
    mixing_beta: float = 1.0,
    lr: float = 1.0,
    beta1: float = 0.9,
    beta2: float = 0.999,
    eps_adam: float = 1e-8,
    bias_correction: bool = True,
    reg_start: Optional[float] = None,
    schedule: Optional[str] = None,
    tol: float = 1e-6,
    dual: bool = True,
    *,
    max_iter: Optional[int] = None,
) -> SinkhornResult:
    """Entropy-regularised optimal transport of ``cost_matrix`` [B,n,m] or [n,m].

    Same signature and result as the reference's ``dot.sinkhorn``
    (``dot/sinkhorn.py:1284-1714``); ``max_iter`` is accepted as an alias of
    ``n_iters``.  ``tol > 0`` stops after the first iteration whose largest
    change of the row potential over the batch is below ``tol`` (the
    reference's CUDA criterion); ``tol = 0`` runs exactly ``n_iters``.
    ``dual=False`` selects the reference's full-matrix formulation, which runs
    a fixed ``n_iters`` (its ``tol`` is ignored); it is computed by the same
    kernels.
    """
    _check_cuda(cost_matrix, "cost_matrix")
    n_it = _resolve_iters(n_iters, max_iter)
    if n_it < 0:
        raise ValueError("n_iters must be >= 0")
    unbatched = cost_matrix.dim() == 2
    C = cost_matrix.unsqueeze(0) if unbatched else cost_matrix
    if C.dim() != 3:
        raise ValueError("cost_matrix must be (B, n, m) or (n, m)")
    B, n, m = C.shape
    a, b = _prepare_marginals([(a, B, n, "a"), (b, B, m, "b")], C.device, C.dtype)
    log_a = torch.log(a) if a is not None else None
    log_b = torch.log(b) if b is not None else None
    tau = _tau_value(reg)
    if not tau > 0:
        raise ValueError("tau must be > 0")
    if backward_iters is None:
        backward_iters = n_it
    _effective_method(method, tau, omega, schedule, reg_start, lr, beta1, beta2, eps_adam, bias_correction, n, m)
    if backward_mode not in ("implicit", "unrolled"):
        raise ValueError("backward_mode must be 'unrolled' or 'implicit'")
    run_tol = float(tol) if dual else 0.0
    if run_tol < 0:
        raise ValueError("tol must be >= 0")

    Cf = C.to(torch.float32).contiguous() if C.dtype != torch.float32 else C.contiguous()
    if backward_mode == "unrolled":
        P, cost, status = _SinkhornUnrolledFn.apply(Cf, reg, -1.0, n_it, log_a, log_b, run_tol, True)
    else:
        P, cost, status = _SinkhornFn.apply(Cf, reg, -1.0, n_it, int(backward_iters), log_a, log_b, run_tol, True)
    if dual and run_tol > 0:
        st = status.cpu()
        n_iters_used = int(st[0])
        converged = bool(st[1])
    else:
        n_iters_used = n_it
        converged = True if (not dual and tol == 0) or dual else False
    if cost_matrix.dtype not in (torch.float32, torch.bfloat16, torch.float16):
        cost = cost.to(cost_matrix.dtype)
    if unbatched:
        P = P.squeeze(0)
        cost = cost.squeeze(0)
    return SinkhornResult(transport_plan=P, cost=cost, converged=converged, n_iters_used=n_iters_used)


def sinkhorn_from_scores(
    log_alpha: torch.Tensor,
    tau: float | torch.Tensor = 1.0,
    n_iters: int | Literal["auto"] = 20,
    backward_mode: Literal["unrolled", "implicit"] = "implicit",
    backward_iters: Optional[int] = None,
    return_log: bool = False,
    a: Optional[torch.Tensor] = None,
    b: Optional[torch.Tensor] = None,
    tol: float = 1e-6,
    dual: bool = True,
    *,
    max_iter: Optional[int] = None,
) -> torch.Tensor:
    """Normalised transport plan (or its log) from log-scores ``log_alpha``.

    Same signature and result as the reference's ``dot.sinkhorn_from_scores``
    (``dot/sinkhorn.py:1717-1860``).  ``return_log=True`` gives a tensor with
    no autograd history, as in the reference.
    """
    _check_cuda(log_alpha, "log_alpha")
    n_it = _resolve_iters(n_iters, max_iter)
    unbatched = log_alpha.dim() == 2
    L = log_alpha.unsqueeze(0) if unbatched else log_alpha
    B, n, m = L.shape
    a, b = _prepare_marginals([(a, B, n, "a"), (b, B, m, "b")], L.device, L.dtype)
    log_a = torch.log(a) if a is not None else None
    log_b = torch.log(b) if b is not None else None
    if backward_iters is None:
        backward_iters = n_it
    if backward_mode not in ("implicit", "unrolled"):
        raise ValueError("backward_mode must be 'unrolled' or 'implicit'")
    run_tol = float(tol) if dual else 0.0
    if return_log:
        out = ops.sinkhorn_forward_raw(L.detach(), 1.0, _tau_value(tau), n_it, log_a, log_b, tol=run_tol,
                                       return_log=True)[0]
    else:
        X = L.to(torch.float32).contiguous() if L.dtype != torch.float32 else L.contiguous()
        if backward_mode == "unrolled":
            out, _, _ = _SinkhornUnrolledFn.apply(X, tau, 1.0, n_it, log_a, log_b, run_tol, False)
        else:
            out, _, _ = _SinkhornFn.apply(X, tau, 1.0, n_it, int(backward_iters), log_a, log_b, run_tol, False)
    return out.squeeze(0) if unbatched else out


def spectral_preflight(log_alpha, tau, tol: float = 1e-6, n_power: int = 5, alpha=None):
    """Iteration-count predictor of the reference (``dot/sinkhorn.py:860-905``): out of scope."""
    raise NotImplementedError("dot_b200: spectral_preflight is not implemented")


class Sinkhorn(nn.Module):
    """``nn.Module`` wrapper of :func:`sinkhorn` (``dot/sinkhorn.py:1863-1906``)."""

    def __init__(self, reg: float = 1.0, n_iters: int = 20,
                 backward_mode: Literal["unrolled", "implicit"] = "implicit",
                 backward_iters: Optional[int] = None, *, max_iter: Optional[int] = None):
        super().__init__()
        self.reg = reg
        self.n_iters = max_iter if max_iter is not None else n_iters
        self.backward_mode = backward_mode
        self.backward_iters = backward_iters

    def forward(self, cost_matrix: torch.Tensor) -> SinkhornResult:
        return sinkhorn(cost_matrix, reg=self.reg, n_iters=self.n_iters, backward_mode=self.backward_mode,
                        backward_iters=self.backward_iters)


class SinkhornFromScores(nn.Module):
    """``nn.Module`` wrapper of :func:`sinkhorn_from_scores` (``dot/sinkhorn.py:1909-1954``)."""

    def __init__(self, tau: float = 1.0, n_iters: int = 20,
                 backward_mode: Literal["unrolled", "implicit"] = "implicit",
                 backward_iters: Optional[int] = None):
        super().__init__()
        self.tau = tau
        self.n_iters = n_iters
        self.backward_mode = backward_mode
        self.backward_iters = backward_iters

    def forward(self, log_alpha: torch.Tensor) -> torch.Tensor:
        return sinkhorn_from_scores(log_alpha, tau=self.tau, n_iters=self.n_iters,
                                    backward_mode=self.backward_mode, backward_iters=self.backward_iters)
