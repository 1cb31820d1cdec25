"""Sinkhorn on point clouds (dot_sinkhorn_points_fwd / dot_b200.sinkhorn_points):
the squared-distance cost built inside the half-step kernels, checked against
the CPU oracle on the oracle's own cost matrix (oracle.sq_dist, the same
operation sequence as dot_sq_dist, which is checked bit for bit), against the
matrix path on dot_sq_dist's matrix, and through size-independent properties
at configs[4]'s full size.

Tolerances (north star): plan normwise rel 1e-5, cost rel 1e-5, gradients
normwise rel 1e-4 (tests/util.py).
"""

import numpy as np
import pytest
import torch

import dot_b200
from dot_b200 import _lib, ops
from oracle import oracle as O
from tests import util as U
from tests.test_sinkhorn_gpu import check_cfg5_regime

pytestmark = pytest.mark.gpu
DEV = "cuda"


def cube(B: int, n: int, d: int, seed: int) -> torch.Tensor:
    return torch.rand(B, n, d, generator=U.gen(seed))


def counted(fn):
    """fn() with launch counting; returns (result, per-class launches)."""
    _lib.prof_begin(time_events=False)
    out = fn()
    torch.cuda.synchronize()
    return out, _lib.prof_end()


@pytest.mark.parametrize("d", [1, 2, 3, 4, 7])
def test_sq_dist_bitwise_vs_oracle(d):
    x, y = cube(2, 37, d, 10 + d), cube(2, 301, d, 20 + d)
    C = ops.sq_dist(x.to(DEV), y.to(DEV), 1.7)
    assert np.array_equal(C.cpu().numpy(), O.sq_dist(x.numpy(), y.numpy(), 1.7))


# (B, n, m, d, reg, T): the point kernels (d <= 4, tol = 0) at sizes that
# cover one and several side-b chunks, ragged chunks, batches and every d
FUSED = [
    (1, 96, 8192, 3, 0.05, 40),      # several chunks per row
    (2, 40, 16384, 2, 0.05, 30),     # two problems
    (1, 70, 8227, 3, 0.05, 20),      # ragged last chunk and step
    (1, 33, 8192, 1, 0.1, 25),       # 1-D clouds
    (1, 50, 8192, 4, 0.05, 25),      # 4-D clouds
    (16, 512, 512, 3, 0.05, 30),     # configs[1]-like shape, one chunk
    (3, 1000, 300, 2, 0.1, 20),      # more points than side b, rows over several CTAs
    (5, 7, 9, 3, 0.3, 15),           # tiny
]


@pytest.mark.parametrize("B,n,m,d,reg,T", FUSED, ids=lambda v: str(v))
def test_fused_points_match_oracle(B, n, m, d, reg, T):
    x, y = cube(B, n, d, 100 + n), cube(B, m, d, 200 + d)
    (P, cost, u, v, status), prof = counted(
        lambda: ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, reg, T))
    assert prof["sk_fwd_iter"]["launches"] == 4 * T, prof   # two half-steps and two merges per iteration
    ref = O.sinkhorn_points_api(x.numpy(), y.numpy(), reg, T, with_grad=False)
    U.assert_normwise(P, ref["P"], U.PLAN_RTOL, "plan")
    U.assert_rel(cost, ref["cost"], U.COST_RTOL, "cost")


@pytest.mark.parametrize("m,d", [(8192, 3), (16384, 2), (600, 4)])
def test_fused_points_match_matrix_path(m, d):
    """The same problem through the matrix solvers on dot_sq_dist's matrix:
    equal within rounding (plan, cost and potentials)."""
    x, y = cube(2, 45, d, 300 + m), cube(2, m, d, 400 + d)
    xd, yd = x.to(DEV), y.to(DEV)
    P1, c1, u1, v1, _ = ops.sinkhorn_points_forward_raw(xd, yd, 0.5, 0.02, 30)
    C = ops.sq_dist(xd, yd, 0.5)
    P2, c2, u2, v2, _ = ops.sinkhorn_forward_raw(C, -1.0, 0.02, 30, want_cost=True)
    U.assert_normwise(P1, P2, U.PLAN_RTOL, "plan")
    U.assert_rel(c1, c2, U.COST_RTOL, "cost")
    # potentials are O(1/reg); their difference stays at fp32 rounding of that scale
    assert (u1 - u2).abs().max().item() <= 1e-4 and (v1 - v2).abs().max().item() <= 1e-4


@pytest.mark.parametrize("n,m,T", [(96, 32768, 100), (700, 32768, 30)], ids=["32768-100it", "32768-700rows"])
def test_fused_points_cfg5_regime(n, m, T):
    """configs[4]'s regime (U[0,1)^3 clouds, reg 0.01, 32768 columns: K spans
    0 .. -300), against the float64 iteration and the reference's fp32
    formulations."""
    x, y = cube(1, n, 3, 500 + n), cube(1, m, 3, 600)
    (P, cost, u, v, status), prof = counted(
        lambda: ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, 0.01, T))
    assert prof["sk_fwd_iter"]["launches"] == 4 * T, prof
    check_cfg5_regime(P, cost, O.sq_dist(x.numpy(), y.numpy()), 0.01, T, f"points {n}x{m}")


def test_cost_only_writes_no_plan_and_matches():
    x, y = cube(1, 64, 3, 700), cube(1, 8192, 3, 701)
    P, c1, u1, v1, _ = ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, 0.05, 20)
    none, c2, u2, v2, _ = ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, 0.05, 20, want_plan=False)
    assert none is None
    assert torch.equal(c1, c2) and torch.equal(u1, u2) and torch.equal(v1, v2)
    res = dot_b200.sinkhorn_points(x[0].to(DEV), y[0].to(DEV), 0.05, 20, return_plan=False)
    assert res.transport_plan is None and res.cost.shape == ()
    assert torch.equal(res.cost, c1[0])


def test_fused_points_marginals():
    B, n, m = 2, 80, 8192
    x, y = cube(B, n, 3, 800), cube(B, m, 3, 801)
    a = U.dirichlet(B, n, 802) + 1e-3
    a = a / a.sum(-1, keepdim=True)
    b = U.dirichlet(B, m, 803) + 1e-4
    b = b / b.sum(-1, keepdim=True)
    res = dot_b200.sinkhorn_points(x.to(DEV), y.to(DEV), 0.05, 25, a=a.to(DEV), b=b.to(DEV))
    ref = O.sinkhorn_points_api(x.numpy(), y.numpy(), 0.05, 25, a.numpy(), b.numpy(), with_grad=False)
    U.assert_normwise(res.transport_plan, ref["P"], U.PLAN_RTOL, "plan")
    U.assert_rel(res.cost, ref["cost"], U.COST_RTOL, "cost")


# requests the point kernels do not take: the cost is materialised and the
# matrix solvers run
FALLBACK = [
    (1, 40, 8192, 6, 0.05, 15, 0.0),  # d > 4 (wide matrix kernel)
    (3, 48, 40, 5, 0.2, 30, 0.0),     # d > 4 (resident solver)
    (2, 64, 300, 3, 0.1, 50, 1e-4),   # tol > 0
]


@pytest.mark.parametrize("B,n,m,d,reg,T,tol", FALLBACK, ids=lambda v: str(v))
def test_materialised_points_match_oracle(B, n, m, d, reg, T, tol):
    x, y = cube(B, n, d, 900 + n), cube(B, m, d, 901 + m)
    res = dot_b200.sinkhorn_points(x.to(DEV), y.to(DEV), reg, T, tol=tol)
    if tol == 0.0:
        ref = O.sinkhorn_points_api(x.numpy(), y.numpy(), reg, T, with_grad=False)
        U.assert_normwise(res.transport_plan, ref["P"], U.PLAN_RTOL, "plan")
        U.assert_rel(res.cost, ref["cost"], U.COST_RTOL, "cost")
    else:   # same stopping iteration and result as the matrix API on the same cost
        C = ops.sq_dist(x.to(DEV), y.to(DEV))
        r2 = dot_b200.sinkhorn(C, reg, T, tol=tol)
        assert res.n_iters_used == r2.n_iters_used and res.converged == r2.converged
        assert torch.equal(res.transport_plan, r2.transport_plan)


@pytest.mark.parametrize("B,n,m,d,reg,T", [(2, 40, 56, 3, 0.2, 30), (1, 64, 8192, 3, 0.05, 25)],
                         ids=["materialised", "fused"])
def test_points_gradients_match_oracle(B, n, m, d, reg, T):
    x, y = cube(B, n, d, 1000 + m), cube(B, m, d, 1001)
    xg = x.to(DEV).requires_grad_(True)
    yg = y.to(DEV).requires_grad_(True)
    r = torch.tensor(reg, device=DEV, requires_grad=True)
    res = dot_b200.sinkhorn_points(xg, yg, r, T, cost_scale=0.75)
    res.cost.sum().backward()
    ref = O.sinkhorn_points_api(x.numpy(), y.numpy(), reg, T, cost_scale=0.75)
    U.assert_normwise(res.transport_plan, ref["P"], U.PLAN_RTOL, "plan")
    U.assert_normwise(xg.grad, ref["dx"], U.GRAD_RTOL, "dx")
    U.assert_normwise(yg.grad, ref["dy"], U.GRAD_RTOL, "dy")
    # d loss / d reg sums signed terms that cancel; as for the matrix path the
    # yardstick is the float64 evaluation of the same backward on the float64
    # plan, and the fp32 oracle may be off by its own gap plus the tolerance
    C = ref["C"]
    _, gtau64 = O.sinkhorn_implicit_fp64(-C, O.sinkhorn_dual_fp64(-C, reg, T), C.astype(np.float64), reg, T)
    dreg64 = float(gtau64.sum())
    assert float(r.grad) == pytest.approx(dreg64, rel=U.GRAD_RTOL, abs=1e-6)
    own = abs(float(ref["dreg"]) - dreg64)
    assert abs(float(r.grad) - float(ref["dreg"])) <= own + U.GRAD_RTOL * abs(dreg64) + 1e-6


def test_points_argument_errors():
    x, y = cube(1, 8, 3, 1), cube(1, 9, 3, 2)
    with pytest.raises(ValueError):
        dot_b200.sinkhorn_points(x.to(DEV), y.to(DEV)[..., :2], 0.1, 5)
    with pytest.raises(ValueError):
        ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, 0.0, 5)
    with pytest.raises(RuntimeError):
        dot_b200.sinkhorn_points(x, y, 0.1, 5)   # CPU tensors: no CPU implementation


def test_points_cfg5_full_size_cost_only():
    """configs[4] (32768 x 32768 U[0,1)^3 clouds, reg 0.01, 500 iterations)
    from the points, writing no plan: potentials finite, the cost equal to
    the matrix path's on dot_sq_dist's matrix, and the potentials equal to
    it within rounding."""
    x, y = cube(1, 32768, 3, 1234), cube(1, 32768, 3, 1235)
    xd, yd = x.to(DEV), y.to(DEV)
    (none, c1, u1, v1, st), prof = counted(
        lambda: ops.sinkhorn_points_forward_raw(xd, yd, 1.0, 0.01, 500, want_plan=False))
    assert none is None and prof["sk_fwd_iter"]["launches"] == 4 * 500
    assert torch.isfinite(u1).all() and torch.isfinite(v1).all() and torch.isfinite(c1).all()
    C = ops.sq_dist(xd, yd)
    P2, c2, u2, v2, _ = ops.sinkhorn_forward_raw(C, -1.0, 0.01, 500, want_cost=True)
    del P2, C
    torch.cuda.empty_cache()
    U.assert_rel(c1, c2, U.COST_RTOL, "cost vs the matrix path")
    # potentials are O(1/reg) = O(100) in magnitude; rounding differences of
    # the two kernel configurations stay at the fp32 level of that scale
    assert (u1 - u2).abs().max().item() <= 1e-3 and (v1 - v2).abs().max().item() <= 1e-3


def test_points_batch_beyond_grid_limit():
    """More problems than one launch's grid.z holds (65535): the half-steps
    run in batch slices."""
    B, n, m, d = 70000, 6, 10, 2
    x, y = cube(B, n, d, 1300), cube(B, m, d, 1301)
    P, cost, _, _, _ = ops.sinkhorn_points_forward_raw(x.to(DEV), y.to(DEV), 1.0, 0.2, 10)
    ref = O.sinkhorn_points_api(x.numpy(), y.numpy(), 0.2, 10, with_grad=False)
    U.assert_normwise(P, ref["P"], U.PLAN_RTOL, "plan")
    U.assert_rel(cost, ref["cost"], U.COST_RTOL, "cost")
