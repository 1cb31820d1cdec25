"""Point-cloud Sinkhorn, host side: the oracle's squared-distance cost (the
operation sequence of the GPU solver) against float64 and against
torch.cdist(x, y) ** 2 -- the form the reference's callers build costs in --
the oracle's chain rule from dC to the points against autograd, and the
C-ABI's argument checks and workspace queries (no GPU needed)."""

import numpy as np
import torch

from dot_b200 import _lib
from oracle import oracle as O


def _clouds(seed, B=2, n=30, m=41, d=3):
    g = np.random.default_rng(seed)
    return g.random((B, n, d), dtype=np.float32), g.random((B, m, d), dtype=np.float32)


def test_oracle_sq_dist_vs_float64_and_cdist():
    for d in (1, 2, 3, 4, 9):
        x, y = _clouds(d, d=d)
        C = O.sq_dist(x, y, 1.5)
        C64 = 1.5 * ((x[:, :, None, :].astype(np.float64) - y[:, None, :, :]) ** 2).sum(-1)
        # d roundings of the differences, d - 1 fused adds, one scale: a few ulp
        assert np.abs(C - C64).max() <= 4 * d * 2.0 ** -24 * np.abs(C64).max()
        Ct = 1.5 * torch.cdist(torch.from_numpy(x).double(), torch.from_numpy(y).double()) ** 2
        np.testing.assert_allclose(C, Ct.numpy(), rtol=1e-5, atol=1e-6)


def test_oracle_sq_dist_uses_fused_adds():
    # s = (2^-15)^2 = 2^-30 exactly, then fma(t, t, s) with t = 1 + 2^-12:
    # t^2 = 1 + 2^-11 + 2^-24 lies on a rounding tie that the separately
    # rounded product breaks downwards (1 + 2^-11) and the fused add, which
    # also sees the 2^-30, upwards (1 + 2^-11 + 2^-23)
    x = np.array([[[2.0 ** -15, 1.0 + 2.0 ** -12]]], np.float32)
    y = np.zeros((1, 1, 2), np.float32)
    fused = np.float32(2.0 ** -30 + (1.0 + 2.0 ** -12) ** 2)
    assert fused == np.float32(1.0 + 2.0 ** -11 + 2.0 ** -23)
    assert O.sq_dist(x, y)[0, 0, 0] == fused


def test_oracle_point_gradients_follow_autograd():
    x, y = _clouds(5, B=1, n=12, m=10)
    out = O.sinkhorn_points_api(x, y, 0.3, 25, cost_scale=0.5)
    xt = torch.from_numpy(x).double().requires_grad_(True)
    yt = torch.from_numpy(y).double().requires_grad_(True)
    C = 0.5 * ((xt[:, :, None, :] - yt[:, None, :, :]) ** 2).sum(-1)
    C.backward(torch.from_numpy(out["dC"]).double())
    np.testing.assert_allclose(out["dx"], xt.grad.numpy(), rtol=1e-5, atol=1e-7)
    np.testing.assert_allclose(out["dy"], yt.grad.numpy(), rtol=1e-5, atol=1e-7)


def test_points_abi_checks_and_workspace():
    lib = _lib.load()
    # fused shape: partials and counters only, no B x n x m array
    fused = lib.dot_sinkhorn_points_fwd_workspace_bytes(1, 32768, 32768, 3, 500, 0.0, 0, 1)
    assert 0 < fused < 32768 * 32768
    # d > 4 or tol > 0: the materialised cost (+ a plan when none is wanted)
    mat = lib.dot_sinkhorn_points_fwd_workspace_bytes(1, 64, 8192, 5, 10, 0.0, 0, 1)
    assert mat >= 2 * 64 * 8192 * 4
    assert lib.dot_sinkhorn_points_fwd_workspace_bytes(1, 64, 8192, 3, 10, 1e-6, 1, 1) >= 64 * 8192 * 4
    assert lib.dot_sinkhorn_points_fwd_workspace_bytes(0, 64, 64, 3, 10, 0.0, 1, 1) == 0
    # argument errors are reported before any device work
    args = dict(tau=0.1, d=3, iters=5, tol=0.0, scale=1.0)
    for bad in (dict(tau=0.0), dict(d=0), dict(iters=-1), dict(tol=-1.0), dict(scale=float("inf"))):
        a = {**args, **bad}
        rc = lib.dot_sinkhorn_points_fwd(None, None, 1, 4, 4, a["d"], a["scale"], None, None, a["tau"], a["iters"],
                                         a["tol"], None, None, None, None, None, None, 0, None)
        assert rc == -1, bad
    assert lib.dot_sq_dist(None, None, 1, 2, 2, 0, 1.0, None, None) == -1
    assert lib.dot_sq_dist(None, None, 0, 2, 2, 3, 1.0, None, None) == 0


def test_points_rowshard_abi_checks():
    lib = _lib.load()
    # workspace: the gather buffer for every rank plus the shard's records and partials
    one = lib.dot_sinkhorn_points_fwd_rowshard_workspace_bytes(1, 4096, 32768, 3, 1)
    eight = lib.dot_sinkhorn_points_fwd_rowshard_workspace_bytes(1, 4096, 32768, 3, 8)
    assert eight - one >= 7 * 32768 * 8
    assert lib.dot_sinkhorn_points_fwd_rowshard_workspace_bytes(1, 4096, 32768, 5, 1) == 0
    assert lib.dot_sinkhorn_points_fwd_rowshard_workspace_bytes(1, 0, 64, 3, 2) > 0   # a shard without rows

    def call(d=3, tau=0.1, iters=5, n=4, n_total=8, scale=1.0):
        return lib.dot_sinkhorn_points_fwd_rowshard(None, None, None, None, 1, n, 4, d, n_total, scale, tau, iters,
                                                    None, None, None, None, None, None, None, 0, None)

    assert call(d=5) == -4            # DOT_ERR_UNSUPPORTED
    for bad in (dict(d=0), dict(tau=0.0), dict(iters=-1), dict(n_total=3), dict(scale=float("nan"))):
        assert call(**bad) == -1, bad
