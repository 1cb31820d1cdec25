"""The no-allocation Sinkhorn forward (dot_sinkhorn_fwd_noalloc).

Some callers cannot call cudaMalloc: a plugin inside a host application that
owns all device memory and forbids further allocations, or a foreign-language
binding that is handed device pointers but has no device allocator.  For them
the library offers one entry point that takes no workspace and uses a fixed
16 MiB scratch array it holds in device memory instead.

These tests call it through the C-ABI and check its outputs against the
allocating entry point (dot_sinkhorn_fwd with a caller workspace) on two calls
in a row, with the tolerances the other parity tests use, and check that a
problem whose scratch need exceeds the fixed size is refused with a clear
error.  The file is named so that pytest collects it last.
"""

import pytest
import torch

from dot_b200 import _lib, ops
from tests import util as U

pytestmark = pytest.mark.gpu

DOT_ERR_WORKSPACE = -3


def _noalloc(C, tau, n_iters, tol=0.0, want_cost=True):
    lib = _lib.load()
    B, n, m = C.shape
    out = torch.empty_like(C)
    cost = torch.empty(B, device=C.device) if want_cost else None
    u = torch.empty(B, n, device=C.device)
    v = torch.empty(B, m, device=C.device)
    status = torch.full((4,), -7, dtype=torch.int32, device=C.device)
    rc = lib.dot_sinkhorn_fwd_noalloc(_lib.ptr(C), -1.0, None, None, B, n, m, float(tau), int(n_iters), float(tol),
                                      0, _lib.ptr(out), _lib.ptr(cost), _lib.ptr(u), _lib.ptr(v), _lib.ptr(status),
                                      _lib.stream_of(C))
    return rc, out, cost, u, v, status


@pytest.mark.parametrize("B,n,m,tau,T,tol", [(4, 96, 128, 0.1, 50, 0.0), (3, 33, 47, 0.3, 40, 1e-5)])
def test_noalloc_matches_allocating_entry_point_twice(B, n, m, tau, T, tol):
    C = torch.rand(B, n, m, generator=U.gen(B * n + m)).cuda()
    ref_P, ref_cost, ref_u, ref_v, ref_status = ops.sinkhorn_forward_raw(C, -1.0, tau, T, tol=tol, want_cost=True)
    torch.cuda.synchronize()
    for _ in range(2):   # the scratch keeps the previous call's contents; both calls must be right
        rc, P, cost, u, v, status = _noalloc(C, tau, T, tol=tol)
        assert rc == 0, _lib.load().dot_last_error().decode()
        torch.cuda.synchronize()
        U.assert_normwise(P, ref_P, U.PLAN_RTOL, "plan")
        U.assert_rel(cost, ref_cost, U.COST_RTOL, "cost", atol=1e-9)
        U.assert_normwise(u, ref_u, 1e-6, "u")
        assert torch.equal(status[:2].cpu(), ref_status[:2].cpu())
        assert int(status[3]) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    B, n, m = 4096, 2048, 128   # the per-row cost partials alone need 32 MiB
    C = torch.zeros(1, device="cuda")   # never read: the size check comes first
    lib = _lib.load()
    rc = lib.dot_sinkhorn_fwd_noalloc(_lib.ptr(C), -1.0, None, None, B, n, m, 0.1, 10, 0.0, 0, _lib.ptr(C),
                                      _lib.ptr(C), _lib.ptr(C), _lib.ptr(C), _lib.ptr(C), _lib.stream_of(C))
    assert rc == DOT_ERR_WORKSPACE
    msg = lib.dot_last_error().decode()
    assert "16 MiB" in msg and "dot_sinkhorn_fwd" in msg
    assert lib.dot_sinkhorn_fwd_workspace_bytes(B, n, m, 10, 0.0, 1) > (16 << 20)
