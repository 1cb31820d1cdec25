"""Test helpers: golden fixtures, tolerance checks, seeded inputs."""

from __future__ import annotations

import glob
import os

import numpy as np
import torch

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

# Tolerances (north star: rel 1e-5 on plan and cost, 1e-4 on gradients).  The
# plan and gradients are compared normwise per batch element,
# max|a - b| <= rtol * max|b|, because elementwise relative error of tiny plan
# entries sits at the fp32 noise floor of the reference itself (~2e-5).
PLAN_RTOL = 1e-5
COST_RTOL = 1e-5
GRAD_RTOL = 1e-4


def golden_files(prefix: str) -> list[str]:
    return sorted(glob.glob(os.path.join(GOLDEN, prefix + "*.npz")))


def load(path: str) -> dict:
    return dict(np.load(path))


def bf16_bits_to_f32(a: np.ndarray) -> np.ndarray:
    return (a.astype(np.int32) << 16).view(np.float32)


def to_np(t) -> np.ndarray:
    if isinstance(t, torch.Tensor):
        return t.detach().float().cpu().numpy()
    return np.asarray(t)


def normwise_err(actual, expected) -> float:
    """max over leading index b of max|a_b - e_b| / max|e_b|."""
    a, e = to_np(actual).astype(np.float64), to_np(expected).astype(np.float64)
    if a.shape != e.shape:
        raise AssertionError(f"shape {a.shape} != {e.shape}")
    if a.ndim < 2:
        a, e = a[None], e[None]
    worst = 0.0
    for b in range(a.shape[0]):
        scale = np.abs(e[b]).max()
        err = np.abs(a[b] - e[b]).max()
        worst = max(worst, err / scale if scale > 0 else err)
    return worst


def assert_normwise(actual, expected, rtol: float, what: str = "") -> None:
    err = normwise_err(actual, expected)
    assert err <= rtol, f"{what}: normwise error {err:.3e} > {rtol:.1e}"


def assert_rel(actual, expected, rtol: float, what: str = "", atol: float = 0.0) -> None:
    a, e = to_np(actual).astype(np.float64), to_np(expected).astype(np.float64)
    bad = np.abs(a - e) > rtol * np.abs(e) + atol
    assert not bad.any(), f"{what}: max rel err {np.max(np.abs(a - e) / np.maximum(np.abs(e), 1e-30)):.3e}"


def gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return g


def sqdist_cost(B: int, n: int, m: int, d: int, seed: int) -> torch.Tensor:
    """cfg2 inputs: squared distances of N(0,1) clouds, divided by the per-batch max."""
    g = gen(seed)
    x = torch.randn(B, n, d, generator=g)
    y = torch.randn(B, m, d, generator=g)
    C = torch.cdist(x, y).square()
    return (C / C.amax(dim=(1, 2), keepdim=True)).float()


def dirichlet(B: int, n: int, seed: int) -> torch.Tensor:
    torch.manual_seed(seed)
    return torch.distributions.Dirichlet(torch.ones(n)).sample((B,)).float()
