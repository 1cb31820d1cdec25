"""Bidirectional softmax on the GPU, checked against the reference's golden
vectors, the CPU oracle, and an fp64 PyTorch restatement of the op; full-size
(configs[2]: B=64, 1024x1024, fp32 and bf16) properties with sampled parity."""

import numpy as np
import pytest
import torch

import dot
from oracle import oracle as O
from tests import util as U

pytestmark = pytest.mark.gpu
DEV = "cuda"
OUT_ATOL = 1e-5   # the reference's own CPU/CUDA consistency bound (tests/test_bidirectional_softmax.py:211)


def run(sim, tau, lengths=None, grad_out=None):
    s = sim.to(DEV).clone().requires_grad_(True)
    ln = None if lengths is None else torch.as_tensor(lengths, dtype=torch.int32).to(DEV)
    out = dot.bidirectional_softmax(s, tau=tau, lengths=ln)
    if grad_out is not None:
        (out * torch.as_tensor(grad_out).to(DEV)).sum().backward()
    return out.detach(), (s.grad if grad_out is not None else None)


def torch_fp64_reference(sim, tau, lengths):
    """Plain PyTorch fp64 restatement of the op (autograd gives the exact gradient)."""
    s = sim.double()
    B, L1, L2 = s.shape
    out = torch.zeros_like(s)
    for b in range(B):
        l1, l2 = int(lengths[b][0]), int(lengths[b][1])
        if l1 == 0 or l2 == 0:
            continue
        x = s[b, :l1, :l2] / tau
        row = torch.softmax(x, dim=1)
        col = torch.softmax(x, dim=0)
        pad = torch.nn.functional.pad(torch.sqrt(1e-9 + row * col), (0, L2 - l2, 0, L1 - l1))
        out = out.index_put((torch.tensor([b]),), pad.unsqueeze(0))
    return out


@pytest.mark.parametrize("path", U.golden_files("bidir_"), ids=lambda p: p.split("/")[-1])
def test_golden_bidir(path):
    d = U.load(path)
    bf16 = str(d["sim_dtype"]) == "torch.bfloat16"
    sim = torch.from_numpy(d["sim"]).view(torch.bfloat16) if bf16 else torch.from_numpy(d["sim"])
    out, grad = run(sim, float(d["tau"]), d.get("lengths"), d["grad_out"])
    assert out.dtype == torch.float32
    assert np.abs(U.to_np(out) - d["out"]).max() <= OUT_ATOL
    U.assert_normwise(out, d["out"], U.PLAN_RTOL, "out")
    ref_grad = U.bf16_bits_to_f32(d["grad"]) if bf16 else d["grad"]
    assert grad.dtype == (torch.bfloat16 if bf16 else torch.float32)
    tol = 1e-2 if bf16 else U.GRAD_RTOL   # bf16 gradients: one bf16 ulp (2^-8) of rounding either side
    U.assert_normwise(grad, ref_grad, tol, "grad")
    if "lengths" in d:
        for b, (l1, l2) in enumerate(d["lengths"]):
            assert (out[b, l1:, :] == 0).all() and (out[b, :, l2:] == 0).all()
            assert (grad[b, l1:, :] == 0).all() and (grad[b, :, l2:] == 0).all()


CASES = [
    # (B, L1, L2, tau, lengths or None)
    (2, 10, 15, 1.0, None),
    (3, 7, 9, 0.3, [[7, 9], [1, 1], [0, 4]]),
    (2, 33, 130, 0.1, [[33, 100], [20, 130]]),
    (1, 1, 1, 1.0, None),
    (2, 129, 127, 0.05, None),
    (1, 1300, 40, 0.2, [[1250, 33]]),   # tall: column statistics span several row chunks
    (2, 64, 1024, 0.1, None),
    # streaming path (L2 <= 1024, L2 % 4 == 0): fewer rows than row slots,
    # ragged and empty windows, more problems than resident CTAs
    (5, 3, 64, 0.5, None),
    (4, 37, 256, 0.2, [[37, 256], [30, 200], [1, 8], [0, 0]]),
    (300, 16, 96, 0.3, None),
    # full-width rows without per-element masks at each row width the sweeps
    # specialise (128, 512 columns: one warp per row; 1024: two), odd row
    # counts so blocks end part-filled
    (2, 50, 128, 0.5, None),
    (3, 41, 512, 0.2, None),
    (2, 23, 1024, 0.05, [[23, 1024], [22, 1024]]),
]


@pytest.mark.parametrize("B,L1,L2,tau,lengths", CASES, ids=lambda v: str(v))
def test_oracle_and_fp64_parity(B, L1, L2, tau, lengths):
    g = U.gen(L1 * 7 + L2)
    sim = torch.randn(B, L1, L2, generator=g)
    go = torch.randn(B, L1, L2, generator=g)
    ln = np.array(lengths if lengths is not None else [[L1, L2]] * B, np.int32)
    ref = O.bidir_api(sim.numpy(), tau, ln, go.numpy())
    out, grad = run(sim, tau, ln, go)
    assert np.abs(U.to_np(out) - ref["out"]).max() <= OUT_ATOL
    U.assert_normwise(out, ref["out"], U.PLAN_RTOL, "out vs oracle")
    U.assert_normwise(grad, ref["grad"], U.GRAD_RTOL, "grad vs oracle")
    # the exact gradient of the op (fp64 autograd) agrees to the same tolerance
    s64 = sim.double().requires_grad_(True)
    o64 = torch_fp64_reference(s64, tau, ln)
    (o64 * go.double()).sum().backward()
    U.assert_normwise(out, o64.detach(), U.PLAN_RTOL, "out vs fp64")
    U.assert_normwise(grad, s64.grad, U.GRAD_RTOL, "grad vs fp64")


@pytest.mark.parametrize("B,L1,L2,lengths", [(3, 45, 136, [[45, 136], [20, 64], [45, 7]]), (2, 9, 1024, None)])
def test_bf16_input_against_oracle(B, L1, L2, lengths):
    """bf16 input on the streaming path: the oracle runs on the same bf16 values
    upcast to fp32 (the reference's own cast); the bf16 gradient is compared
    within one bf16 rounding."""
    g = U.gen(L1 * 11 + L2)
    sim = torch.randn(B, L1, L2, generator=g).bfloat16()
    go = torch.randn(B, L1, L2, generator=g)
    ln = np.array(lengths if lengths is not None else [[L1, L2]] * B, np.int32)
    ref = O.bidir_api(sim.float().numpy(), 0.1, ln, go.numpy())
    out, grad = run(sim, 0.1, ln, go)
    assert grad.dtype == torch.bfloat16
    assert np.abs(U.to_np(out) - ref["out"]).max() <= OUT_ATOL
    U.assert_normwise(out, ref["out"], U.PLAN_RTOL, "out")
    ref_bf = torch.from_numpy(ref["grad"]).bfloat16().float()
    U.assert_normwise(grad.float(), ref_bf, 1e-2, "grad")


def test_reference_behaviour():
    sim = torch.randn(2, 10, 15, device=DEV)
    P = dot.bidirectional_softmax(sim, tau=1.0)
    assert P.shape == (2, 10, 15) and (P >= 0).all() and (P <= 1).all()
    P2 = dot.bidirectional_softmax(torch.randn(10, 15, device=DEV), tau=1.0)
    assert P2.shape == (10, 15)
    P3 = dot.BidirectionalSoftmax(tau=0.5)(torch.randn(1, 5, 7, device=DEV))
    assert P3.shape == (1, 5, 7)
    s = torch.zeros(1, 5, 5, device=DEV)
    for i in range(5):
        s[0, i, i] = 10.0
    sharp = dot.bidirectional_softmax(s, tau=0.1)[0].diag().sum()
    soft = dot.bidirectional_softmax(s, tau=10.0)[0].diag().sum()
    assert sharp > soft
    with pytest.raises(ValueError):
        dot.bidirectional_softmax(sim, tau=1.0, lengths=torch.ones(2, 2, dtype=torch.int64, device=DEV))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_cfg3_full_size(dtype):
    """B=64, 1024x1024, tau 0.1, upstream grad N(0,1)."""
    g = U.gen(0)
    sim = torch.randn(64, 1024, 1024, generator=g).to(dtype)
    go = torch.randn(64, 1024, 1024, generator=g)
    s = sim.to(DEV).requires_grad_(True)
    out = dot.bidirectional_softmax(s, tau=0.1)
    (out * go.to(DEV)).sum().backward()
    assert out.dtype == torch.float32 and s.grad.dtype == dtype
    assert torch.isfinite(out).all() and (out >= 0).all() and (out <= 1).all()
    for bi in (0, 63):
        ref = O.bidir_api(sim[bi:bi + 1].float().numpy(), 0.1, None, go[bi:bi + 1].numpy())
        assert np.abs(U.to_np(out[bi:bi + 1]) - ref["out"]).max() <= OUT_ATOL
        U.assert_normwise(out[bi:bi + 1], ref["out"], U.PLAN_RTOL, f"out[{bi}]")
        if dtype == torch.float32:
            U.assert_normwise(s.grad[bi:bi + 1], ref["grad"], U.GRAD_RTOL, f"grad[{bi}]")
        else:
            ref_bf = torch.from_numpy(ref["grad"]).bfloat16().float()
            U.assert_normwise(s.grad[bi:bi + 1].float(), ref_bf, 1e-2, f"grad[{bi}]")


def test_multi_chunk_ragged():
    """Ragged windows on rows split over two warps (L2 = 1024), 14 problems
    spread over the persistent CTAs' ranges (problems shared by several CTAs
    and merged by the last to arrive): a sample of them against the oracle."""
    B = 14
    g = U.gen(14)
    sim = torch.randn(B, 1024, 1024, generator=g)
    go = torch.randn(B, 1024, 1024, generator=g)
    rng = np.random.default_rng(14)
    ln = np.stack([rng.integers(1, 1025, B), rng.integers(1, 1025, B)], 1).astype(np.int32)
    ln[3] = [1024, 1024]
    out, grad = run(sim, 0.1, ln, go)
    for bi in (0, 5, 6, 11, 12, 13):
        ref = O.bidir_api(sim[bi:bi + 1].numpy(), 0.1, ln[bi:bi + 1], go[bi:bi + 1].numpy())
        assert np.abs(U.to_np(out[bi:bi + 1]) - ref["out"]).max() <= OUT_ATOL
        U.assert_normwise(out[bi:bi + 1], ref["out"], U.PLAN_RTOL, f"out[{bi}]")
        U.assert_normwise(grad[bi:bi + 1], ref["grad"], U.GRAD_RTOL, f"grad[{bi}]")
        l1, l2 = ln[bi]
        assert (out[bi, l1:, :] == 0).all() and (out[bi, :, l2:] == 0).all()
        assert (grad[bi, l1:, :] == 0).all() and (grad[bi, :, l2:] == 0).all()


def test_deterministic_bitwise():
    sim = torch.randn(4, 256, 512, device=DEV)
    go = torch.randn(4, 256, 512, device=DEV)
    res = []
    for _ in range(2):
        s = sim.clone().requires_grad_(True)
        o = dot.bidirectional_softmax(s, tau=0.1)
        (o * go).sum().backward()
        res.append((o.detach(), s.grad))
    assert torch.equal(res[0][0], res[1][0]) and torch.equal(res[0][1], res[1][1])
