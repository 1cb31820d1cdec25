"""The CPU oracle is pinned to the reference before anything is checked against it.

* the C restatement (oracle/dot_oracle.c) composed as the reference's public
  API (oracle/oracle.py) reproduces the golden vectors that the reference's own
  Python package produced (tests/golden/make_golden.py);
* when oracle/_ref/libdotref.so (the reference's CPU kernels compiled from
  their sources) is present, the restatement agrees with it bit for bit on
  random inputs.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests import util as U


@pytest.mark.parametrize("path", U.golden_files("sinkhorn_"), ids=lambda p: p.split("/")[-1])
def test_oracle_matches_reference_golden_sinkhorn(path):
    d = U.load(path)
    r = O.sinkhorn_api(d["C"], float(d["reg"]), int(d["n_iters"]), d.get("a"), d.get("b"),
                       backward_iters=int(d["backward_iters"]) if "backward_iters" in d else None,
                       g_cost=d["cost_weight"], grad_P=d.get("plan_weight"), bwd_tol=1e-6,
                       backward_mode=str(d["backward_mode"]) if "backward_mode" in d else "implicit")
    # the reference's CPU path, restated: plan and gradients bit-identical
    assert np.array_equal(r["P"], d["P"])
    assert np.array_equal(r["dC"], d["dC"])
    U.assert_rel(r["cost"], d["cost"], 1e-6, "cost", atol=1e-9)  # ATen fp32 sum vs fp64 sum
    if "dreg" in d:
        assert r["dreg"] == pytest.approx(float(d["dreg"]), rel=1e-6)
    assert int(d["n_iters_used"]) == int(d["n_iters"])


def test_oracle_matches_reference_golden_scores():
    d = U.load(U.golden_files("scores_")[0])
    P = O.sinkhorn_forward(d["log_alpha"], float(d["tau"]), int(d["n_iters"]))
    logP = O.sinkhorn_forward(d["log_alpha"], float(d["tau"]), int(d["n_iters"]), return_log=True)
    assert np.array_equal(P, d["P"])
    assert np.array_equal(logP, d["logP"])
    g, _ = O.sinkhorn_backward_implicit(d["log_alpha"], P, d["plan_weight"], float(d["tau"]), int(d["n_iters"]),
                                        tol=1e-6)
    assert np.array_equal(g, d["dlog_alpha"])


@pytest.mark.parametrize("path", U.golden_files("bidir_"), ids=lambda p: p.split("/")[-1])
def test_oracle_matches_reference_golden_bidir(path):
    d = U.load(path)
    sim = d["sim"]
    if str(d["sim_dtype"]) == "torch.bfloat16":
        sim = U.bf16_bits_to_f32(sim)
    r = O.bidir_api(sim, float(d["tau"]), d.get("lengths"), d["grad_out"])
    assert np.array_equal(r["out"], d["out"])
    grad = r["grad"]
    if str(d["grad_dtype"]) == "torch.bfloat16":
        import torch

        grad = torch.from_numpy(grad).bfloat16().view(torch.int16).numpy()
    assert np.array_equal(grad, d["grad"])


@pytest.mark.skipif(not O.available("reference"), reason="oracle/_ref not built (reference sources absent)")
@pytest.mark.parametrize("shape,tau,iters", [((2, 7, 11), 0.3, 20), ((1, 40, 33), 0.05, 60), ((3, 16, 16), 1.0, 5)])
def test_restatement_bitwise_vs_reference_kernels(shape, tau, iters):
    rng = np.random.default_rng(sum(shape))
    C = rng.random(shape, dtype=np.float32)
    la = np.log(rng.dirichlet(np.ones(shape[1]), size=shape[0]).astype(np.float32))
    for kind_args in [dict(), dict(log_a=la)]:
        a = O.sinkhorn_forward(-C, tau, iters, kind="restated", **kind_args)
        b = O.sinkhorn_forward(-C, tau, iters, kind="reference", **kind_args)
        assert np.array_equal(a, b)
    G = rng.standard_normal(shape).astype(np.float32)
    for tol in (0.0, 1e-6):
        ga, ta = O.sinkhorn_backward_implicit(-C, a, G, tau, iters, tol=tol, kind="restated")
        gb, tb = O.sinkhorn_backward_implicit(-C, a, G, tau, iters, tol=tol, kind="reference")
        assert np.array_equal(ga, gb) and np.array_equal(ta, tb)
    lengths = np.array([[shape[1], shape[2]]] * shape[0], np.int32)
    lengths[0] = [max(1, shape[1] - 2), max(1, shape[2] - 3)]
    oa, ra, ca = O.bidir_forward(C, tau, lengths, kind="restated")
    ob, rb, cb = O.bidir_forward(C, tau, lengths, kind="reference")
    assert np.array_equal(oa, ob) and np.array_equal(ra, rb) and np.array_equal(ca, cb)
    ga, ta = O.bidir_backward(C, oa, G, ra, ca, tau, lengths, kind="restated")
    gb, tb = O.bidir_backward(C, ob, G, rb, cb, tau, lengths, kind="reference")
    assert np.array_equal(ga, gb) and np.array_equal(ta, tb)


def test_dual_form_matches_primal_form():
    """The dual-potential restatement of the CUDA path (u, v) gives the same
    plan as the primal restatement of the CPU path (tests/test_sinkhorn.py:791-803)."""
    rng = np.random.default_rng(3)
    C = rng.random((2, 24, 31), dtype=np.float32)
    tau, T = 0.1, 50
    u, v, used, conv = O.sinkhorn_dual(-C, tau, T)
    K = (-C) * np.float32(1.0 / tau)
    P_dual = np.exp(K + u[:, :, None] + v[:, None, :])
    P_primal = O.sinkhorn_forward(-C, tau, T)
    U.assert_normwise(P_dual, P_primal, 1e-5, "dual vs primal")
    assert used == T and not conv


def test_dual_tol_stops_early():
    rng = np.random.default_rng(4)
    C = rng.random((2, 32, 32), dtype=np.float32)
    u, v, used, conv = O.sinkhorn_dual(-C, 0.5, 200, tol=1e-5)
    assert conv and used < 200
