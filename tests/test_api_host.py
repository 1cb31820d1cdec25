"""Host-side API logic that needs no GPU: argument handling, marginal
validation, method dispatch, error behaviour."""

import pytest
import torch

import dot
import importlib

S = importlib.import_module("dot_b200.sinkhorn")


def test_cpu_tensors_are_rejected_loudly():
    with pytest.raises(RuntimeError, match="CUDA"):
        dot.sinkhorn(torch.rand(2, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        dot.sinkhorn_from_scores(torch.rand(2, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        dot.bidirectional_softmax(torch.rand(2, 4, 4))
    with pytest.raises(RuntimeError, match="CUDA"):
        dot._ops.sinkhorn(torch.rand(2, 4, 4), 1.0, 5)


def test_prepare_marginal_validation():
    assert S._prepare_marginal(None, 2, 3, "a", "cpu", torch.float32) is None
    a = torch.tensor([0.2, 0.3, 0.5])
    out = S._prepare_marginal(a, 2, 3, "a", "cpu", torch.float32)
    assert out.shape == (2, 3)
    with pytest.raises(ValueError, match="shape"):
        S._prepare_marginal(torch.ones(4) / 4, 2, 3, "a", "cpu", torch.float32)
    with pytest.raises(ValueError, match="positive"):
        S._prepare_marginal(torch.tensor([0.0, 0.5, 0.5]), 2, 3, "a", "cpu", torch.float32)
    with pytest.raises(ValueError, match="sum to 1"):
        S._prepare_marginal(torch.tensor([0.2, 0.2, 0.2]), 2, 3, "a", "cpu", torch.float32)


def test_iteration_aliases():
    assert S._resolve_iters(20, None) == 20
    assert S._resolve_iters(20, 100) == 100
    assert S._resolve_iters(100, 100) == 100
    with pytest.raises(ValueError):
        S._resolve_iters(30, 100)
    with pytest.raises(NotImplementedError):
        S._resolve_iters("auto", None)
    with pytest.raises(ValueError):
        S._resolve_iters("fast", None)


@pytest.mark.parametrize("kw,ok", [
    (dict(method="vanilla"), True),
    (dict(method="momentum"), True),                     # omega=None -> vanilla (dot/sinkhorn.py:1372)
    (dict(method="momentum", omega=1.5), False),
    (dict(method="anderson"), True),                     # tau >= 0.05 -> vanilla
    (dict(method="anderson", tau=0.01), False),
    (dict(method="adam"), True),                         # default adam -> vanilla
    (dict(method="adam", lr=0.5, tau=0.01), False),
    (dict(method="newton"), False),
    (dict(method="auto", n=200, m=200), True),           # large -> vanilla
    (dict(method="auto", n=50, m=50), False),            # small -> newton
    (dict(method="vanilla", schedule="linear"), False),
])
def test_method_dispatch_mirrors_reference(kw, ok):
    args = dict(method="vanilla", tau=0.1, omega=None, schedule=None, reg_start=None, lr=1.0, beta1=0.9,
                beta2=0.999, eps_adam=1e-8, bias_correction=True, n=200, m=200)
    args.update(kw)
    if ok:
        assert S._effective_method(**args) == "vanilla"
    else:
        with pytest.raises(NotImplementedError):
            S._effective_method(**args)


def test_modules_keep_their_settings():
    m = dot.Sinkhorn(reg=0.3, n_iters=7)
    assert (m.reg, m.n_iters, m.backward_mode) == (0.3, 7, "implicit")
    m2 = dot.Sinkhorn(reg=0.3, max_iter=9)
    assert m2.n_iters == 9
    bs = dot.BidirectionalSoftmax(tau=0.5)
    assert bs.tau == 0.5


def test_out_of_scope_entry_points_raise():
    with pytest.raises(NotImplementedError):
        dot.spectral_preflight(torch.rand(1, 4, 4), 0.1)


def test_unrolled_op_rejects_cpu_tensors():
    # implemented on the GPU only: no CPU fallback
    with pytest.raises(RuntimeError, match="CUDA"):
        dot._ops.sinkhorn_with_grads_unrolled(torch.rand(1, 4, 4), torch.rand(1, 4, 4), 1.0, 5)
    with pytest.raises(RuntimeError, match="CUDA"):
        dot.sinkhorn(torch.rand(1, 4, 4), reg=0.5, n_iters=5, backward_mode="unrolled")


def test_prepare_marginals_error_order():
    """Both marginals validated with one read-back, errors in the reference's
    order (a's checks before b's, shape before values per marginal)."""
    import pytest
    import torch

    from dot_b200.sinkhorn import _prepare_marginals

    good = torch.full((2, 3), 1 / 3)
    bad_sum = torch.full((2, 3), 0.5)
    neg = torch.tensor([[0.5, 0.6, -0.1]] * 2)
    dev, dt = torch.device("cpu"), torch.float32
    a, b = _prepare_marginals([(good, 2, 3, "a"), (good[:, :2] * 1.5, 2, 2, "b")], dev, dt)
    assert a.shape == (2, 3) and b.shape == (2, 2)
    with pytest.raises(ValueError, match="a must sum to 1"):
        _prepare_marginals([(bad_sum, 2, 3, "a"), (torch.ones(5), 2, 4, "b")], dev, dt)   # a before b's shape
    with pytest.raises(ValueError, match="b must have shape"):
        _prepare_marginals([(good, 2, 3, "a"), (torch.ones(5), 2, 4, "b")], dev, dt)
    with pytest.raises(ValueError, match="a must be strictly positive"):
        _prepare_marginals([(neg, 2, 3, "a"), (neg, 2, 3, "b")], dev, dt)
    with pytest.raises(ValueError, match="b must be strictly positive"):
        _prepare_marginals([(good, 2, 3, "a"), (neg, 2, 3, "b")], dev, dt)
    assert _prepare_marginals([(None, 2, 3, "a"), (None, 2, 3, "b")], dev, dt) == [None, None]
