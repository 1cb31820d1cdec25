"""Low-level operator access under the reference's module name ``dot._ops``
(``dot/_ops.py:70-82`` of caseysm/dot); implemented by :mod:`dot_b200.ops`."""

from dot_b200.ops import (  # noqa: F401
    bidirectional_softmax,
    bidirectional_softmax_backward,
    sinkhorn,
    sinkhorn_dual_forward,
    sinkhorn_log,
    sinkhorn_spectral_preflight,
    sinkhorn_with_grads_implicit,
    sinkhorn_with_grads_unrolled,
)
