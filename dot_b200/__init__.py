"""dot_b200: B200-native (sm_100a) implementation of dot's operator hot paths.

Public API (same names and behaviour as the reference package ``dot``,
``dot/__init__.py:32-64``):

    result = sinkhorn(cost_matrix, reg=1.0, n_iters=20)   # SinkhornResult
    P = sinkhorn_from_scores(log_alpha, tau=1.0)
    P = bidirectional_softmax(sim_matrix, tau=1.0)

plus the nn.Module wrappers ``Sinkhorn``, ``SinkhornFromScores`` and
``BidirectionalSoftmax``, and one extension with no counterpart in the
reference: ``sinkhorn_points(x, y, reg, n_iters)``, Sinkhorn on two point
clouds with the squared-distance cost built inside the solver.  Low-level
operators mirroring the reference's ``dot._ops`` live in
:mod:`dot_b200.ops`; the C-ABI they call is
``include/dot_b200.h``.  Importing the package loads the native library and
fails if it is missing.
"""

from . import _lib

_lib.load()

from . import ops as _ops  # noqa: E402
from .bidirectional_softmax import (  # noqa: E402
    BidirectionalSoftmax,
    bidirectional_softmax,
    bidirectional_softmax_with_lengths,
)
from .points import sinkhorn_points  # noqa: E402
from .sinkhorn import (  # noqa: E402
    Sinkhorn,
    SinkhornFromScores,
    SinkhornResult,
    sinkhorn,
    sinkhorn_from_scores,
    spectral_preflight,
)

__all__ = [
    "sinkhorn",
    "sinkhorn_from_scores",
    "spectral_preflight",
    "SinkhornResult",
    "Sinkhorn",
    "SinkhornFromScores",
    "bidirectional_softmax",
    "bidirectional_softmax_with_lengths",
    "BidirectionalSoftmax",
    "sinkhorn_points",
]
