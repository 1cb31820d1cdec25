"""Bidirectional softmax: the drop-in for ``dot.bidirectional_softmax``.

    out[i,j] = sqrt(1e-9 + softmax_j(sim/T)[i,j] * softmax_i(sim/T)[i,j])

inside each batch's (L1, L2) length window, 0 outside.  Public surface and
behaviour follow the reference's ``dot/bidirectional_softmax.py`` (:19-162).
The output is float32 for float32 and bfloat16 inputs (the reference upcasts,
``src/bidirectional_softmax/torch_cuda.cpp:58``); bfloat16 is read natively.
The autograd Function saves only per-row/per-column softmax statistics, not
the reference's two full-size softmax buffers (:30-35).
"""

from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import ops


class _BidirectionalSoftmaxFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, sim_matrix: torch.Tensor, tau: float, lengths: torch.Tensor) -> torch.Tensor:
        out, rs, cs = ops.bidirectional_softmax(sim_matrix, tau, lengths)
        ctx.save_for_backward(sim_matrix, lengths, rs, cs)
        ctx.tau = float(tau)
        return out

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        sim, lengths, rs, cs = ctx.saved_tensors
        gdt = torch.bfloat16 if sim.dtype == torch.bfloat16 else None
        # tau is a plain float here (no gradient), so its gradient is not computed
        grad_sim, _ = ops.bidirectional_softmax_backward(sim, None, grad_output, rs, cs, ctx.tau, lengths,
                                                         grad_dtype=gdt, want_grad_tau=False)
        return grad_sim, None, None


def _make_lengths(B: int, L1: int, L2: int, device) -> torch.Tensor:
    """Default [B,2] int32 lengths (``dot/bidirectional_softmax.py:52-57``)."""
    lengths = torch.empty(B, 2, dtype=torch.int32, device=device)
    lengths[:, 0] = L1
    lengths[:, 1] = L2
    return lengths


def bidirectional_softmax(sim_matrix: torch.Tensor, tau: float = 1.0,
                          lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Soft matching matrix of ``sim_matrix`` [B,L1,L2] or [L1,L2] (``dot/bidirectional_softmax.py:60-106``)."""
    if not sim_matrix.is_cuda:
        raise RuntimeError("dot_b200: sim_matrix must be a CUDA tensor (dot_b200 runs on NVIDIA GPUs only)")
    unbatched = sim_matrix.dim() == 2
    if unbatched:
        sim_matrix = sim_matrix.unsqueeze(0)
    B, L1, L2 = sim_matrix.shape
    if lengths is None:
        lengths = _make_lengths(B, L1, L2, sim_matrix.device)
    result = _BidirectionalSoftmaxFn.apply(sim_matrix, tau, lengths)
    return result.squeeze(0) if unbatched else result


def bidirectional_softmax_with_lengths(sim_matrix: torch.Tensor, lengths: torch.Tensor,
                                       tau: float = 1.0) -> torch.Tensor:
    """Same as :func:`bidirectional_softmax` with ``lengths`` required (``:109-126``)."""
    return bidirectional_softmax(sim_matrix, tau=tau, lengths=lengths)


class BidirectionalSoftmax(nn.Module):
    """``nn.Module`` wrapper (``dot/bidirectional_softmax.py:129-162``)."""

    def __init__(self, tau: float = 1.0):
        super().__init__()
        self.tau = tau

    def forward(self, sim_matrix: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        return bidirectional_softmax(sim_matrix, tau=self.tau, lengths=lengths)
