"""Multi-GPU drivers: one process per GPU, ``torch.distributed`` over NCCL.

Two ways to spread Sinkhorn work over the GPUs of one box (the reference has
no multi-GPU path):

* **batch sharding** -- independent problems: each rank solves its contiguous
  share of the batch (:func:`shard_range`) with the ordinary single-GPU call;
  there is no collective on the data path.
* **row sharding** -- one problem too large or too slow for one GPU (e.g.
  32768 x 32768): rank r holds rows ``shard_range(n_total, r, world)`` of the
  cost.  Per iteration the row half-step is local; the column half-step needs
  LSE over all rows, which is combined from per-rank ``(max, sum)`` partials
  with one all-gather of every rank's ``(max, sum)`` pairs, merged in rank
  order on every rank (:func:`gather_column_pairs` and
  ``dot_sinkhorn_col_merge``), so all ranks hold the same ``v``.  This is the
  combine the single-GPU kernels use across row chunks; the only difference to
  one GPU is where the row chunks end.  :func:`combine_column_partials` is the
  two-all-reduce form of the same combine (MAX of the maxima, then SUM of the
  sums rescaled to the global maximum).
"""

from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from . import _lib


def shard_range(total: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced ``[lo, hi)`` share of ``total`` items for ``rank``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(int(total), int(world))
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


def combine_column_partials(col_max: torch.Tensor, col_sum: torch.Tensor,
                            rescale: Callable[[torch.Tensor, torch.Tensor, torch.Tensor], None],
                            group=None) -> tuple[torch.Tensor, torch.Tensor]:
    """Combine per-rank column (max, sum) partials into global ones.

    ``rescale(col_max, col_sum, gmax)`` must set ``col_sum *= exp(col_max - gmax)``
    in place.  Returns ``(gmax, gsum)``; ``col_sum`` is consumed.  Every rank
    performs the same two collectives in the same order.
    """
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return col_max, col_sum
    gmax = col_max.clone()
    dist.all_reduce(gmax, op=dist.ReduceOp.MAX, group=group)
    rescale(col_max, col_sum, gmax)
    dist.all_reduce(col_sum, op=dist.ReduceOp.SUM, group=group)
    return gmax, col_sum


def gather_column_pairs(pairs: torch.Tensor, group=None) -> tuple[torch.Tensor, int]:
    """All-gather this rank's column ``(max, sum)`` pairs ``[B, m, 2]`` into
    ``[world, B, m, 2]`` in rank order.  Returns ``(gathered, world)``; every
    rank performs the same single collective."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return pairs, 1
    world = dist.get_world_size(group)
    flat = pairs.contiguous()
    # concatenated along dim 0 (the layout every backend accepts), viewed stacked
    out = flat.new_empty((world * flat.shape[0],) + tuple(flat.shape[1:]))
    dist.all_gather_into_tensor(out, flat, group=group)
    return out.view((world,) + tuple(flat.shape)), world


def _c_rescale(col_max: torch.Tensor, col_sum: torch.Tensor, gmax: torch.Tensor) -> None:
    lib = _lib.load()
    _lib.check(lib.dot_sinkhorn_col_rescale(_lib.ptr(col_max), _lib.ptr(col_sum), _lib.ptr(gmax), col_max.numel(),
                                            _lib.stream_of(col_max)), "dot_sinkhorn_col_rescale")


def sinkhorn_rowshard(C_local: torch.Tensor, reg: float, n_iters: int, n_total: int,
                      log_a_local: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                      score_sign: float = -1.0, want_plan: bool = True, want_cost: bool = True,
                      group=None) -> dict:
    """Row-sharded Sinkhorn forward (fixed ``n_iters``).

    ``C_local`` [B, n_local, m] holds this rank's rows of the [B, n_total, m]
    matrix (cost with ``score_sign=-1``, log-scores with ``+1``);
    ``log_a_local`` [B, n_local] / ``log_b`` [B, m] are natural-log marginals
    (None = uniform over ``n_total`` / ``m``).  Returns ``{"P": plan rows or
    None, "cost": [B] global cost sum(P*C) or None, "u": [B, n_local],
    "v": [B, m]}``; ``v`` and ``cost`` are identical on every rank.
    """
    if not C_local.is_cuda:
        raise RuntimeError("dot_b200: C_local must be a CUDA tensor")
    X = C_local.to(torch.float32).contiguous()
    B, n, m = X.shape
    dev = X.device
    tau = float(reg)
    lib = _lib.load()
    st = _lib.stream_of(X)
    la = None if log_a_local is None else log_a_local.to(device=dev, dtype=torch.float32).contiguous()
    lb = None if log_b is None else log_b.to(device=dev, dtype=torch.float32).contiguous()
    u = torch.zeros((B, n), dtype=torch.float32, device=dev)
    v = torch.zeros((B, m), dtype=torch.float32, device=dev)
    pairs = torch.empty((B, m, 2), dtype=torch.float32, device=dev)
    nb = lib.dot_sinkhorn_rows_colpairs_workspace_bytes(B, n, m)
    ws = _lib.workspace(nb, dev)
    for _ in range(int(n_iters)):
        # row half-step and this shard's column pairs (one pass for wide rows)
        _lib.check(lib.dot_sinkhorn_rows_colpairs(_lib.ptr(X), float(score_sign), _lib.ptr(la), B, n, m,
                                                  int(n_total), tau, _lib.ptr(v), _lib.ptr(u), _lib.ptr(pairs),
                                                  _lib.ptr(ws), nb, st), "dot_sinkhorn_rows_colpairs")
        gathered, parts = gather_column_pairs(pairs, group=group)
        _lib.check(lib.dot_sinkhorn_col_merge(_lib.ptr(gathered), parts, _lib.ptr(lb), B, m, _lib.ptr(v), st),
                   "dot_sinkhorn_col_merge")
    out = {"u": u, "v": v, "P": None, "cost": None}
    if want_plan or want_cost:
        P = torch.empty((B, n, m), dtype=torch.float32, device=dev)
        cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
        pb = lib.dot_sinkhorn_plan_workspace_bytes(B, n, m)
        pws = _lib.workspace(pb, dev)
        _lib.check(lib.dot_sinkhorn_plan(_lib.ptr(X), float(score_sign), _lib.ptr(u), _lib.ptr(v), B, n, m, tau, 0,
                                         _lib.ptr(P), _lib.ptr(cost), _lib.ptr(pws), pb, st), "dot_sinkhorn_plan")
        if want_cost:
            if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
                dist.all_reduce(cost, op=dist.ReduceOp.SUM, group=group)
            out["cost"] = cost
        out["P"] = P if want_plan else None
    return out
