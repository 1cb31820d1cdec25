"""Multi-GPU drivers: one process per GPU, ``torch.distributed`` for the
plumbing (the reference has no multi-GPU path).

Two ways to spread Sinkhorn work over the GPUs of one box:

* **batch sharding** (:func:`sinkhorn_batchshard`) -- independent problems:
  each rank solves its contiguous share of the batch (:func:`shard_range`)
  with the ordinary single-GPU call; there is no collective on the data path,
  only a gather of the results at the end when the caller asks for them.
* **row sharding** (:func:`sinkhorn_rowshard`) -- one problem too large or
  too slow for one GPU (e.g. 32768 x 32768): rank r holds rows
  ``shard_range(n_total, r, world)`` of the cost.  Per iteration the row
  half-step is local; the column half-step needs the LSE over all rows, which
  is combined from per-rank ``(max, sum)`` pairs: one NCCL all-gather of
  every rank's pairs, merged in rank order on every rank, so all ranks hold
  the same ``v``.  The whole loop runs inside the C-ABI
  (``dot_sinkhorn_fwd_rowshard``) on an NCCL communicator the library creates
  once per process group (:func:`nccl_communicator`).
"""

from __future__ import annotations

import ctypes
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


def _world(group) -> tuple[int, int]:
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


# ---------------------------------------------------------------------------
# NCCL communicator owned by the library (row sharding)
# ---------------------------------------------------------------------------

_COMMS: dict = {}


def broadcast_unique_id(make_id: Callable[[], bytes], group=None) -> bytes:
    """Rank 0 of ``group`` calls ``make_id()``; every rank returns its bytes.
    Works over any ``torch.distributed`` backend (object broadcast)."""
    rank, world = _world(group)
    if world == 1:
        return make_id()
    obj = [make_id() if rank == 0 else None]
    src = dist.get_global_rank(group, 0) if group is not None else 0
    dist.broadcast_object_list(obj, src=src, group=group)
    return obj[0]


def _new_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _lib.check(_lib.load().dot_nccl_unique_id(buf), "dot_nccl_unique_id")
    return buf.raw


def nccl_communicator(group=None, device: Optional[torch.device] = None):
    """The library's NCCL communicator for ``group`` (ranks in group order),
    created on first use with ``device`` current and cached; ``None`` for a
    single rank.  Every rank of the group must call this together the first
    time."""
    rank, world = _world(group)
    if world == 1:
        return None
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    key = (id(group) if group is not None else None, dev.index)
    comm = _COMMS.get(key)
    if comm is not None:
        return comm
    uid = broadcast_unique_id(_new_unique_id, group)
    handle = ctypes.c_void_p()
    with torch.cuda.device(dev):
        _lib.check(_lib.load().dot_nccl_comm_init(ctypes.byref(handle), world, ctypes.c_char_p(uid), rank),
                   "dot_nccl_comm_init")
    _COMMS[key] = handle
    return handle


def release_communicators() -> None:
    """Destroy the communicators created by :func:`nccl_communicator` (call
    before ``destroy_process_group``; their work must be complete)."""
    lib = _lib.load()
    for key in list(_COMMS):
        _lib.check(lib.dot_nccl_comm_destroy(_COMMS.pop(key)), "dot_nccl_comm_destroy")


# ---------------------------------------------------------------------------
# row sharding
# ---------------------------------------------------------------------------

def sinkhorn_rowshard(C_local: torch.Tensor, reg: float, n_iters: int, n_total: int,
                      log_a_local: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                      score_sign: float = -1.0, want_plan: bool = True, want_cost: bool = True,
                      group=None) -> dict:
    """Row-sharded Sinkhorn forward (fixed ``n_iters``).

    ``C_local`` [B, n_local, m] holds this rank's rows of the [B, n_total, m]
    matrix (cost with ``score_sign=-1``, log-scores with ``+1``), the ranks of
    ``group`` holding consecutive row blocks in rank order (as
    :func:`shard_range` gives them); ``log_a_local`` [B, n_local] / ``log_b``
    [B, m] are natural-log marginals (None = uniform over ``n_total`` / ``m``).
    Returns ``{"P": plan rows or None, "cost": [B] global cost sum(P*C) or
    None, "u": [B, n_local], "v": [B, m]}``; ``v`` and ``cost`` are identical
    on every rank.  Every rank must call it with the same arguments apart from
    its rows.  Raises ``RuntimeError`` if a bounded wait inside the kernels
    expired.
    """
    if not C_local.is_cuda:
        raise RuntimeError("dot_b200: C_local must be a CUDA tensor")
    X = C_local.to(torch.float32).contiguous()
    B, n, m = X.shape
    dev = X.device
    tau = float(reg)
    lib = _lib.load()
    _, world = _world(group)
    comm = nccl_communicator(group, dev)
    la = None if log_a_local is None else log_a_local.to(device=dev, dtype=torch.float32).contiguous()
    lb = None if log_b is None else log_b.to(device=dev, dtype=torch.float32).contiguous()
    u = torch.empty((B, n), dtype=torch.float32, device=dev)
    v = torch.empty((B, m), dtype=torch.float32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    need_plan = want_plan or want_cost
    P = torch.empty((B, n, m), dtype=torch.float32, device=dev) if need_plan else None
    cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
    nb = lib.dot_sinkhorn_fwd_rowshard_workspace_bytes(B, n, m, world)
    ws = _lib.workspace(nb, dev)
    _lib.check(lib.dot_sinkhorn_fwd_rowshard(_lib.ptr(X), float(score_sign), _lib.ptr(la), _lib.ptr(lb), B, n, m,
                                             int(n_total), tau, int(n_iters), comm, _lib.ptr(P), _lib.ptr(cost),
                                             _lib.ptr(u), _lib.ptr(v), _lib.ptr(status), _lib.ptr(ws), nb,
                                             _lib.stream_of(X)), "dot_sinkhorn_fwd_rowshard")
    if int(status.item()) != 0:
        raise RuntimeError(f"dot_sinkhorn_fwd_rowshard: a bounded wait expired (status 0x{int(status.item()):x})")
    return {"u": u, "v": v, "P": P if want_plan else None, "cost": cost}


def sinkhorn_points_rowshard(x_local: torch.Tensor, y: torch.Tensor, reg: float, n_iters: int, n_total: int,
                             log_a_local: Optional[torch.Tensor] = None, log_b: Optional[torch.Tensor] = None,
                             cost_scale: float = 1.0, want_plan: bool = False, want_cost: bool = True,
                             group=None) -> dict:
    """Row-sharded Sinkhorn forward on point clouds (the cost
    ``cost_scale * |x_i - y_j|^2`` built in the half-steps, fixed ``n_iters``,
    1 <= d <= 4).

    ``x_local`` [B, n_local, d] holds this rank's points of the n_total rows,
    ``y`` [B, m, d] all column points; ``log_a_local`` / ``log_b`` as for
    :func:`sinkhorn_rowshard`.  Per iteration the library runs the row and
    column half-steps on this rank's rows and all-gathers one (max, sum) pair
    per column over NCCL.  Returns ``{"P": plan rows or None, "cost": [B] or
    None, "u": [B, n_local], "v": [B, m]}``; ``v`` and ``cost`` are the same on
    every rank.  Every rank must call it with the same arguments apart from
    its rows.
    """
    if not (x_local.is_cuda and y.is_cuda):
        raise RuntimeError("dot_b200: x_local and y must be CUDA tensors")
    x = x_local.to(torch.float32).contiguous()
    yy = y.to(device=x.device, dtype=torch.float32).contiguous()
    if x.dim() != 3 or yy.dim() != 3 or x.size(0) != yy.size(0) or x.size(2) != yy.size(2):
        raise ValueError("x_local and y must be [B, n_local, d] and [B, m, d]")
    B, n, d = x.shape
    m = yy.size(1)
    dev = x.device
    lib = _lib.load()
    _, world = _world(group)
    comm = nccl_communicator(group, dev)
    la = None if log_a_local is None else log_a_local.to(device=dev, dtype=torch.float32).contiguous()
    lb = None if log_b is None else log_b.to(device=dev, dtype=torch.float32).contiguous()
    u = torch.empty((B, n), dtype=torch.float32, device=dev)
    v = torch.empty((B, m), dtype=torch.float32, device=dev)
    status = torch.zeros((1,), dtype=torch.int32, device=dev)
    P = torch.empty((B, n, m), dtype=torch.float32, device=dev) if want_plan else None
    cost = torch.empty((B,), dtype=torch.float32, device=dev) if want_cost else None
    nb = lib.dot_sinkhorn_points_fwd_rowshard_workspace_bytes(B, n, m, d, world)
    ws = _lib.workspace(nb, dev)
    _lib.check(lib.dot_sinkhorn_points_fwd_rowshard(_lib.ptr(x), _lib.ptr(yy), _lib.ptr(la), _lib.ptr(lb), B, n, m, d,
                                                    int(n_total), float(cost_scale), float(reg), int(n_iters), comm,
                                                    _lib.ptr(P), _lib.ptr(cost), _lib.ptr(u), _lib.ptr(v),
                                                    _lib.ptr(status), _lib.ptr(ws), nb, _lib.stream_of(x)),
               "dot_sinkhorn_points_fwd_rowshard")
    return {"u": u, "v": v, "P": P, "cost": cost}


# ---------------------------------------------------------------------------
# batch sharding
# ---------------------------------------------------------------------------

def _gather_batch(local: torch.Tensor, B: int, world: int, group) -> torch.Tensor:
    """All-gather per-rank batch slices (``shard_range`` sizes, possibly
    unequal) into the full [B, ...] tensor on every rank."""
    sizes = [shard_range(B, r, world) for r in range(world)]
    most = max(hi - lo for lo, hi in sizes)
    pad = local.new_zeros((most,) + tuple(local.shape[1:]))
    pad[: local.shape[0]] = local
    out = local.new_empty((world * most,) + tuple(local.shape[1:]))
    dist.all_gather_into_tensor(out, pad.contiguous(), group=group)
    return torch.cat([out[r * most: r * most + (hi - lo)] for r, (lo, hi) in enumerate(sizes)], dim=0)


def sinkhorn_batchshard(C: torch.Tensor, reg: float = 1.0, n_iters: int = 20, a: Optional[torch.Tensor] = None,
                        b: Optional[torch.Tensor] = None, gather_costs: bool = True, gather_plans: bool = False,
                        group=None, device=None, solve: Optional[Callable] = None, **kwargs) -> dict:
    """Batch-sharded Sinkhorn: rank r solves problems ``shard_range(B, r,
    world)`` of the [B, n, m] cost ``C`` (every rank passes the same full
    batch, on any device; only its own slice is moved to ``device``, by
    default the current CUDA device) with ``dot.sinkhorn(...)``, keyword
    arguments passed through; ``a`` / ``b`` may be 1-D (shared) or [B, n] /
    [B, m].

    Returns ``{"lo", "hi", "plan": local plans [hi-lo, n, m], "cost": local
    costs [hi-lo], "costs": all B costs (if ``gather_costs``), "plans": all B
    plans (if ``gather_plans``)}``.  The gathers are the only collectives and
    carry no gradient; backpropagate through the local ``cost`` / ``plan``.
    ``solve`` replaces ``dot.sinkhorn`` (same signature; for tests of the
    host logic).
    """
    rank, world = _world(group)
    B = C.shape[0]
    lo, hi = shard_range(B, rank, world)
    if solve is None:
        from .sinkhorn import sinkhorn as solve
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    Cl = C[lo:hi].to(dev)
    al = None if a is None else (a if a.dim() == 1 else a[lo:hi]).to(dev)
    bl = None if b is None else (b if b.dim() == 1 else b[lo:hi]).to(dev)
    res = solve(Cl, reg=reg, n_iters=n_iters, a=al, b=bl, **kwargs)
    out = {"lo": lo, "hi": hi, "plan": res.transport_plan, "cost": res.cost}
    if world > 1 and (gather_costs or gather_plans):
        if gather_costs:
            out["costs"] = _gather_batch(res.cost.detach(), B, world, group)
        if gather_plans:
            out["plans"] = _gather_batch(res.transport_plan.detach(), B, world, group)
    else:
        if gather_costs:
            out["costs"] = res.cost.detach()
        if gather_plans:
            out["plans"] = res.transport_plan.detach()
    return out
