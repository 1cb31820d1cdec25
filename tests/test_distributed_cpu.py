"""Host-side logic of the multi-GPU drivers, run as world_size-2 gloo ranks on
CPU: shard ranges, the hand-over of the NCCL id that the row-sharded solver's
communicator is built from, and the batch-sharded solver's split and gathers
(with the CPU oracle standing in for the GPU solve)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dot_b200.distributed import broadcast_unique_id, nccl_communicator, shard_range


def test_shard_range_partitions_exactly():
    for total in (0, 1, 7, 32768, 4097):
        for world in (1, 2, 3, 8):
            spans = [shard_range(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
                assert hi == lo2 and hi >= lo
            sizes = [hi - lo for lo, hi in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(10, 2, 2)


def test_single_rank_needs_no_communicator():
    assert nccl_communicator() is None
    assert broadcast_unique_id(lambda: b"x" * 128) == b"x" * 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))


def _worker_id(rank, world, port, out):
    _init(rank, world, port)
    try:
        calls = []

        def make():
            calls.append(rank)
            return bytes(np.random.default_rng(1234 + rank).integers(0, 256, 128, dtype=np.uint8))

        out[rank] = (broadcast_unique_id(make), list(calls))
    finally:
        dist.destroy_process_group()


def test_unique_id_reaches_every_rank_gloo():
    """Only rank 0 makes the id; every rank receives the same 128 bytes."""
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker_id, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert len(out) == world
    assert out[0][0] == out[1][0] and len(out[0][0]) == 128
    assert out[0][1] == [0] and out[1][1] == []


class _Result:
    def __init__(self, P, cost):
        self.transport_plan = P
        self.cost = cost


def _oracle_solve(C, reg, n_iters, a=None, b=None, **kw):
    from oracle import oracle as O

    B = C.shape[0]
    a2 = None if a is None else (a if a.dim() == 2 else a.expand(B, -1)).numpy()
    b2 = None if b is None else (b if b.dim() == 2 else b.expand(B, -1)).numpy()
    r = O.sinkhorn_api(C.numpy(), reg, n_iters, a2, b2, with_grad=False)
    return _Result(torch.from_numpy(r["P"]), torch.from_numpy(np.asarray(r["cost"], np.float32)))


def _worker_batch(rank, world, port, out):
    from dot_b200.distributed import sinkhorn_batchshard

    _init(rank, world, port)
    try:
        g = torch.Generator().manual_seed(3)
        B, n, m = 5, 9, 7           # 5 problems over 2 ranks: 3 + 2
        C = torch.rand(B, n, m, generator=g)
        b = torch.full((m,), 1.0 / m)
        r = sinkhorn_batchshard(C, reg=0.3, n_iters=15, b=b, gather_plans=True, device="cpu", solve=_oracle_solve)
        out[rank] = (r["lo"], r["hi"], r["costs"].numpy(), r["plans"].numpy(), r["cost"].numpy())
    finally:
        dist.destroy_process_group()


def test_batchshard_splits_and_gathers_gloo():
    """Each rank solves its shard_range slice; the gathered costs and plans
    equal one solve of the whole batch, on every rank, uneven split included."""
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker_batch, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert len(out) == world
    g = torch.Generator().manual_seed(3)
    C = torch.rand(5, 9, 7, generator=g)
    ref = _oracle_solve(C, 0.3, 15)
    assert (out[0][0], out[0][1], out[1][0], out[1][1]) == (0, 3, 3, 5)
    for rank in range(world):
        lo, hi, costs, plans, local = out[rank]
        np.testing.assert_array_equal(costs, ref.cost.numpy())
        np.testing.assert_array_equal(plans, ref.transport_plan.numpy())
        np.testing.assert_array_equal(local, ref.cost.numpy()[lo:hi])
