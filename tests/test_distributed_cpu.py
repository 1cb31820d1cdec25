"""Host-side logic of the multi-GPU drivers, run as world_size-2 gloo ranks on
CPU: shard ranges, and the exactness of the two-all-reduce combine of
per-rank column (max, sum) partials (the rescale step is stood in for by a
torch expression here; on the GPU it is dot_sinkhorn_col_rescale)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from dot_b200.distributed import combine_column_partials, gather_column_pairs, shard_range


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


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rescale_cpu(col_max, col_sum, gmax):
    col_sum.mul_(torch.exp(col_max - gmax))


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(0)
        n, m = 37, 11
        t = torch.randn(n, m, generator=g, dtype=torch.float64) * 30.0   # wide range: partial maxima differ
        lo, hi = shard_range(n, rank, world)
        local = t[lo:hi]
        cmax = local.max(0).values.float()
        csum = torch.exp(local - local.max(0).values).sum(0).float()
        gmax, gsum = combine_column_partials(cmax, csum, _rescale_cpu)
        lse = (gmax.double() + torch.log(gsum.double()))
        ref = torch.logsumexp(t, dim=0)
        out[rank] = float((lse - ref).abs().max())
    finally:
        dist.destroy_process_group()


def _merge_cpu(gathered):
    """Rank-order merge of gathered (max, sum) pairs [world, m, 2] (the
    arithmetic of dot_sinkhorn_col_merge, in float64 here)."""
    mm = torch.full(gathered.shape[1:-1], -3.4e38, dtype=torch.float64)
    ss = torch.zeros_like(mm)
    for p in gathered.double():
        mn = torch.maximum(mm, p[..., 0])
        ss = ss * torch.exp(mm - mn) + p[..., 1] * torch.exp(p[..., 0] - mn)
        mm = mn
    return mm + torch.log(ss)


def _worker_pairs(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        g = torch.Generator().manual_seed(1)
        n, m = 41, 13
        t = torch.randn(n, m, generator=g, dtype=torch.float64) * 30.0
        lo, hi = shard_range(n, rank, world)
        local = t[lo:hi]
        pairs = torch.stack([local.max(0).values, torch.exp(local - local.max(0).values).sum(0)], -1).float()
        gathered, parts = gather_column_pairs(pairs)
        assert parts == world and tuple(gathered.shape) == (world, m, 2)
        lse = _merge_cpu(gathered)
        out[rank] = (float((lse - torch.logsumexp(t, dim=0)).abs().max()), lse.numpy().tobytes())
    finally:
        dist.destroy_process_group()


def test_gather_column_pairs_two_ranks_gloo():
    """One all-gather of (max, sum) pairs, merged in rank order, gives the
    exact column LSE and the same bits on every rank."""
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker_pairs, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert len(out) == world
    assert max(v[0] for v in out.values()) < 1e-5
    assert out[0][1] == out[1][1]


def test_combine_column_partials_two_ranks_gloo():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert len(out) == world
    assert max(out.values()) < 1e-5
