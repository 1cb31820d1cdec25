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

from dot_b200.distributed import combine_column_partials, shard_range


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


def test_combine_column_partials_two_ranks_gloo():
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.start_processes(_worker, args=(world, _free_port(), out), nprocs=world, join=True, start_method="spawn")
    assert len(out) == world
    assert max(out.values()) < 1e-5
