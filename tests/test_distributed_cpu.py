"""Multi-rank host logic on CPU: gloo ranks, world size 2.

The GPU path shards rows/images/heads with no collective and finishes a
global sum with one all-reduce of an f64 partial; here the partials come from
the oracle so the partitioning and the all-reduce step run without a GPU.
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from forma_b200.shard import shard_range


def test_shard_range_covers_exactly():
    for total in (0, 1, 7, 65536, 65537):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_range(4, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        from oracle import oracle as orc

        rng = np.random.default_rng(1)
        x = rng.standard_normal((1024, 256)).astype(np.float32)
        b, e = shard_range(x.shape[0], world, rank)
        part = torch.tensor([orc.sum_f64(x[b:e])], dtype=torch.float64)
        dist.all_reduce(part)
        rows = torch.from_numpy(orc.row_reduce(x[b:e], 3))
        gathered = [torch.zeros(shard_range(x.shape[0], world, r)[1] - shard_range(x.shape[0], world, r)[0])
                    for r in range(world)]
        dist.all_gather(gathered, rows)
        if rank == 0:
            q.put((float(part.item()), torch.cat(gathered).numpy().tolist(), orc.sum_f64(x),
                   orc.row_reduce(x, 3).tolist()))
    finally:
        dist.destroy_process_group()


def test_gloo_row_sharding_and_global_sum():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    total, rows, want_total, want_rows = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert abs(total - want_total) <= 1e-9 * max(1.0, abs(want_total))
    assert rows == want_rows
