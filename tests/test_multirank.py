"""Multi-rank host logic on CPU (gloo, world size 2): whole-request sharding
covers every request exactly once, per-rank results computed on the shards
equal the single-process result (rows are independent), and the timing
reduction takes the max over ranks."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, out_dir):
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import torch
    import torch.distributed as dist
    import bench
    import oracle
    from datetime import timedelta
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        n_req, rows_per_req, K, N = 7, 4 * 3, 64, 48
        rng = np.random.default_rng(0)            # same data on every rank
        x = rng.standard_normal((n_req * rows_per_req, K)).astype(np.float32)
        W = oracle.weight_quantize((rng.standard_normal((N, K)) * 0.05).astype(np.float32))
        lo, hi = bench.shard_requests(n_req, world, rank)
        rows = x[lo * rows_per_req:hi * rows_per_req]
        q, s, z = oracle.quantize_rows(rows)
        y, _ = oracle.linear_ex(q, s, z, W)
        sizes = [None] * world
        dist.all_gather_object(sizes, (lo, hi))
        parts = [None] * world
        dist.all_gather_object(parts, y)
        t = bench.max_over_ranks(float(rank + 1) * 0.5, dist)
        if rank == 0:
            np.savez(os.path.join(out_dir, "r.npz"), y=np.concatenate(parts), t=t,
                     cover=np.array([v for (a, b) in sizes for v in range(a, b)]))
    finally:
        dist.destroy_process_group()


def test_two_rank_sharding_is_exact(tmp_path):
    port = _free_port()
    mp.start_processes(_worker, args=(2, port, str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    r = np.load(tmp_path / "r.npz")
    assert list(r["cover"]) == list(range(7))
    assert float(r["t"]) == 1.0
    rng = np.random.default_rng(0)
    x = rng.standard_normal((7 * 12, 64)).astype(np.float32)
    W = oracle.weight_quantize((rng.standard_normal((48, 64)) * 0.05).astype(np.float32))
    q, s, z = oracle.quantize_rows(x)
    y, _ = oracle.linear_ex(q, s, z, W)
    assert (r["y"].view(np.uint32) == y.view(np.uint32)).all()


@pytest.mark.parametrize("n,world", [(1, 8), (8, 8), (64, 8), (5, 2), (512, 4)])
def test_shard_requests_partitions(n, world):
    sys.path.insert(0, ROOT)
    import bench
    got = [bench.shard_requests(n, world, r) for r in range(world)]
    covered = [i for a, b in got for i in range(a, b)]
    assert covered == list(range(n))
    sizes = [b - a for a, b in got]
    assert max(sizes) - min(sizes) <= 1
