"""Whole-request sharding with the library on every rank: two processes
(gloo for the host-side gather, both on cuda:0 -- their kernels never wait on
each other) each run the DiT Euler step of the device library on their own
contiguous block of requests (bench.shard_requests).  The concatenation of
the per-rank states must equal, bit for bit, one process stepping all the
requests: every row's arithmetic is independent of which other requests
share its launch (integer sums, per-row quantisation, attention and the CFG
combine within a request)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")

pytestmark = pytest.mark.gpu

CASE = dict(seed=61, layers=2, R=5, cfg=2, S=40, C=16)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _step(iro, oracle, inputs, lo, hi):
    c = CASE
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(c["seed"], c["layers"], c["R"],
                                                              c["cfg"], c["S"], c["C"])
    dev_blocks = []
    for adaln, qn, kn, ws in blocks:
        W = [oracle.weight_quantize(w) for w in ws]
        dev_blocks.append(iro.DiTBlock(adaln, qn, kn, *[(w.data, w.scale, w.colsum) for w in W]))
    m = iro.DiTModel(dev_blocks, *head.values())
    R = hi - lo
    kd = [iro.DevBuf.from_host(np.ascontiguousarray(k[lo:hi])) for k in ck]
    vd = [iro.DevBuf.from_host(np.ascontiguousarray(v[lo:hi])) for v in cv]
    md = iro.DevBuf.from_host(np.ascontiguousarray(mask[lo * c["cfg"]:hi * c["cfg"]]))
    sd = iro.DevBuf.from_host(np.ascontiguousarray(state[lo:hi]))
    m.euler_step(sd, R, c["cfg"], c["S"], 0.9, 0.775, [1.5], kd, vd, md, c["C"])
    iro.synchronize()
    return sd.get().reshape(R, c["S"], -1)


def _worker(rank, world, port, out_dir):
    for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "irodori-c_b200"), GOLDEN):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from datetime import timedelta
    import bench
    import inputs
    import iro_b200 as iro
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        iro.init(0)
        lo, hi = bench.shard_requests(CASE["R"], world, rank)
        part = _step(iro, oracle, inputs, lo, hi)
        parts = [None] * world
        dist.all_gather_object(parts, part)
        if rank == 0:
            np.save(os.path.join(out_dir, "sharded.npy"), np.concatenate(parts))
    finally:
        dist.destroy_process_group()


def test_two_rank_dit_step_equals_one_process(tmp_path):
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for p in (os.path.join(ROOT, "oracle"), GOLDEN):
        sys.path.insert(0, p)
    import inputs
    import iro_b200 as iro
    import oracle
    iro.init(0)
    whole = _step(iro, oracle, inputs, 0, CASE["R"])
    sharded = np.load(tmp_path / "sharded.npy")
    assert sharded.shape == whole.shape
    assert (sharded.view(np.uint32) == whole.view(np.uint32)).all()
