"""A step split across ranks by CFG branch (fewer requests than GPUs: one
request's CFG rows sharded across the ranks): each rank runs
iro_dit_velocity_dev on its own branches (their mask rows), the velocities
meet by an all-gather in branch order, and iro_dit_cfg_update_dev applies
the guided Euler update (sampler.c:283-297).  Two gloo ranks share cuda:0
(their kernels never wait on each other); the result must equal one
iro_dit_euler_step_dev over all branches bit for bit, and so must the
single-process velocity + update pair."""
import os
import socket
import sys

import numpy as np
import pytest
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")

pytestmark = pytest.mark.gpu

CASE = dict(seed=83, layers=2, R=1, cfg=4, S=48, C=16)
T, TN, SCALES = 0.875, 0.75, [2.0, 1.5, 1.0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _model(iro, oracle, inputs):
    c = CASE
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(c["seed"], c["layers"], c["R"],
                                                              c["cfg"], c["S"], c["C"])
    dev = []
    for adaln, qn, kn, ws in blocks:
        W = [oracle.weight_quantize(w) for w in ws]
        dev.append(iro.DiTBlock(adaln, qn, kn, *[(w.data, w.scale, w.colsum) for w in W]))
    m = iro.DiTModel(dev, *head.values())
    kd = [iro.DevBuf.from_host(k) for k in ck]
    vd = [iro.DevBuf.from_host(v) for v in cv]
    return m, state, kd, vd, mask


def _velocity(iro, m, state, kd, vd, mask, branches):
    c = CASE
    md = iro.DevBuf.from_host(np.ascontiguousarray(mask[branches]))
    vel = iro.DevBuf((len(branches), c["S"], 32), np.float32)
    m.velocity(iro.DevBuf.from_host(state), 1, len(branches), c["S"], T, kd, vd, md, c["C"], vel)
    iro.synchronize()
    return vel.get()


def _worker(rank, world, port, out_dir):
    for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "irodori-c_b200"), GOLDEN):
        sys.path.insert(0, p)
    import torch.distributed as dist
    from datetime import timedelta
    import inputs
    import iro_b200 as iro
    import oracle
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        iro.init(0)
        m, state, kd, vd, mask = _model(iro, oracle, inputs)
        mine = [b for b in range(CASE["cfg"]) if b % world == rank]
        v = _velocity(iro, m, state, kd, vd, mask, mine)
        parts = [None] * world
        dist.all_gather_object(parts, (mine, v))
        if rank == 0:
            full = np.empty((CASE["cfg"], CASE["S"], 32), np.float32)
            for bs, vv in parts:
                for i, b in enumerate(bs):
                    full[b] = vv[i]
            sd = iro.DevBuf.from_host(state)
            m.cfg_update(sd, iro.DevBuf.from_host(full), 1, CASE["cfg"], CASE["S"], T, TN, SCALES)
            iro.synchronize()
            np.save(os.path.join(out_dir, "split.npy"), sd.get())
    finally:
        dist.destroy_process_group()


def test_cfg_branch_split_equals_one_step(tmp_path):
    mp.start_processes(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True,
                       start_method="spawn")
    for p in (os.path.join(ROOT, "oracle"), GOLDEN):
        sys.path.insert(0, p)
    import inputs
    import iro_b200 as iro
    import oracle
    iro.init(0)
    m, state, kd, vd, mask = _model(iro, oracle, inputs)
    sd = iro.DevBuf.from_host(state)
    m.euler_step(sd, 1, CASE["cfg"], CASE["S"], T, TN, SCALES, kd, vd, iro.DevBuf.from_host(mask),
                 CASE["C"])
    iro.synchronize()
    whole = sd.get()
    # Velocity + update in one process.
    v = _velocity(iro, m, state, kd, vd, mask, list(range(CASE["cfg"])))
    sd2 = iro.DevBuf.from_host(state)
    m.cfg_update(sd2, iro.DevBuf.from_host(v), 1, CASE["cfg"], CASE["S"], T, TN, SCALES)
    iro.synchronize()
    assert (sd2.get().view(np.uint32) == whole.view(np.uint32)).all()
    split = np.load(tmp_path / "split.npy")
    assert (split.view(np.uint32) == whole.view(np.uint32)).all()
