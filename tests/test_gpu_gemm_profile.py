"""IRO_GEMM_PROFILE on the device path (ops.c:14-110 schema): a child
process with the switch set runs two linear shapes and the gated GEMM a few
times, emits the profile, and one DiT sampling run emits its own record (the
sampler resets and emits, as sampler.c:142-144, 312-321 do).  The JSON lines
must parse, carry the reference's keys, count every launch under its shape,
and report positive device seconds."""
import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

pytestmark = pytest.mark.gpu

CHILD = r"""
import sys, numpy as np
sys.path[:0] = [{root!r} + '/irodori-c_b200', {root!r} + '/oracle', {root!r} + '/tests/golden']
import iro_b200 as iro, oracle, inputs
iro.init(0)
L = iro.lib()
assert L.iro_cuda_gemm_profile_enabled() == 1
rng = np.random.default_rng(1)
def lin(M, N, K, reps):
    w = iro.DevWeight.upload(iro.HostWeight((rng.standard_normal((N, K)) * 0.02).astype(np.float32)))
    x = iro.DevBuf.from_host(rng.standard_normal((M, K)).astype(np.float32))
    q, s, z = iro.DevBuf((M, K), np.uint8), iro.DevBuf(M, np.float32), iro.DevBuf(M, np.int32)
    iro.quantize_rows_dev(x, M, K, q, s, z)
    y = iro.DevBuf((M, N), np.float32)
    for _ in range(reps):
        iro.linear_dev(q, s, z, w, None, y, M)
L.iro_cuda_gemm_profile_reset()
lin(256, 512, 1024, 3)
lin(100, 256, 512, 2)
iro.synchronize()
L.iro_cuda_gemm_profile_emit_json(b"ok", 0, 0, 0)
state, ck, cv, mask, blocks, head = inputs.dit_model_case(5, 1, 1, 2, 24, 8)
dev = []
for adaln, qn, kn, ws in blocks:
    W = [oracle.weight_quantize(w) for w in ws]
    dev.append(iro.DiTBlock(adaln, qn, kn, *[(w.data, w.scale, w.colsum) for w in W]))
m = iro.DiTModel(dev, *head.values())
sd = iro.DevBuf.from_host(state)
m.sample_euler(sd, 1, 2, 24, 2, 1.0, 0.0, 1.0, [1.5], [iro.DevBuf.from_host(k) for k in ck],
               [iro.DevBuf.from_host(v) for v in cv], iro.DevBuf.from_host(mask), 8)
iro.synchronize()
"""


def test_gemm_profile_records_device_gemms():
    env = dict(os.environ, IRO_GEMM_PROFILE="1")
    r = subprocess.run([sys.executable, "-c", CHILD.format(root=ROOT)], env=env,
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    recs = [json.loads(ln) for ln in r.stderr.splitlines() if ln.startswith('{"type":"iro_gemm_profile"')]
    assert len(recs) == 2, r.stderr[-2000:]
    first, sampler = recs
    for rec in recs:
        assert rec["status"] == "ok" and rec["backend"] == "cuda-sm100a-tcgen05-i8"
        assert rec["dropped_shapes"] == 0
        for row in rec["rows"]:
            assert set(row) == {"kind", "M", "N", "K", "lda", "ldb", "ldc", "beta", "backend",
                                "calls", "seconds"}
            assert row["calls"] > 0 and row["seconds"] > 0
    shapes = {(row["kind"], row["M"], row["N"], row["K"]): row["calls"] for row in first["rows"]}
    assert shapes == {("linear_int8", 256, 512, 1024): 3, ("linear_int8", 100, 256, 512): 2}
    assert sampler["steps"] == 2 and sampler["sequence_length"] == 24
    assert sampler["context_tokens"] == 8
    kinds = {row["kind"] for row in sampler["rows"]}
    assert "qkvg_int8" in kinds and "gated_int8" in kinds, kinds
