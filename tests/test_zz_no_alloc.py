"""The allocation-free SwiGLU entry point, iro_int8_swiglu_noalloc_dev.

It exists for callers that cannot allocate device memory where they run the
block: code that records the block into a CUDA graph under global-mode
stream capture (cudaMalloc is not permitted there), engines that reserve all
their device memory at start-up, and latency-critical loops (growing the
library's arena calls cudaFree, which waits for the whole device).  It runs
the same kernels as iro_int8_swiglu_dev on a fixed 64 MiB scratch array
built into the library.

These tests call it through the C ABI and compare it with the allocating
entry point on the same inputs, twice in a row with different inputs (the
second call would expose stale scratch), with the SwiGLU block tolerance of
tests/test_gpu_swiglu.py.  This file is collected last on purpose.
"""
import numpy as np
import pytest

import iro_b200 as iro
import oracle

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-5          # single-term W2, as in tests/test_gpu_swiglu.py
OUT_TOL_RESID = 1e-4    # two-term W2


def _weights(rng, D, H):
    ws = [oracle.weight_quantize((rng.standard_normal(sh) * 0.02).astype(np.float32))
          for sh in ((H, D), (H, D), (D, H))]
    b = [(rng.standard_normal(n) * 0.01).astype(np.float32) for n in (H, H, D)]
    w13 = iro.DevWeight.gated_pair((ws[0].data, ws[0].scale, ws[0].colsum),
                                   (ws[1].data, ws[1].scale, ws[1].colsum), b[0], b[1])
    w2 = iro.DevWeight.upload((ws[2].data, ws[2].scale, ws[2].colsum), b[2])
    return w13, w2


@pytest.mark.parametrize("residual", [False, True])
def test_noalloc_matches_allocating_entry_point_twice(residual):
    iro.init(0)
    M, D, H = 1024, 1024, 2816
    rng = np.random.default_rng(31 if residual else 30)
    w13, w2 = _weights(rng, D, H)
    tol = OUT_TOL_RESID if residual else OUT_TOL
    for call in range(2):
        x = (rng.standard_normal((M, D)) * (1.0 + call)).astype(np.float32)
        xd = iro.DevBuf.from_host(x)
        want = iro.DevBuf((M, D), np.float32)
        got = iro.DevBuf((M, D), np.float32)
        iro.swiglu_dev(xd, M, w13, w2, None, want, residual_w2=residual)
        iro.synchronize()
        # Same stream as the copies that read the result back.
        stream = iro.lib().iro_cuda_stream()
        rc = iro.swiglu_noalloc_dev(xd, M, w13, w2, None, got, residual_w2=residual,
                                    stream=stream)
        assert rc == iro.IRO_OK, rc
        iro.synchronize()
        g, w = got.get(), want.get()
        err = float(np.abs(g - w).max())
        assert err <= tol * float(np.abs(w).max()), f"call {call}: max abs error {err}"


def test_noalloc_rejects_rows_beyond_its_scratch():
    iro.init(0)
    rng = np.random.default_rng(3)
    D, H = 256, 512
    w13, w2 = _weights(rng, D, H)
    M = 100_000  # needs far more than the 64 MiB scratch
    assert iro.swiglu_workspace_bytes(M, D, H) > (64 << 20)
    x = iro.DevBuf((16, D), np.float32)     # never read: the call is rejected first
    out = iro.DevBuf((16, D), np.float32)
    assert iro.swiglu_noalloc_dev(x, M, w13, w2, None, out) == iro.IRO_ERR_UNSUPPORTED
