"""The allocation-free SwiGLU entry point, iro_int8_swiglu_noalloc_dev.

It exists for callers that cannot allocate device memory where they run the
block: engines that reserve their whole memory budget at start-up and treat
a later allocation as a failure, hosts whose device memory belongs to another
allocator, and latency-critical loops (growing the library's arena calls
cudaFree, which waits for the whole device).  It runs the same kernels as
iro_int8_swiglu_dev on a fixed 64 MiB scratch array built into the library.

These tests call it through the C ABI, twice in a row with different inputs
(the second call would expose stale scratch), and require its output to be
bit-identical to the allocating entry point's on the same inputs: both run
the same kernels, so any difference is a bug.  Each call is also held to
the SwiGLU block bar of tests/test_gpu_swiglu.py against the CPU oracle on
a row sample.  This file is collected last on purpose.
"""
import numpy as np
import pytest

import iro_b200 as iro
import oracle

pytestmark = pytest.mark.gpu

OUT_TOL = 1e-5          # single-term W2 block vs the oracle (tests/test_gpu_swiglu.py)
OUT_TOL_RESID = 1e-4    # two-term W2


def _weights(rng, D, H):
    ws = [oracle.weight_quantize((rng.standard_normal(sh) * 0.02).astype(np.float32))
          for sh in ((H, D), (H, D), (D, H))]
    b = [(rng.standard_normal(n) * 0.01).astype(np.float32) for n in (H, H, D)]
    w13 = iro.DevWeight.gated_pair((ws[0].data, ws[0].scale, ws[0].colsum),
                                   (ws[1].data, ws[1].scale, ws[1].colsum), b[0], b[1])
    w2 = iro.DevWeight.upload((ws[2].data, ws[2].scale, ws[2].colsum), b[2])
    return w13, w2, ws, b


@pytest.mark.parametrize("residual", [False, True])
def test_noalloc_matches_allocating_entry_point_twice(residual):
    iro.init(0)
    M, D, H = 1024, 1024, 2816
    rng = np.random.default_rng(31 if residual else 30)
    w13, w2, ws, b = _weights(rng, D, H)
    tol = OUT_TOL_RESID if residual else OUT_TOL
    # The caller's own stream (here the library stream, which the copies
    # that read the results back also use).
    stream = iro.lib().iro_cuda_stream()
    for call in range(2):
        x = (rng.standard_normal((M, D)) * (1.0 + call)).astype(np.float32)
        xd = iro.DevBuf.from_host(x)
        want = iro.DevBuf((M, D), np.float32)
        got = iro.DevBuf((M, D), np.float32)
        got.fill_byte(0xFF)  # NaN pattern: every output element must be written
        iro.swiglu_dev(xd, M, w13, w2, None, want, residual_w2=residual)
        iro.synchronize()
        rc = iro.swiglu_noalloc_dev(xd, M, w13, w2, None, got, residual_w2=residual,
                                    stream=stream)
        assert rc == iro.IRO_OK, rc
        assert iro.lib().iro_cuda_synchronize(stream) == iro.IRO_OK
        g, w = got.get(), want.get()
        assert (g.view(np.uint32) == w.view(np.uint32)).all(), f"call {call}: not bit-identical"
        rows = np.r_[0:24, M - 24:M]
        ref = oracle.swiglu(x[rows], *ws, *b, residual_w2=residual)
        err = float(np.abs(g[rows] - ref).max())
        assert err <= tol * float(np.abs(ref).max()), f"call {call}: max abs error {err}"


def test_noalloc_rejects_rows_beyond_its_scratch():
    iro.init(0)
    rng = np.random.default_rng(3)
    D, H = 256, 512
    w13, w2, _, _ = _weights(rng, D, H)
    M = 100_000  # needs far more than the 64 MiB scratch
    assert iro.swiglu_workspace_bytes(M, D, H) > (64 << 20)
    x = iro.DevBuf((16, D), np.float32)     # never read: the call is rejected first
    out = iro.DevBuf((16, D), np.float32)
    assert iro.swiglu_noalloc_dev(x, M, w13, w2, None, out) == iro.IRO_ERR_UNSUPPORTED


def test_noalloc_timeouts_surface_through_synchronize():
    """The no-allocation path's kernels report into the device's one error
    word, the same word the bounded-wait probe records its timeout in.  The
    probe's report must come back from iro_cuda_synchronize exactly once,
    and the no-allocation path must keep working afterwards."""
    iro.init(0)
    rng = np.random.default_rng(5)
    D, H, M = 256, 512, 96
    w13, w2, _, _ = _weights(rng, D, H)
    x = iro.DevBuf.from_host(rng.standard_normal((M, D)).astype(np.float32))
    want = iro.DevBuf((M, D), np.float32)
    got = iro.DevBuf((M, D), np.float32)
    stream = iro.lib().iro_cuda_stream()
    iro.swiglu_dev(x, M, w13, w2, None, want)
    assert iro.swiglu_noalloc_dev(x, M, w13, w2, None, got, stream=stream) == iro.IRO_OK
    assert iro.lib().iro_cuda_synchronize(stream) == iro.IRO_OK
    # A 20 ms wait that nothing completes: the probe returns the timeout it
    # read through iro_cuda_synchronize, which clears the word.
    assert iro.lib().iro_debug_bounded_wait_probe(20_000_000) == iro.IRO_ERR_DEVICE_TIMEOUT
    got.fill_byte(0xFF)
    assert iro.swiglu_noalloc_dev(x, M, w13, w2, None, got, stream=stream) == iro.IRO_OK
    assert iro.lib().iro_cuda_synchronize(stream) == iro.IRO_OK
    assert (got.get().view(np.uint32) == want.get().view(np.uint32)).all()


def test_noalloc_records_under_global_stream_capture():
    """The point of the entry point: after one warm-up call it can be
    recorded into a CUDA graph under global-mode stream capture (which fails
    on any allocation, synchronisation or other non-capturable call made while
    the capture is open), and the replayed graph writes the same bits as the
    allocating entry point."""
    import ctypes
    import torch

    iro.init(0)
    M, D, H = 512, 1024, 2816
    rng = np.random.default_rng(32)
    w13, w2, _, _ = _weights(rng, D, H)
    xd = iro.DevBuf.from_host(rng.standard_normal((M, D)).astype(np.float32))
    want = iro.DevBuf((M, D), np.float32)
    got = iro.DevBuf((M, D), np.float32)
    iro.swiglu_dev(xd, M, w13, w2, None, want)
    iro.synchronize()
    cap = torch.cuda.Stream()
    handle = ctypes.c_void_p(cap.cuda_stream)
    assert iro.swiglu_noalloc_dev(xd, M, w13, w2, None, got, stream=handle) == iro.IRO_OK
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap, capture_error_mode="global"):
        rc = iro.swiglu_noalloc_dev(xd, M, w13, w2, None, got, stream=handle)
    assert rc == iro.IRO_OK, rc
    got.fill_byte(0xFF)
    iro.synchronize()
    graph.replay()
    torch.cuda.synchronize()
    assert iro.lib().iro_cuda_synchronize(None) == iro.IRO_OK
    g, w = got.get(), want.get()
    assert (g.view(np.uint32) == w.view(np.uint32)).all()
    del graph
