"""GPU parity of the codec's W8A8 kernel-7 convolution (dacvae.c:543-688)
against the reference fixtures and the CPU oracle, bit-exact.

Full-size check (benchmark config 4: 4 x 48000 frames, 512 -> 512 channels,
kernel 7): the GPU runs the whole batch; the oracle recomputes sampled
windows of output rows.  Each window's input slice is cut out with explicit
zero rows where it crosses the sequence ends.  That is exact: 0 is always
inside a row's range, so a zero row quantises to the zero point and leaves
a remainder code of 128, which is what the reference writes for padding
taps.
"""
import os
import sys

import numpy as np
import pytest

import iro_b200 as iro
import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import inputs  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    iro.init(0)
    yield


def same(a, b):
    return a.shape == b.shape and bool((np.ascontiguousarray(a).view(np.uint32) ==
                                        np.ascontiguousarray(b).view(np.uint32)).all())


def run_gpu(inp, W, kernel, stride, dilation, padding, bias, residual):
    """inp: [batch, T_in, C]."""
    B, T_in, C = inp.shape
    T_out = iro.conv1d_out_len(T_in, kernel, stride, dilation, padding)
    dw = iro.DevWeight.upload((W.data, W.scale, W.colsum))
    xd = iro.DevBuf.from_host(inp)
    bd = iro.DevBuf.from_host(bias) if bias is not None else None
    out = iro.DevBuf((B, T_out, W.N), np.float32)
    rc = iro.conv1d_dev(xd, B, T_in, C, dw, kernel, stride, dilation, padding, bd, residual, out)
    assert rc == T_out
    iro.synchronize()
    return out.get()


@pytest.mark.parametrize("idx", range(4))
def test_conv_matches_reference_fixture(idx):
    g = np.load(os.path.join(GOLDEN, "conv7.npz"))
    case, inp, w, bias = inputs.conv_cases()[idx]
    W = oracle.Weight(g[f"c{idx}_wdata"], g[f"c{idx}_wscale"], g[f"c{idx}_wcolsum"])
    got = run_gpu(inp[None], W, case["kernel"], case["stride"], case["dilation"],
                  case["padding"], bias, case["residual"])[0]
    assert same(got, g[f"c{idx}_out"])


@pytest.mark.parametrize("B,T,C,N,d,stride,res", [
    (2, 300, 96, 64, 1, 1, False), (1, 250, 96, 40, 3, 1, True), (3, 90, 32, 24, 9, 1, True),
    (1, 200, 20, 16, 1, 2, False), (2, 500, 512, 512, 1, 1, False), (1, 160, 512, 512, 3, 1, True),
    (1, 5, 64, 32, 1, 1, True),
    # implicit-GEMM path (stride 1, 512 output channels, C a multiple of 64)
    (1, 300, 64, 512, 1, 1, False), (3, 200, 128, 512, 9, 1, False), (2, 130, 64, 512, 3, 1, False),
    (1, 7, 192, 512, 1, 1, False), (1, 1000, 256, 512, 1, 1, False)])
def test_conv_matches_oracle(B, T, C, N, d, stride, res):
    rng = np.random.default_rng(B * 1000 + T + C + d)
    inp = (rng.standard_normal((B, T, C)) * 0.5).astype(np.float32)
    inp[0, min(3, T - 1)] = 0.0
    W = oracle.weight_quantize((rng.standard_normal((N, 7 * C)) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(N) * 0.01).astype(np.float32)
    pad = 3 * d
    got = run_gpu(inp, W, 7, stride, d, pad, bias, res)
    for b in range(B):
        want = oracle.conv1d_int8(inp[b], W, 7, stride, d, pad, bias, res)
        assert same(got[b], want), f"item {b}"


def _oracle_window(x, W, t0, t1, kernel, dilation, padding, bias, residual):
    """Output rows [t0, t1) of a stride-1 conv of one sequence x [T, C]."""
    T, C = x.shape
    lo = t0 - padding
    hi = (t1 - 1) - padding + (kernel - 1) * dilation + 1
    sub = np.zeros((hi - lo, C), np.float32)
    a, b = max(lo, 0), min(hi, T)
    sub[a - lo:b - lo] = x[a:b]
    out = oracle.conv1d_int8(sub, W, kernel, 1, dilation, 0, bias, residual)
    assert out.shape[0] == t1 - t0
    return out


def test_conv_config4_full_size_sampled_windows():
    B, T, C, N = 4, 48000, 512, 512
    rng = np.random.default_rng(4)
    inp = (rng.standard_normal((B, T, C), dtype=np.float32) * np.float32(0.5))
    W = oracle.weight_quantize((rng.standard_normal((N, 7 * C), dtype=np.float32) * np.float32(0.02)))
    bias = (rng.standard_normal(N, dtype=np.float32) * np.float32(0.01))
    got = run_gpu(inp, W, 7, 1, 1, 3, bias, False)
    assert got.shape == (B, T, N)
    windows = [(0, 64), (T - 64, T), (23990, 24020)]
    for b in range(B):
        for (t0, t1) in windows + [(int(v), int(v) + 16) for v in rng.integers(0, T - 16, 2)]:
            want = _oracle_window(inp[b], W, t0, t1, 7, 1, 3, bias, False)
            assert same(got[b, t0:t1], want), f"item {b} rows {t0}:{t1}"
