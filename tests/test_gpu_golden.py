"""GPU outputs against the committed reference fixtures (tests/golden/),
through the C ABI: bit-exact for codes, sums and linear outputs; the dit.c
SwiGLU block within the SwiGLU tolerance of tests/test_gpu_swiglu.py."""
import os
import sys

import numpy as np
import pytest

import iro_b200 as iro

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import inputs  # noqa: E402

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    iro.init(0)
    yield


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def same(a, b):
    a = np.ascontiguousarray(a); b = np.ascontiguousarray(b)
    if a.dtype == np.float32:
        return a.shape == b.shape and bool((a.view(np.uint32) == b.view(np.uint32)).all())
    return a.shape == b.shape and bool((a == b).all())


@pytest.mark.parametrize("idx", range(4))
def test_gpu_matches_reference_int8_ops(idx):
    g = load("int8_ops")
    M, N, K, outlier, w, x, bias = inputs.int8_ops_cases()[idx]
    hw = iro.HostWeight(w)
    assert same(hw.data, g[f"c{idx}_wdata"]) and same(hw.scale, g[f"c{idx}_wscale"])
    assert same(hw.colsum, g[f"c{idx}_wcolsum"])
    q, s, z = iro.quantize_rows(x)
    assert same(q, g[f"c{idx}_q"]) and same(s, g[f"c{idx}_s"]) and same(z, g[f"c{idx}_z"])
    y, work = iro.linear_ex(q, s, z, hw, bias)
    assert same(work, g[f"c{idx}_work"]) and same(y, g[f"c{idx}_y"])


def test_gpu_matches_reference_residual():
    g = load("residual")
    (q1, s1, z1), r, (q2, s2, z2) = iro.quantize_rows_residual(inputs.residual_input())
    for a, name in zip((q1, s1, z1, r, q2, s2, z2), ("q1", "s1", "z1", "r", "q2", "s2", "z2")):
        assert same(a, g[name]), name
    hw = iro.HostWeight(inputs.residual_weight())
    y1, _ = iro.linear_ex(q1, s1, z1, hw)
    y2, _ = iro.linear_ex(q2, s2, z2, hw, None, y=y1, accumulate=True)
    assert same(y2, g["y_two_term"])


def test_gpu_matches_reference_symmetric():
    g = load("sym_quant")
    x = inputs.sym_input()
    M, K = x.shape
    xd = iro.DevBuf.from_host(x)
    q = iro.DevBuf((M, K), np.uint8); s = iro.DevBuf(M, np.float32); z = iro.DevBuf(M, np.int32)
    iro.quantize_rows_dev(xd, M, K, q, s, z, symmetric=True)
    iro.synchronize()
    assert same(q.get(), g["q"]) and same(s.get(), g["s"]) and (z.get() == 128).all()


@pytest.mark.parametrize("mode,residual", [("residual_default", True), ("single_term", False)])
def test_gpu_matches_reference_dit_swiglu(mode, residual):
    g = load("dit_swiglu")
    D, H = (int(v) for v in g["dims"])
    x, w1, w3, w2 = inputs.dit_swiglu_inputs(D, H)
    h1, h3, h2 = iro.HostWeight(w1), iro.HostWeight(w3), iro.HostWeight(w2)
    w13 = iro.DevWeight.gated_pair(h1, h3)
    dw2 = iro.DevWeight.upload(h2)
    out = iro.swiglu_host(x, w13, dw2, residual_w2=residual)
    want = g[mode]
    tol = (1e-4 if residual else 1e-5) * float(np.abs(want).max())
    assert float(np.abs(out - want).max()) <= tol
