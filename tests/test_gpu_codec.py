"""GPU parity of the codec's transposed (upsampling) convolution
(dacvae.c:696-790) and of the residual unit's skip + 1x1 projection
(dacvae.c:979-1009) against the reference fixtures and the CPU oracle,
bit-exact.

The transposed convolution at decoder scale is checked through windows: an
output row's value depends only on the input rows whose taps reach it
(bias + their expanded rows, added in input-row order), and each input row
is quantised on its own, so the oracle run on an input slice reproduces
every output row whose contributing rows all lie inside the slice.
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


def run_convt(inp, W, C_out, kernel, stride, padding, output_padding, bias, residual):
    """inp: [batch, T_in, C_in] -> [batch, T_out, C_out]."""
    B, T_in, C_in = inp.shape
    T_out = iro.convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding)
    dw = iro.DevWeight.upload((W.data, W.scale, W.colsum))
    xd = iro.DevBuf.from_host(inp)
    bd = iro.DevBuf.from_host(bias) if bias is not None else None
    out = iro.DevBuf((B, T_out, C_out), np.float32)
    rc = iro.convtranspose1d_dev(xd, B, T_in, C_in, dw, C_out, kernel, stride, padding,
                                 output_padding, bd, residual, out)
    assert rc == T_out
    iro.synchronize()
    return out.get()


def decoder_geometry(stride):
    return 2 * stride, (stride + 1) // 2, stride & 1


@pytest.mark.parametrize("idx", range(5))
@pytest.mark.parametrize("mode", ["single", "two_term"])
def test_convt_matches_reference_fixture(idx, mode):
    g = np.load(os.path.join(GOLDEN, "convt.npz"))
    case, inp, w, bias = inputs.convt_cases()[idx]
    W = oracle.Weight(g[f"c{idx}_wdata"], g[f"c{idx}_wscale"], g[f"c{idx}_wcolsum"])
    got = run_convt(inp[None], W, case["C_out"], case["kernel"], case["stride"],
                    case["padding"], case["output_padding"], bias, mode == "two_term")[0]
    assert same(got, g[f"c{idx}_{mode}"])


@pytest.mark.parametrize("B,T,Cin,Cout,stride,res", [
    (2, 40, 1536, 768, 12, False), (2, 30, 768, 384, 10, True), (1, 200, 384, 192, 8, False),
    (3, 500, 192, 96, 2, True), (2, 1, 64, 16, 4, False), (1, 77, 32, 10, 3, True)])
def test_convt_matches_oracle(B, T, Cin, Cout, stride, res):
    rng = np.random.default_rng(B * 7919 + T + Cin + stride)
    k, p, op = decoder_geometry(stride)
    inp = (rng.standard_normal((B, T, Cin)) * 0.5).astype(np.float32)
    inp[0, min(2, T - 1)] = 0.0
    W = oracle.weight_quantize((rng.standard_normal((k * Cout, Cin)) * 0.03).astype(np.float32))
    bias = (rng.standard_normal(Cout) * 0.01).astype(np.float32)
    got = run_convt(inp, W, Cout, k, stride, p, op, bias, res)
    for b in range(B):
        want = oracle.convtranspose1d_int8(inp[b], W, Cout, k, stride, p, op, bias, res)
        assert same(got[b], want), f"item {b}"


def test_convt_without_bias_starts_from_zero():
    rng = np.random.default_rng(5)
    inp = rng.standard_normal((1, 33, 48)).astype(np.float32)
    W = oracle.weight_quantize((rng.standard_normal((6 * 8, 48)) * 0.05).astype(np.float32))
    got = run_convt(inp, W, 8, 6, 3, 2, 1, None, False)[0]
    want = oracle.convtranspose1d_int8(inp[0], W, 8, 6, 3, 2, 1, np.zeros(8, np.float32), False)
    assert same(got, want)


def _convt_window(x, W, C_out, kernel, stride, padding, r0, r1, bias, residual):
    """Output rows fully determined by input rows [r0, r1), with their
    global indices."""
    sub = oracle.convtranspose1d_int8(x[r0:r1], W, C_out, kernel, stride, padding, 0, bias,
                                      residual)
    # Global output row ot takes input rows r with r*s - p <= ot <= r*s - p + k - 1.
    lo = r0 * stride - padding + kernel - 1 if r0 > 0 else 0
    hi = (r1 - 1) * stride - padding + 1
    rows = [ot for ot in range(max(lo, 0), hi) if ot - r0 * stride >= 0]
    return rows, {ot: sub[ot - r0 * stride] for ot in rows}


def test_convt_stage1_chunk_boundary_windows():
    """Decoder stage 1 (1536 -> 768, stride 12): 4000 input rows take two
    workspace chunks; windows around the chunk boundary and the ends."""
    T, Cin, Cout, s = 4000, 1536, 768, 12
    k, p, op = decoder_geometry(s)
    rng = np.random.default_rng(12)
    inp = (rng.standard_normal((1, T, Cin), dtype=np.float32) * np.float32(0.5))
    W = oracle.weight_quantize((rng.standard_normal((k * Cout, Cin), dtype=np.float32) *
                                np.float32(0.02)))
    bias = (rng.standard_normal(Cout, dtype=np.float32) * np.float32(0.01))
    got = run_convt(inp, W, Cout, k, s, p, op, bias, False)[0]
    assert got.shape == (T * s, Cout)
    checked = 0
    for (r0, r1) in [(0, 12), (3570, 3600), (1990, 2005), (T - 12, T)]:
        rows, want = _convt_window(inp[0], W, Cout, k, s, p, r0, r1, bias, False)
        for ot in rows:
            if ot < got.shape[0]:
                assert same(got[ot], want[ot]), f"output row {ot}"
                checked += 1
    assert checked > 500


@pytest.mark.parametrize("mode", ["single", "two_term"])
def test_conv1_matches_reference_fixture(mode):
    g = np.load(os.path.join(GOLDEN, "conv1.npz"))
    hidden, skip, w, bias = inputs.conv1_case()
    W = oracle.Weight(g["wdata"], g["wscale"], g["wcolsum"])
    dw = iro.DevWeight.upload((W.data, W.scale, W.colsum))
    rows, C = hidden.shape
    hd = iro.DevBuf.from_host(hidden)
    sd = iro.DevBuf.from_host(skip)
    bd = iro.DevBuf.from_host(bias)
    out = iro.DevBuf((rows, C), np.float32)
    iro.codec_conv1_dev(hd, rows, dw, bd, sd, mode == "two_term", out)
    iro.synchronize()
    assert same(out.get(), g[f"out_{mode}"])


@pytest.mark.parametrize("rows,C,res,inplace", [
    (3000, 768, False, False), (3000, 768, True, True), (1000, 96, True, False),
    (130, 192, False, True), (1, 384, True, False)])
def test_conv1_matches_oracle(rows, C, res, inplace):
    rng = np.random.default_rng(rows + C)
    hidden = rng.standard_normal((rows, C)).astype(np.float32)
    skip = (rng.standard_normal((rows, C)) * 0.3).astype(np.float32)
    W = oracle.weight_quantize((rng.standard_normal((C, C)) * 0.03).astype(np.float32))
    bias = (rng.standard_normal(C) * 0.01).astype(np.float32)
    dw = iro.DevWeight.upload((W.data, W.scale, W.colsum))
    hd = iro.DevBuf.from_host(hidden)
    sd = iro.DevBuf.from_host(skip)
    bd = iro.DevBuf.from_host(bias)
    out = sd if inplace else iro.DevBuf((rows, C), np.float32)
    iro.codec_conv1_dev(hd, rows, dw, bd, sd, res, out)
    iro.synchronize()
    want = oracle.codec_conv1(hidden, W, bias, skip, res)
    assert same(out.get(), want)
