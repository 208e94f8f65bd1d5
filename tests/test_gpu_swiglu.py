"""GPU parity of the fused int8 SwiGLU block (dit.c:913-969) and its stages.

Stage gates (bit-exact): the W1|W3 dequantised sums before the gate, the
requantisation of a given hidden, and W2 on given codes.  The gate itself,
silu(a) * b = (a / (1 + expf(-a))) * b (ops.c:781-784), calls expf, which is
not bit-identical between the GPU's expf and the host libm, so the hidden is
gated at HIDDEN_ULPS units in the last place and the block output at
OUT_TOL relative to the output's max magnitude (single-term W2) and
OUT_TOL_RESID with the two-term W2 (its second term codes a remainder that
is small by construction, so ulp flips in the hidden move it further).
"""
import numpy as np
import pytest

import iro_b200 as iro
import oracle

pytestmark = pytest.mark.gpu

HIDDEN_ULPS = 4
OUT_TOL = 1e-5
OUT_TOL_RESID = 1e-4


@pytest.fixture(scope="module", autouse=True)
def device():
    iro.init(0)
    yield


def ulp_diff(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def make_block(seed, M, D, H, bias=True, x_scale=1.0):
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((M, D)) * x_scale).astype(np.float32)
    ws = [oracle.weight_quantize((rng.standard_normal(sh) * 0.02).astype(np.float32))
          for sh in ((H, D), (H, D), (D, H))]
    bs = [(rng.standard_normal(n) * 0.01).astype(np.float32) if bias else None
          for n in (H, H, D)]
    return x, ws, bs


def upload(ws, bs):
    w1, w3, w2 = ws
    b1, b3, b2 = bs
    w13 = iro.DevWeight.gated_pair((w1.data, w1.scale, w1.colsum), (w3.data, w3.scale, w3.colsum),
                                   b1, b3)
    dw2 = iro.DevWeight.upload((w2.data, w2.scale, w2.colsum), b2)
    return w13, dw2


@pytest.mark.parametrize("M,D,H,x_scale", [(64, 1024, 2816, 1.0), (300, 1280, 3680, 1.0),
                                           (2048, 1024, 2816, 1.0), (5, 256, 200, 1.0),
                                           (256, 1024, 2816, 60.0)])
def test_gated_hidden(M, D, H, x_scale):
    """x_scale 60 spreads the gate inputs over roughly +-100, through the
    overflow of e^-a (a < -88.7) and the flush of e^-a to 0 (a > 87)."""
    x, ws, bs = make_block(M + H, M, D, H, x_scale=x_scale)
    w13, _ = upload(ws, bs)
    q, s, z = oracle.quantize_rows(x)
    qd, sd, zd = iro.DevBuf.from_host(q), iro.DevBuf.from_host(s), iro.DevBuf.from_host(z)
    hid = iro.DevBuf((M, H), np.float32)
    iro.gated_dev(qd, sd, zd, w13, hid, M)
    iro.synchronize()
    a1, _ = oracle.linear_ex(q, s, z, ws[0], bs[0])
    a3, _ = oracle.linear_ex(q, s, z, ws[1], bs[1])
    want = oracle.silu_mul(a1, a3)
    got = hid.get()
    u = ulp_diff(got, want)
    assert u.max() <= HIDDEN_ULPS, f"hidden differs by {u.max()} ulp"
    # With the gate inputs bit-exact, only expf can move the hidden: check the
    # gate inputs through the plain linear on the same codes.
    dw1 = iro.DevWeight.upload((ws[0].data, ws[0].scale, ws[0].colsum))
    y1 = iro.DevBuf((M, H), np.float32)
    b1d = iro.DevBuf.from_host(bs[0])
    iro.linear_dev(qd, sd, zd, dw1, b1d, y1, M)
    iro.synchronize()
    assert (y1.get().view(np.uint32) == a1.view(np.uint32)).all()


def test_requant_of_hidden_is_byte_exact():
    """Given the GPU hidden, the GPU requantisation equals the oracle's."""
    M, D, H = 256, 1024, 2816
    x, ws, bs = make_block(7, M, D, H)
    w13, _ = upload(ws, bs)
    q, s, z = oracle.quantize_rows(x)
    qd, sd, zd = iro.DevBuf.from_host(q), iro.DevBuf.from_host(s), iro.DevBuf.from_host(z)
    hid = iro.DevBuf((M, H), np.float32)
    iro.gated_dev(qd, sd, zd, w13, hid, M)
    qh = iro.DevBuf((M, H), np.uint8); sh = iro.DevBuf(M, np.float32)
    zh = iro.DevBuf(M, np.int32)
    iro.quantize_rows_dev(hid, M, H, qh, sh, zh)
    iro.synchronize()
    oq, os_, oz = oracle.quantize_rows(hid.get())
    assert (qh.get() == oq).all() and (sh.get().view(np.uint32) == os_.view(np.uint32)).all()
    assert (zh.get() == oz).all()


@pytest.mark.parametrize("M,D,H", [(2048, 1024, 2816), (300, 1280, 3680), (1, 1024, 2816)])
@pytest.mark.parametrize("residual", [False, True])
def test_swiglu_block(M, D, H, residual):
    x, ws, bs = make_block(M * 3 + H, M, D, H)
    w13, dw2 = upload(ws, bs)
    xd = iro.DevBuf.from_host(x)
    out = iro.DevBuf((M, D), np.float32)
    iro.swiglu_dev(xd, M, w13, dw2, None, out, residual_w2=residual)
    iro.synchronize()
    want = oracle.swiglu(x, *ws, *bs, residual_w2=residual)
    got = out.get()
    tol = (OUT_TOL_RESID if residual else OUT_TOL) * float(np.abs(want).max())
    err = float(np.abs(got - want).max())
    assert err <= tol, f"max abs error {err} > {tol}"
    # host-pointer form of the same block
    got_h = iro.swiglu_host(x, w13, dw2, residual_w2=residual)
    assert (got_h.view(np.uint32) == got.view(np.uint32)).all()


def test_swiglu_caller_workspace_matches_arena():
    M, D, H = 512, 1024, 2816
    x, ws, bs = make_block(99, M, D, H)
    w13, dw2 = upload(ws, bs)
    xd = iro.DevBuf.from_host(x)
    o1 = iro.DevBuf((M, D), np.float32); o2 = iro.DevBuf((M, D), np.float32)
    wsb = iro.DevBuf(iro.swiglu_workspace_bytes(M, D, H, True), np.uint8)
    iro.swiglu_dev(xd, M, w13, dw2, None, o1, residual_w2=True)
    iro.swiglu_dev(xd, M, w13, dw2, None, o2, residual_w2=True, workspace=wsb)
    iro.synchronize()
    assert (o1.get().view(np.uint32) == o2.get().view(np.uint32)).all()


def test_swiglu_host_pinned_pipelined_matches_device():
    """With page-locked host buffers iro_int8_swiglu runs the block in row
    chunks with the copies overlapped; rows are independent, so the result is
    bit-identical to one device-pointer call."""
    import ctypes as C
    M, D, H = 2048, 1024, 2816
    x, ws, bs = make_block(123, M, D, H)
    w13, dw2 = upload(ws, bs)
    L = iro.lib()
    px, po = L.iro_host_alloc_pinned(M * D * 4), L.iro_host_alloc_pinned(M * D * 4)
    try:
        xp = np.ctypeslib.as_array((C.c_float * (M * D)).from_address(px)).reshape(M, D)
        op = np.ctypeslib.as_array((C.c_float * (M * D)).from_address(po)).reshape(M, D)
        xp[:] = x
        iro.check(L.iro_int8_swiglu(iro._p(xp), M, C.byref(w13.st), C.byref(dw2.st), None,
                                    iro._p(op), 0), "iro_int8_swiglu")
        xd = iro.DevBuf.from_host(x)
        out = iro.DevBuf((M, D), np.float32)
        iro.swiglu_dev(xd, M, w13, dw2, None, out)
        iro.synchronize()
        assert (op.view(np.uint32) == out.get().view(np.uint32)).all()
    finally:
        L.iro_host_free_pinned(px)
        L.iro_host_free_pinned(po)


@pytest.mark.parametrize("residual", [False, True])
def test_swiglu_plan_replays_the_block(residual):
    """A recorded plan (CUDA graph) gives the block's result bit-for-bit, and
    reads the input buffer afresh at every launch."""
    M, D, H = 1024, 1024, 2816
    x, ws, bs = make_block(55, M, D, H)
    w13, dw2 = upload(ws, bs)
    xd = iro.DevBuf.from_host(x)
    out = iro.DevBuf((M, D), np.float32)
    plan = iro.Plan(xd, M, w13, dw2, None, out, residual_w2=residual)
    ref = iro.DevBuf((M, D), np.float32)
    for step in range(2):
        xs = (x * (1.0 + step)).astype(np.float32)
        xd.upload(xs)
        plan.launch()
        iro.synchronize()
        iro.swiglu_dev(xd, M, w13, dw2, None, ref, residual_w2=residual)
        iro.synchronize()
        assert (out.get().view(np.uint32) == ref.get().view(np.uint32)).all(), f"step {step}"
    plan.free()


def test_swiglu_pipe_submits_overlap_and_match():
    """The submit/wait pipeline: several steps in flight on a 2-slot ring,
    each result bit-identical to a device-pointer call on the same input."""
    M, D, H = 1024, 1024, 2816
    x, ws, bs = make_block(77, M, D, H)
    w13, dw2 = upload(ws, bs)
    import torch
    pipe = iro.SwigluPipe(M, w13, dw2, depth=2)
    xs = [torch.empty((M, D), dtype=torch.float32, pin_memory=True) for _ in range(5)]
    outs = [torch.empty((M, D), dtype=torch.float32, pin_memory=True) for _ in range(5)]
    for i in range(5):
        xs[i].numpy()[:] = x * (1.0 + 0.25 * i)
        pipe.submit(xs[i].numpy(), outs[i].numpy())
    pipe.wait()
    xd = iro.DevBuf((M, D), np.float32)
    ref = iro.DevBuf((M, D), np.float32)
    for i in range(5):
        xd.upload(xs[i].numpy())
        iro.swiglu_dev(xd, M, w13, dw2, None, ref)
        iro.synchronize()
        assert (outs[i].numpy().view(np.uint32) == ref.get().view(np.uint32)).all(), f"step {i}"
    pipe.free()
