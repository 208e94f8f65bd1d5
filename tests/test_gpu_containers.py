"""The device int8 model containers (iro_dit_int8_dev_upload,
iro_dacvae_int8_dev_upload): built from host copies laid out as the
reference's IroDiTInt8 / IroDACVAEInt8, their `bytes` is the sum of the
members' device payloads, and a DiT block / codec conv run on a container's
weights is bit-identical to the same call on separately uploaded weights."""
import ctypes as C
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


def _host(w):
    return iro.HostWeight.from_arrays(w.data, w.scale, w.colsum)


def test_dit_container_matches_separate_uploads():
    iro.init(0)
    L = iro.lib()
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(12, 2, 1, 2, 40, 16)
    keep, layers = [], (iro.IroDiTInt8HostLayer * 2)()
    for li, (adaln, qn, kn, ws) in enumerate(blocks):
        hw = [_host(oracle.weight_quantize(w)) for w in ws]
        keep.append(hw)
        for name, h in zip(("wq", "wk", "wv", "gate", "wo", "w1", "w3", "w2"), hw):
            setattr(layers[li], name, h.st)
    cont = iro.IroDiTInt8Dev()
    assert L.iro_dit_int8_dev_upload(C.byref(cont), layers, 2) == iro.IRO_OK
    assert cont.layers == 2
    parts = [getattr(cont.layer[li], n) for li in range(2) for n in ("qkvg", "wo", "w13", "w2")]
    assert cont.bytes == sum(L.iro_int8_dev_weight_bytes(C.byref(p)) for p in parts)
    D, H = 1280, 3680
    expect = 0
    Hp = (H + 127) // 128 * 128  # the W1|W3 pair layout pads H to whole 128-row blocks
    for n, k in ((4 * D, D), (D, D), (2 * Hp, D), (D, H)):
        expect += n * ((k + 15) // 16 * 16) + 8 * n
    assert cont.bytes == 2 * expect
    # Layer 0 through the container's weights vs a block built separately.
    adaln, qn, kn, _ = blocks[0]
    blk = iro.DiTBlock(adaln, qn, kn, *keep[0])
    st = iro.IroDiTBlockDev.from_buffer_copy(blk.st)
    st.qkvg, st.wo, st.w13, st.w2 = (cont.layer[0].qkvg, cont.layer[0].wo, cont.layer[0].w13,
                                     cont.layer[0].w2)
    rng = np.random.default_rng(4)
    x = rng.standard_normal((2 * 40, D)).astype(np.float32)
    cond = iro.DevBuf.from_host((rng.standard_normal((1, 3 * D)) * 0.5).astype(np.float32))
    kd, vd = iro.DevBuf.from_host(ck[0]), iro.DevBuf.from_host(cv[0])
    md = iro.DevBuf.from_host(mask)
    rc, rs = iro.dit_rope_table(40)
    rcd, rsd = iro.DevBuf.from_host(rc), iro.DevBuf.from_host(rs)
    outs = []
    for s_ in (blk.st, st):
        xd = iro.DevBuf.from_host(x)
        iro.check(L.iro_dit_block_dev(C.byref(s_), iro._p(xd), iro._p(cond), 1, iro._p(kd),
                                      iro._p(vd), iro._p(md), 1, 2, 40, 16, iro._p(rcd),
                                      iro._p(rsd), None, None), "dit_block_dev")
        iro.synchronize()
        outs.append(xd.get())
    assert (outs[0].view(np.uint32) == outs[1].view(np.uint32)).all()
    L.iro_dit_int8_dev_free(C.byref(cont))
    assert cont.bytes == 0 and not cont.layer[0].qkvg.data


def test_dacvae_container_matches_separate_uploads():
    iro.init(0)
    L = iro.lib()
    rng = np.random.default_rng(8)
    C_ = 64
    qw = lambda n, k: oracle.weight_quantize((rng.standard_normal((n, k)) * 0.02)  # noqa: E731
                                             .astype(np.float32))
    host = iro.IroDACVAEInt8Host()
    keep = []

    def put(field_owner, name, w):
        h = _host(w)
        keep.append(h)
        setattr(field_owner, name, h.st)

    put(host, "initial", qw(C_, 7 * C_))
    for s in range(4):
        put(host.stage[s], "upsample", qw(2 * 2 * C_, C_))
        for r in range(3):
            put(host.stage[s].residual[r], "conv0", qw(C_, 7 * C_))
            put(host.stage[s].residual[r], "conv1", qw(C_, C_))
    cont = iro.IroDACVAEInt8Dev()
    assert L.iro_dacvae_int8_dev_upload(C.byref(cont), C.byref(host)) == iro.IRO_OK
    expect = (C_ * 7 * C_ + 8 * C_) * 13 + (C_ * C_ + 8 * C_) * 12 + (4 * C_ * C_ + 32 * C_) * 4
    assert cont.bytes == expect
    # The stage-2 unit-1 kernel-7 conv from the container vs a separate upload.
    inp = (rng.standard_normal((2, 50, C_)) * 0.5).astype(np.float32)
    xd = iro.DevBuf.from_host(inp)
    # keep: initial, then per stage upsample and (conv0, conv1) x 3.
    k = keep[1 + 2 * 7 + 1 + 2 * 1]
    sep = iro.DevWeight.upload((k.data, k.scale, k.colsum))
    outs = []
    for w in (sep.st, cont.stage[2].residual[1].conv0):
        out = iro.DevBuf((2, 50, C_), np.float32)
        rc = L.iro_int8_conv1d_dev(iro._p(xd), 2, 50, C_, C.byref(w), 7, 1, 1, 3, None, 0,
                                   iro._p(out), None)
        assert rc == 50
        iro.synchronize()
        outs.append(out.get())
    assert (outs[0].view(np.uint32) == outs[1].view(np.uint32)).all()
    L.iro_dacvae_int8_dev_free(C.byref(cont))
    assert cont.bytes == 0
