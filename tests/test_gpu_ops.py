"""GPU parity of the int8 operators against the CPU oracle, through the C ABI.

Bar: integer and byte outputs bit-exact; fp32 outputs of the linear paths
bit-exact too (the kernels use the reference's rounding order, so the
1e-6 relative bound of the spec is met with zero error).  Ports every check
of the reference's tests/test_int8_ops.c and its selfcheck (ops.c:375-398).
"""
import numpy as np
import pytest

import iro_b200 as iro
import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def device():
    iro.init(0)
    yield


def bits(a):
    a = np.ascontiguousarray(a)
    return a.view(np.uint32 if a.dtype.itemsize == 4 else np.uint8)


def assert_same(a, b, what):
    a = np.asarray(a); b = np.asarray(b)
    assert a.shape == b.shape, what
    if a.dtype == np.float32:
        diff = bits(a) != bits(b)
        both_nan = np.isnan(a) & np.isnan(b)
        bad = diff & ~both_nan
    else:
        bad = a != b
    n = int(bad.sum())
    assert n == 0, f"{what}: {n} of {a.size} differ; first at {np.argwhere(bad)[:3].tolist()}"


def test_selfcheck_exact_sums():
    # ops.c:375-398 via the tensor-core GEMM.
    assert iro.selfcheck() == 0
    assert iro.lib().iro_int8_fast_available() == 1
    assert iro.lib().iro_int8_prepare_backend() is not None


def _ops_case(g, M, N, K, outlier):
    w = g.rnd(N * K).reshape(N, K) * np.float32(0.08)
    x = g.rnd(M * K).reshape(M, K) * np.float32(3.0)
    if outlier:
        for m in range(M):
            x[m, 17] = np.float32(20.0) + g.rnd(1)[0]
    bias = g.rnd(N)
    return w, x, bias


@pytest.mark.parametrize("case", [(7, 32, 64, 0), (23, 96, 128, 1), (112, 160, 1280, 0),
                                  (37, 184, 1280, 1)])
def test_reference_int8_ops_cases(case):
    """tests/test_int8_ops.c:34-119 through the host-pointer ops.h API."""
    g = oracle.XorShift()
    # Reproduce the generator state of the reference test for this case.
    for prev in [(7, 32, 64, 0), (23, 96, 128, 1), (112, 160, 1280, 0), (37, 184, 1280, 1)]:
        w, x, bias = _ops_case(g, *prev)
        if prev == case:
            break
    M, N, K, outlier = case
    qw = iro.HostWeight(w)
    ow = oracle.weight_quantize(w)
    assert_same(qw.data, ow.data, "weight codes")
    assert_same(qw.scale, ow.scale, "weight scales")
    assert_same(qw.colsum, ow.colsum, "weight colsum")
    # reconstruction bound |w - s*q| <= s/2 (test_int8_ops.c:57-69)
    rec = np.abs(w - qw.scale[:, None] * qw.data.astype(np.float32))
    assert (rec <= qw.scale[:, None] * 0.5 + 1e-7).all()
    assert (qw.data.astype(np.int32).sum(1) == qw.colsum).all()

    q, s, z = iro.quantize_rows(x)
    oq, os_, oz = oracle.quantize_rows(x)
    assert_same(q, oq, "activation codes")
    assert_same(s, os_, "activation scales")
    assert_same(z, oz, "zero points")
    assert ((z >= 0) & (z <= 255)).all() and (s > 0).all()
    rec = np.abs(s[:, None] * (q.astype(np.float32) - z[:, None].astype(np.float32)) - x)
    assert (rec <= s[:, None] * 0.5 + 1e-5).all()

    y, work = iro.linear_ex(q, s, z, qw, bias)
    oy, owork = oracle.linear_ex(q, s, z, ow, bias)
    assert_same(work, owork, "int32 sums")
    assert_same(y, oy, "dequantised outputs")
    # cross-M determinism (test_int8_ops.c:87-97)
    sub = min(M, 5)
    y2, work2 = iro.linear_ex(q[M - sub:], s[M - sub:], z[M - sub:], qw, bias)
    assert_same(work2, owork[M - sub:], "cross-M sums")
    # float error budget vs an fp32 GEMM (test_int8_ops.c:99-109)
    yf = x.astype(np.float64) @ w.astype(np.float64).T + bias
    rel = np.sqrt(((y - yf) ** 2).sum() / max((yf ** 2).sum(), 1.0))
    assert rel < (0.05 if outlier else 0.02)
    nbytes = qw.nbytes()
    assert nbytes == N * K + N * 8
    qw.free()
    assert qw.st.data is None and qw.nbytes() == 0


def test_degenerate_rows():
    """test_int8_ops.c:126-134: an all-zero row and a constant positive row."""
    x = np.zeros((2, 16), np.float32)
    x[1] = 2.5
    q, s, z = iro.quantize_rows(x)
    assert s[0] > 0 and 0 <= z[0] <= 255 and q[1, 0] == 255 and z[1] == 0
    oq, os_, oz = oracle.quantize_rows(x)
    assert_same(q, oq, "codes"); assert_same(s, os_, "scales"); assert_same(z, oz, "zp")


@pytest.mark.parametrize("K", [16, 100, 1024, 1030, 2816, 3680, 5000])
@pytest.mark.parametrize("mode", ["asym", "sym", "residual"])
def test_quantizer_byte_exact(K, mode):
    rng = np.random.default_rng(K)
    M = 67
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[3] = 0.0                                  # all-zero row
    x[5] = 1.75                                 # constant row
    x[7, :: max(K // 7, 1)] *= 40.0             # outliers
    x[9] = -np.abs(x[9])                        # all negative
    x[11, 1] = np.nan                           # NaN is skipped by min/max
    x[13] *= 1e-30                              # tiny scale
    xd = iro.DevBuf.from_host(x)
    q = iro.DevBuf((M, K), np.uint8); s = iro.DevBuf(M, np.float32); z = iro.DevBuf(M, np.int32)
    if mode == "residual":
        r = iro.DevBuf((M, K), np.float32)
        q2 = iro.DevBuf((M, K), np.uint8); s2 = iro.DevBuf(M, np.float32)
        z2 = iro.DevBuf(M, np.int32)
        iro.quantize_rows_residual_dev(xd, M, K, q, s, z, r, q2, s2, z2)
        iro.synchronize()
        (oq, os_, oz), orr, (oq2, os2, oz2) = oracle.quantize_rows_residual(x)
        assert_same(r.get(), orr, "residual")
        assert_same(q2.get(), oq2, "codes2"); assert_same(s2.get(), os2, "scales2")
        assert_same(z2.get(), oz2, "zp2")
    else:
        iro.quantize_rows_dev(xd, M, K, q, s, z, symmetric=(mode == "sym"))
        iro.synchronize()
        oq, os_, oz = oracle.quantize_rows(x, symmetric=(mode == "sym"))
    assert_same(q.get(), oq, "codes"); assert_same(s.get(), os_, "scales")
    assert_same(z.get(), oz, "zp")


def test_host_residual_quantizer():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((33, 2816)) * np.exp(rng.standard_normal((33, 1)))).astype(np.float32)
    got = iro.quantize_rows_residual(x)
    want = oracle.quantize_rows_residual(x)
    for a, b, name in zip(got[0] + (got[1],) + got[2], want[0] + (want[1],) + want[2],
                          ["q1", "s1", "z1", "r", "q2", "s2", "z2"]):
        assert_same(a, b, name)


def _rand_weight(rng, N, K, scale=0.02):
    return (rng.standard_normal((N, K)) * scale).astype(np.float32)


@pytest.mark.parametrize("M,N,K", [(1, 8, 64), (7, 96, 128), (129, 160, 200), (300, 1000, 1024),
                                   (512, 4096, 1024), (1000, 520, 2816), (64, 1024, 16),
                                   (2048, 1024, 2816)])
@pytest.mark.parametrize("bias,accumulate", [(True, False), (False, True), (True, True)])
def test_linear_dev_bit_exact(M, N, K, bias, accumulate):
    rng = np.random.default_rng(M * 7 + N + K)
    w = _rand_weight(rng, N, K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    ow = oracle.weight_quantize(w)
    q, s, z = oracle.quantize_rows(x)
    b = (rng.standard_normal(N) * 0.01).astype(np.float32) if bias else None
    y0 = rng.standard_normal((M, N)).astype(np.float32) if accumulate else None
    dw = iro.DevWeight.upload((ow.data, ow.scale, ow.colsum))
    qd, sd, zd = iro.DevBuf.from_host(q), iro.DevBuf.from_host(s), iro.DevBuf.from_host(z)
    bd = iro.DevBuf.from_host(b) if bias else None
    yd = iro.DevBuf.from_host(y0) if accumulate else iro.DevBuf((M, N), np.float32)
    wk = iro.DevBuf((M, N), np.int32)
    iro.linear_dev(qd, sd, zd, dw, bd, yd, M, work=wk, accumulate=accumulate)
    iro.synchronize()
    oy, owork = oracle.linear_ex(q, s, z, ow, b, y=y0, accumulate=accumulate)
    assert_same(wk.get(), owork, "int32 sums")
    assert_same(yd.get(), oy, "outputs")


@pytest.mark.parametrize("M", [64, 256, 4096, 65536])
@pytest.mark.parametrize("N", [1024, 2816, 4096])
def test_linear_sweep_shapes_bit_exact(M, N):
    """Config 5's isolated GEMM sweep (K = 1024, config 1's distributions:
    N(0,1) activations with 0.1% outliers x20, N(0,0.02) weights, N(0,0.01)
    bias): the whole M on the device, every tile schedule up to 65536 rows;
    the codes, raw int32 sums and outputs of a row sample (the first and last
    96 rows and 128 random rows; rows are independent) bit-exact against
    the oracle."""
    K = 1024
    rng = np.random.default_rng(M + N)
    w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[rng.random((M, K)) < 0.001] *= 20.0
    b = (rng.standard_normal(N) * 0.01).astype(np.float32)
    ow = oracle.weight_quantize(w)
    dw = iro.DevWeight.upload((ow.data, ow.scale, ow.colsum))
    xd = iro.DevBuf.from_host(x)
    qd, sd, zd = iro.DevBuf((M, K), np.uint8), iro.DevBuf(M, np.float32), iro.DevBuf(M, np.int32)
    iro.quantize_rows_dev(xd, M, K, qd, sd, zd)
    bd = iro.DevBuf.from_host(b)
    yd = iro.DevBuf((M, N), np.float32)
    wk = iro.DevBuf((M, N), np.int32)
    iro.linear_dev(qd, sd, zd, dw, bd, yd, M, work=wk)
    iro.synchronize()
    rows = np.unique(np.r_[0:min(96, M), max(0, M - 96):M, rng.integers(0, M, 128)])
    q, s, z = oracle.quantize_rows(x[rows])
    assert_same(qd.get()[rows], q, "codes")
    oy, owork = oracle.linear_ex(q, s, z, ow, b)
    assert_same(wk.get()[rows], owork, "int32 sums")
    assert_same(yd.get()[rows], oy, "outputs")
    # The no-raw-sum path (what the DiT and the sweep bench run) too.
    yd2 = iro.DevBuf((M, N), np.float32)
    iro.linear_dev(qd, sd, zd, dw, bd, yd2, M)
    iro.synchronize()
    assert_same(yd2.get()[rows], oy, "outputs without raw sums")


def test_linear_symmetric_mode_undoes_offset():
    """Symmetric s8 activations stored as u8+128 with zero=128: the s32 sum of
    the u8 GEMM minus 128*colsum equals the s8 x s8 sum."""
    rng = np.random.default_rng(11)
    M, N, K = 96, 256, 1024
    x = rng.standard_normal((M, K)).astype(np.float32)
    ow = oracle.weight_quantize(_rand_weight(rng, N, K))
    xd = iro.DevBuf.from_host(x)
    q = iro.DevBuf((M, K), np.uint8); s = iro.DevBuf(M, np.float32); z = iro.DevBuf(M, np.int32)
    iro.quantize_rows_dev(xd, M, K, q, s, z, symmetric=True)
    dw = iro.DevWeight.upload((ow.data, ow.scale, ow.colsum))
    y = iro.DevBuf((M, N), np.float32); wk = iro.DevBuf((M, N), np.int32)
    iro.linear_dev(q, s, z, dw, None, y, M, work=wk)
    iro.synchronize()
    qh = q.get()
    s8 = qh.astype(np.int32) - 128
    want = s8 @ ow.data.astype(np.int32).T
    assert_same(wk.get() - 128 * ow.colsum[None, :], want.astype(np.int32), "s8 sums")
    oy, _ = oracle.linear_ex(qh, s.get(), z.get(), ow)
    assert_same(y.get(), oy, "outputs")


@pytest.mark.parametrize("M,N,K", [(5, 64, 128), (300, 1024, 1024), (2048, 1024, 2816)])
def test_linear2_dual_term(M, N, K):
    """dit.c:479-486: y = linear(q1) [+ bias] then += linear(q2), fused."""
    rng = np.random.default_rng(N + M)
    h = (rng.standard_normal((M, K)) * 0.3).astype(np.float32)
    ow = oracle.weight_quantize(_rand_weight(rng, N, K))
    b = (rng.standard_normal(N) * 0.01).astype(np.float32)
    (q1, s1, z1), _, (q2, s2, z2) = oracle.quantize_rows_residual(h)
    dw = iro.DevWeight.upload((ow.data, ow.scale, ow.colsum))
    args = [iro.DevBuf.from_host(a) for a in (q1, s1, z1, q2, s2, z2)]
    bd = iro.DevBuf.from_host(b)
    y = iro.DevBuf((M, N), np.float32)
    iro.linear2_dev(*args, dw, bd, y, M)
    iro.synchronize()
    y1, _ = oracle.linear_ex(q1, s1, z1, ow, b)
    y2, _ = oracle.linear_ex(q2, s2, z2, ow, None, y=y1, accumulate=True)
    assert_same(y.get(), y2, "two-term outputs")


@pytest.mark.parametrize("M,N", [(24000, 1024), (19999, 1280)])
def test_linear2_dual_term_cta_pairs(M, N):
    """The two-term linear at the DiT's W2 size (K = 2816, many waves) runs
    on CTA pairs (tcgen05 cta_group::2, 256-row pair tiles, each CTA staging
    half of the weight tile); the last pair tile of M = 19999 is ragged.  A
    row sample (first and last 128 rows, 256 random) bit-exact against the
    oracle."""
    K = 2816
    rng = np.random.default_rng(M + N)
    h = (rng.standard_normal((M, K)) * 0.3).astype(np.float32)
    ow = oracle.weight_quantize(_rand_weight(rng, N, K))
    b = (rng.standard_normal(N) * 0.01).astype(np.float32)
    hd = iro.DevBuf.from_host(h)
    bufs = [iro.DevBuf((M, K), np.uint8), iro.DevBuf(M, np.float32), iro.DevBuf(M, np.int32),
            iro.DevBuf((M, K), np.uint8), iro.DevBuf(M, np.float32), iro.DevBuf(M, np.int32)]
    iro.quantize_rows_residual_dev(hd, M, K, *bufs[:3], None, *bufs[3:])
    dw = iro.DevWeight.upload((ow.data, ow.scale, ow.colsum))
    bd = iro.DevBuf.from_host(b)
    y = iro.DevBuf((M, N), np.float32)
    iro.linear2_dev(*bufs, dw, bd, y, M)
    iro.synchronize()
    rows = np.unique(np.r_[0:128, M - 128:M, rng.integers(0, M, 256)])
    (q1, s1, z1), _, (q2, s2, z2) = oracle.quantize_rows_residual(h[rows])
    y1, _ = oracle.linear_ex(q1, s1, z1, ow, b)
    y2, _ = oracle.linear_ex(q2, s2, z2, ow, None, y=y1, accumulate=True)
    assert_same(y.get()[rows], y2, "two-term outputs")


@pytest.mark.parametrize("M,seg", [(512, 1024), (37, 1280), (750, 256)])
def test_qkvg_split(M, seg):
    """dit.c:785-792: one quantised x, four projections; fused N-concat GEMM
    whose column blocks go to four buffers, bit-identical per column."""
    rng = np.random.default_rng(seg + M)
    K = 1024
    x = rng.standard_normal((M, K)).astype(np.float32)
    ws = [oracle.weight_quantize(_rand_weight(rng, seg, K)) for _ in range(4)]
    q, s, z = oracle.quantize_rows(x)
    dw = iro.DevWeight.concat([(w.data, w.scale, w.colsum) for w in ws])
    qd, sd, zd = iro.DevBuf.from_host(q), iro.DevBuf.from_host(s), iro.DevBuf.from_host(z)
    outs = [iro.DevBuf((M, seg), np.float32) for _ in range(4)]
    iro.linear_split_dev(qd, sd, zd, dw, outs, seg, M)
    iro.synchronize()
    for o, w in zip(outs, ws):
        oy, _ = oracle.linear_ex(q, s, z, w)
        assert_same(o.get(), oy, "qkvg block")


def test_weight_quantize_device_and_transposed():
    rng = np.random.default_rng(5)
    for (N, K) in [(3, 40), (96, 128), (1536, 7 * 96), (300, 1030)]:
        w = _rand_weight(rng, N, K)
        w[1, :] = 0.0
        hw = iro.HostWeight(w)
        ow = oracle.weight_quantize(w)
        assert_same(hw.data, ow.data, "codes"); assert_same(hw.scale, ow.scale, "scales")
        assert_same(hw.colsum, ow.colsum, "colsum")
        wt = np.ascontiguousarray(w.T)
        ht = iro.HostWeight(wt, transposed=True)
        otw = oracle.weight_quantize_transposed(wt)
        assert_same(ht.data, otw.data, "t codes"); assert_same(ht.scale, otw.scale, "t scales")
        assert_same(ht.colsum, ow.colsum, "t colsum")


def test_bounded_wait_reports_timeout_and_context_survives():
    """A device wait on a barrier nothing completes gives up after its limit
    and the host reads IRO_ERR_DEVICE_TIMEOUT; later work still runs."""
    rc = iro.lib().iro_debug_bounded_wait_probe(20_000_000)  # 20 ms
    assert rc == iro.IRO_ERR_DEVICE_TIMEOUT
    assert iro.selfcheck() == 0


def test_invalid_arguments_fail_loudly():
    w = iro.IroInt8Weight()
    assert iro.lib().iro_int8_weight_quantize(None, None, 4, 4) == -1
    x = np.ones((2, 4), np.float32)
    assert iro.lib().iro_int8_weight_quantize(iro.C.byref(w), iro._p(x), 0, 4) == -1
    iro.lib().iro_int8_quantize_rows(None, 2, 4, None, None, None)
    assert iro.lib().iro_cuda_last_error() == iro.IRO_ERR_INVALID
    assert iro.lib().iro_cuda_last_error() == 0
