"""The CPU oracle (oracle/iro_oracle.c) pinned against the reference.

1. Against the committed fixtures in tests/golden/, which tests/golden/make_golden.py
   recorded from the reference's own code (ops.c, dacvae.c, dit.c, the VNNI
   prototype) compiled from its sources: bit-exact.
2. Against those reference builds live (oracle/_ref, when present) on fresh
   seeded inputs including NaN / inf / degenerate rows: bit-exact.
3. The property checks of the reference's tests/test_int8_ops.c, run on the
   oracle.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
sys.path.insert(0, GOLDEN)
import inputs  # noqa: E402


def load(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def same(a, b):
    a = np.ascontiguousarray(a); b = np.ascontiguousarray(b)
    if a.shape != b.shape:
        return False
    if a.dtype == np.float32:
        return bool((a.view(np.uint32) == b.view(np.uint32)).all())
    return bool((a == b).all())


# ---------------------------------------------------------------- fixtures --

@pytest.mark.parametrize("idx", range(4))
def test_golden_int8_ops_cases(idx):
    g = load("int8_ops")
    M, N, K, outlier, w, x, bias = inputs.int8_ops_cases()[idx]
    assert bytes(g[f"c{idx}_inputs_sha"]) == inputs.sha(w, x, bias), "input generator drift"
    W = oracle.weight_quantize(w)
    assert same(W.data, g[f"c{idx}_wdata"]) and same(W.scale, g[f"c{idx}_wscale"])
    assert same(W.colsum, g[f"c{idx}_wcolsum"])
    q, s, z = oracle.quantize_rows(x)
    assert same(q, g[f"c{idx}_q"]) and same(s, g[f"c{idx}_s"]) and same(z, g[f"c{idx}_z"])
    y, work = oracle.linear_ex(q, s, z, W, bias)
    assert same(work, g[f"c{idx}_work"]) and same(y, g[f"c{idx}_y"])
    sub = min(M, 5)
    _, work_sub = oracle.linear_ex(q[M - sub:], s[M - sub:], z[M - sub:], W, bias)
    assert same(work_sub, g[f"c{idx}_work_sub"])


def test_golden_degenerate_rows_and_selfcheck():
    g = load("int8_ops")
    q, s, z = oracle.quantize_rows(inputs.degenerate_rows())
    assert same(q, g["degen_q"]) and same(s, g["degen_s"]) and same(z, g["degen_z"])
    assert int(g["selfcheck_rc"][0]) == 0
    a, b, want = oracle.selfcheck_case()
    assert same(oracle.gemm_u8s8(a, b), want)
    # The probe's sums overflow int16 (the reason it exists).
    assert np.abs(want).max() > 32767


def test_golden_residual():
    g = load("residual")
    x = inputs.residual_input()
    assert bytes(g["inputs_sha"]) == inputs.sha(x)
    (q1, s1, z1), r, (q2, s2, z2) = oracle.quantize_rows_residual(x)
    for a, name in zip((q1, s1, z1, r, q2, s2, z2), ("q1", "s1", "z1", "r", "q2", "s2", "z2")):
        assert same(a, g[name]), name
    W = oracle.weight_quantize(inputs.residual_weight())
    y1, _ = oracle.linear_ex(q1, s1, z1, W)
    y2, _ = oracle.linear_ex(q2, s2, z2, W, None, y=y1, accumulate=True)
    assert same(y2, g["y_two_term"])


@pytest.mark.parametrize("idx", range(4))
def test_golden_conv7(idx):
    g = load("conv7")
    case, inp, w, bias = inputs.conv_cases()[idx]
    assert bytes(g[f"c{idx}_inputs_sha"]) == inputs.sha(inp, w, bias)
    W = oracle.weight_quantize(w)
    assert same(W.data, g[f"c{idx}_wdata"])
    out = oracle.conv1d_int8(inp, W, case["kernel"], case["stride"], case["dilation"],
                             case["padding"], bias, case["residual"])
    assert same(out, g[f"c{idx}_out"])


@pytest.mark.parametrize("idx", range(5))
@pytest.mark.parametrize("mode", ["single", "two_term"])
def test_golden_convtranspose(idx, mode):
    g = load("convt")
    case, inp, w, bias = inputs.convt_cases()[idx]
    assert bytes(g[f"c{idx}_inputs_sha"]) == inputs.sha(inp, w, bias)
    W = oracle.weight_quantize(w)
    assert same(W.data, g[f"c{idx}_wdata"])
    out = oracle.convtranspose1d_int8(inp, W, case["C_out"], case["kernel"], case["stride"],
                                      case["padding"], case["output_padding"], bias,
                                      mode == "two_term")
    assert same(out, g[f"c{idx}_{mode}"])


@pytest.mark.parametrize("mode", ["single", "two_term"])
def test_golden_codec_conv1(mode):
    g = load("conv1")
    hidden, skip, w, bias = inputs.conv1_case()
    assert bytes(g["inputs_sha"]) == inputs.sha(hidden, skip, w, bias)
    W = oracle.weight_quantize(w)
    out = oracle.codec_conv1(hidden, W, bias, skip, mode == "two_term")
    assert same(out, g[f"out_{mode}"])


def test_golden_symmetric_quantiser():
    g = load("sym_quant")
    x = inputs.sym_input()
    assert bytes(g["inputs_sha"]) == inputs.sha(x)
    q, s, z = oracle.quantize_rows(x, symmetric=True)
    assert same(q, g["q"]) and same(s, g["s"]) and (z == 128).all()


def test_golden_dit_swiglu_both_policies():
    """dit.c's own int8 SwiGLU (dit.c:913-969) at its fixed 1280/3680 dims, with
    the default two-term W2 and with IRO_INT8_RESIDUAL=0."""
    g = load("dit_swiglu")
    D, H = (int(v) for v in g["dims"])
    x, w1, w3, w2 = inputs.dit_swiglu_inputs(D, H)
    assert bytes(g["inputs_sha"]) == inputs.sha(x, w1, w3, w2)
    W = [oracle.weight_quantize(w) for w in (w1, w3, w2)]
    assert same(oracle.swiglu(x, *W, residual_w2=True), g["residual_default"])
    assert same(oracle.swiglu(x, *W, residual_w2=False), g["single_term"])


# ------------------------------------------------------ live reference ---

@pytest.fixture(scope="module")
def ref():
    if not oracle.ref_available("ieee"):
        pytest.skip("oracle/_ref reference builds are not present")
    return oracle


def _edge_matrix(rng, M, K):
    x = rng.standard_normal((M, K)).astype(np.float32)
    x[0] = 0.0
    x[1] = -np.abs(x[1])
    x[2] = np.abs(x[2]) + 1.0
    x[3, 0] = np.nan
    x[4] = 1e-30 * x[4]
    x[5, 1] = np.inf
    x[6, 2] = -np.inf
    x[7] = np.float32(3.0)
    x[8] = -0.0
    return x


@pytest.fixture(scope="module")
def ref_dit():
    if not oracle.ref_available("dit"):
        pytest.skip("oracle/_ref reference DiT build is not present")
    if os.environ.get("IRO_INT8_RESIDUAL"):
        pytest.skip("the reference reads its residual policy from the environment")
    return oracle


def test_golden_dit_block_and_step_reproduced(ref_dit):
    """The committed DiT fixtures are what the reference block, and the
    step composed from the reference's pieces, produce now."""
    g = load("dit_block")
    seed, B, S, C, cb = (int(v) for v in g["c0_case"])
    x, cond, ck, cv, mask, adaln, qn, kn, ws = inputs.dit_block_case(seed, B, S, C, cb)
    W = [oracle.weight_quantize(w) for w in ws]
    assert same(oracle.ref_dit_block(x, cond, ck, cv, mask, cb, B, S, C, adaln, qn, kn, W),
                g["c0_out"])
    g = load("dit_step")
    seed, layers, R, cfg, S, C = (int(v) for v in g["case"])
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(seed, layers, R, cfg, S, C)
    bw = [(a, q, k, [oracle.weight_quantize(w) for w in w8]) for a, q, k, w8 in blocks]
    t, tn, s1, s2 = (float(v) for v in g["step_args"])
    assert same(oracle.ref_dit_euler_step(state, ck, cv, mask, bw, head, R, cfg, S, C, t, tn,
                                          [s1, s2]), g["step_out"])


def test_golden_dit_block_diag_reproduced(ref_dit, tmp_path):
    """The diagnostic-mode fixture (IRO_INT8_MASK / IRO_INT8_EMULATE set in
    a child process, as tests/golden/make_golden.py records it) is what the
    reference produces now: activation emulation on a mixed mask."""
    import make_golden
    idx = 5
    path = str(tmp_path / "diag.npz")
    make_golden.run_dit_block_diag_child(idx, path)
    got, g = np.load(path), load("dit_block_diag")
    assert same(got["case"], g[f"c{idx}_case"]) and same(got["out"], g[f"c{idx}_out"])


def test_reference_dit_block_sensitivity(ref_dit):
    """The int8 block is sensitive to fp32 rounding: a one-ulp perturbation
    of the reference's own input moves its output by about 1e-3 of its
    magnitude (an activation code moves by one step and the MLP amplifies
    it).  The GPU block tolerance (5e-3 max, 1.5e-4 mean, relative to
    max |out|) is set just above this envelope; this test keeps the
    measurement behind that bound reproducible."""
    seed, B, S, C, cb = 303, 3, 130, 33, 3
    x, cond, ck, cv, mask, adaln, qn, kn, ws = inputs.dit_block_case(seed, B, S, C, cb)
    W = [oracle.weight_quantize(w) for w in ws]
    base = oracle.ref_dit_block(x, cond, ck, cv, mask, cb, B, S, C, adaln, qn, kn, W)
    scale = float(np.abs(base).max())
    rng = np.random.default_rng(1)
    worst = 0.0
    for _ in range(2):
        xp = (x * (1 + rng.choice([-1, 1], x.shape) * 2.0 ** -23)).astype(np.float32)
        out = oracle.ref_dit_block(xp, cond, ck, cv, mask, cb, B, S, C, adaln, qn, kn, W)
        worst = max(worst, float(np.abs(out.astype(np.float64) - base).max()) / scale)
    assert 5e-4 < worst < 5e-3, worst


@pytest.mark.parametrize("M,K", [(9, 16), (16, 100), (24, 1027), (12, 2816)])
def test_live_quantisers_match_reference(ref, M, K):
    rng = np.random.default_rng(M * K)
    x = _edge_matrix(rng, M, K)
    got = oracle.quantize_rows(x)
    want = ref.ref_quantize_rows(x)
    for a, b in zip(got, want):
        assert same(a, b)
    g2 = oracle.quantize_rows_residual(x)
    w2 = ref.ref_quantize_rows_residual(x)
    for a, b in zip(g2[0] + (g2[1],) + g2[2], w2[0] + (w2[1],) + w2[2]):
        assert same(a, b)


@pytest.mark.parametrize("N,K", [(7, 16), (33, 130), (64, 1280)])
def test_live_weight_quantiser_matches_reference(ref, N, K):
    rng = np.random.default_rng(N + K)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    w[0] = 0.0
    w[1, 3] = np.inf
    w[2, 5] = np.nan
    a = oracle.weight_quantize(w)
    b = ref.ref_weight_quantize(w)
    assert same(a.data, b.data) and same(a.scale, b.scale) and same(a.colsum, b.colsum)
    wt = np.ascontiguousarray(w.T)
    a = oracle.weight_quantize_transposed(wt)
    b = ref.ref_weight_quantize_transposed(wt)
    assert same(a.data, b.data) and same(a.scale, b.scale) and same(a.colsum, b.colsum)


@pytest.mark.parametrize("M,N,K", [(1, 3, 5), (31, 40, 96), (70, 130, 1030)])
def test_live_linear_matches_reference(ref, M, N, K):
    rng = np.random.default_rng(M + N + K)
    x = rng.standard_normal((M, K)).astype(np.float32)
    W = oracle.weight_quantize((rng.standard_normal((N, K)) * 0.03).astype(np.float32))
    b = rng.standard_normal(N).astype(np.float32)
    q, s, z = oracle.quantize_rows(x)
    y0 = rng.standard_normal((M, N)).astype(np.float32)
    for bias in (None, b):
        for acc in (False, True):
            ya, wa = oracle.linear_ex(q, s, z, W, bias, y=y0, accumulate=acc)
            yb, wb = ref.ref_linear_ex(q, s, z, W, bias, y=y0, accumulate=acc)
            assert same(wa, wb) and same(ya, yb)


def test_live_silu_matches_reference(ref):
    rng = np.random.default_rng(5)
    a = (rng.standard_normal(4096) * 6).astype(np.float32)
    a[:4] = [0.0, -100.0, 100.0, -89.0]
    g = rng.standard_normal(4096).astype(np.float32)
    assert same(oracle.silu_mul(a, g), ref.ref_silu_mul(a, g))


@pytest.mark.parametrize("d,res,stride", [(1, 0, 1), (3, 1, 1), (9, 1, 1), (1, 1, 2)])
def test_live_conv_matches_reference(ref, d, res, stride):
    if not oracle.ref_available("codec"):
        pytest.skip("codec reference build missing")
    rng = np.random.default_rng(d * 10 + res)
    inp = (rng.standard_normal((150, 48)) * 0.5).astype(np.float32)
    inp[10] = 0.0
    W = oracle.weight_quantize((rng.standard_normal((40, 7 * 48)) * 0.02).astype(np.float32))
    bias = (rng.standard_normal(40) * 0.01).astype(np.float32)
    a = oracle.conv1d_int8(inp, W, 7, stride, d, 3 * d, bias, res)
    b = ref.ref_conv1d_int8(inp, W, 7, stride, d, 3 * d, bias, res)
    assert same(a, b)


# --------------------------------------- tests/test_int8_ops.c on the oracle --

@pytest.mark.parametrize("idx", range(4))
def test_reference_property_checks_on_oracle(idx):
    M, N, K, outlier, w, x, bias = inputs.int8_ops_cases()[idx]
    W = oracle.weight_quantize(w)
    rec = np.abs(w - W.scale[:, None] * W.data.astype(np.float32))
    assert (rec <= W.scale[:, None] * 0.5 + 1e-7).all()
    assert (W.data.astype(np.int32).sum(1) == W.colsum).all()
    q, s, z = oracle.quantize_rows(x)
    assert ((z >= 0) & (z <= 255)).all() and (s > 0).all()
    rec = np.abs(s[:, None] * (q.astype(np.float32) - z[:, None]) - x)
    assert (rec <= s[:, None] * 0.5 + 1e-5).all()
    y, work = oracle.linear_ex(q, s, z, W, bias)
    assert (work == q.astype(np.int64) @ W.data.astype(np.int64).T).all()
    yf = x.astype(np.float64) @ w.astype(np.float64).T + bias
    rel = np.sqrt(((y - yf) ** 2).sum() / max((yf ** 2).sum(), 1.0))
    assert rel < (0.05 if outlier else 0.02)


def test_fixture_generator_is_committed_and_runs_offline():
    """make_golden.py only needs oracle/_ref; it must not touch the network."""
    src = open(os.path.join(GOLDEN, "make_golden.py")).read()
    assert "oracle.ref_" in src and "urllib" not in src and "requests" not in src


def test_dit_branch_split_and_vec_build_agree(ref_dit):
    """The config-3 fixture (tests/golden/make_dit_cfg3.py) runs each CFG
    branch as its own batch-1 forward, from the -O3 IEEE-semantics build
    (libiro_ref_dit_vec.so) where it exists.  Both must give the reference
    sampler's result bit for bit: batched (dit.c's B = cfg) from the -O2
    parity build, on a two-step, one-layer case through the CFG window."""
    R, cfg, S, C = 1, 4, 24, 12
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(71, 1, R, cfg, S, C)
    bw = [(a, q, k, [oracle.weight_quantize(w) for w in w8]) for a, q, k, w8 in blocks]
    scales = [2.0, 1.5, 1.0]
    want = oracle.ref_dit_sample_euler(state, ck, cv, mask, bw, head, R, cfg, S, C, 2, 0.999,
                                       0.6, 1.0, scales)
    kinds = ["dit"] + (["dit_vec"] if oracle.ref_available("dit_vec") else [])
    for kind in kinds:
        fin, vel, rows = oracle.ref_dit_sample_request(
            state[0], [k[0:1] for k in ck], [v[0:1] for v in cv], mask[:cfg], bw, head, cfg, S,
            C, 2, 0.999, 0.6, 1.0, scales, kind=kind)
        assert rows == [4, 1]
        assert same(fin, want[0]), kind


def test_cfg3_fixture_generator_is_committed():
    src = open(os.path.join(GOLDEN, "make_dit_cfg3.py")).read()
    assert "ref_dit_sample_request" in src and "urllib" not in src
    g = load("dit_cfg3")
    assert tuple(int(v) for v in g["case"]) == tuple(inputs.CFG3[k] for k in
                                                     ("seed", "layers", "R", "cfg", "S", "C"))
    assert list(g["rows_per_step"]) == [4, 4, 4, 4, 1, 1, 1, 1]
    assert np.isfinite(g["velocity"]).all() and np.isfinite(g["final"]).all()
    assert g["env_velocity_max"].shape == (8,) and (g["env_final"] > 0).all()
