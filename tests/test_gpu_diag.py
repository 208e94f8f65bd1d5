"""The DiT's int8 activation diagnostics on the device sampler (dit.c:340-412):
IRO_INT8_STATS per (layer, group) row statistics and IRO_INT8_DUMP raw
activation files at the reference's four recording points (Q/K/V/gate input
dit.c:787, Wo input :879, W1/W3 input :944, W2 input :964).

The dumped activations are checked against the statistics accumulated on the
device (rows and argmax histogram exact, the ratio sum to 1e-9 relative: the
device sums squares in another order), and against each other: the dumped W2
input is the SwiGLU hidden of the dumped W1/W3 input through the oracle
(HIDDEN_ULPS, the gate's expf differs from the host's).  With diagnostics on
the block materialises the AdaLN output instead of quantising it in the
same pass, whose mean square sums in another order, so the step result is
held to the step tolerance against the run without diagnostics."""
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

HIDDEN_ULPS = 4
MAX_REL = 2e-2
MEAN_REL = 3e-3


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


def test_stats_and_dumps_match_the_activations(tmp_path, monkeypatch, capfd):
    R, cfg, S, n_ctx, layers = 1, 2, 40, 12, 2
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(5, layers, R, cfg, S, n_ctx)
    qw = [[oracle.weight_quantize(w) for w in b[3]] for b in blocks]
    dev_blocks = [iro.DiTBlock(a, q, k, *[(w.data, w.scale, w.colsum) for w in W])
                  for (a, q, k, _), W in zip(blocks, qw)]
    m = iro.DiTModel(dev_blocks, head["cond_w0"], head["cond_w1"], head["cond_w2"], head["in_w"],
                     head["in_b"], head["out_norm"], head["out_w"], head["out_b"])
    kd = [iro.DevBuf.from_host(k) for k in ck]
    vd = [iro.DevBuf.from_host(v) for v in cv]
    md = iro.DevBuf.from_host(mask)

    def step():
        sd = iro.DevBuf.from_host(state)
        m.euler_step(sd, R, cfg, S, 0.8, 0.6, [1.5], kd, vd, md, n_ctx)
        iro.synchronize()
        return sd.get().reshape(state.shape)

    monkeypatch.delenv("IRO_INT8_STATS", raising=False)
    monkeypatch.delenv("IRO_INT8_DUMP", raising=False)
    plain = step()
    monkeypatch.setenv("IRO_INT8_STATS", "1")
    monkeypatch.setenv("IRO_INT8_DUMP", str(tmp_path))
    iro.dit_stats_reset()
    diag = step()
    monkeypatch.delenv("IRO_INT8_STATS")
    monkeypatch.delenv("IRO_INT8_DUMP")

    upd_p, upd_d = plain.astype(np.float64) - state, diag.astype(np.float64) - state
    err, scale = np.abs(upd_p - upd_d), np.abs(upd_p).max()
    assert err.max() <= MAX_REL * scale and err.mean() <= MEAN_REL * scale

    M, D, H = R * cfg * S, head["in_w"].shape[0], qw[0][5].N
    for layer in range(layers):
        acts = []
        for g, K in enumerate((D, D, D, H)):
            names = sorted(p.name for p in tmp_path.glob(f"act_L{layer:02d}_G{g}_*"))
            assert names == [f"act_L{layer:02d}_G{g}_0_M{M}_K{K}.f32"]
            a = np.fromfile(tmp_path / names[0], np.float32).reshape(M, K)
            assert np.isfinite(a).all()
            acts.append(a)
            rows, ratio, hist = iro.dit_stats(layer, g)
            ab = np.abs(a)
            rms = np.sqrt((a.astype(np.float64) ** 2).sum(1) / K)
            want = np.where(rms > 0, ab.max(1) / np.where(rms > 0, rms, 1), 0.0).sum()
            assert rows == M
            assert abs(ratio - want) <= 1e-9 * want, (layer, g)
            assert (hist == np.bincount(ab.argmax(1), minlength=hist.size)).all(), (layer, g)
        w1, w3, w2 = qw[layer][5:8]
        _, hid = oracle.swiglu(acts[2], w1, w3, w2, want_hidden=True)
        assert ulp_diff(acts[3], hid).max() <= HIDDEN_ULPS
    assert iro.dit_stats(layers, 0)[0] == 0

    capfd.readouterr()
    iro.dit_stats_report()
    lines = [ln for ln in capfd.readouterr().err.splitlines() if ln.startswith("int8-stats")]
    assert len(lines) == 4 * layers
    assert lines[0].startswith(f"int8-stats layer= 0 group=qkvg rows={M} mean_max/rms=")
    assert lines[-1].startswith(f"int8-stats layer= 1 group=w2   rows={M} mean_max/rms=")
    iro.dit_stats_reset()
    assert iro.dit_stats(0, 0)[0] == 0
