"""Seeded inputs behind the golden fixtures (shared by make_golden.py and the
tests).  The test_int8_ops.c cases use that test's own xorshift generator
(tests/test_int8_ops.c:12-16, 49-53, 122-125); the others use numpy PCG64."""
import hashlib

import numpy as np

CONV_KEYS = ("T", "C", "N", "kernel", "stride", "dilation", "padding", "residual", "bias")


def sha(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        if a is not None:
            h.update(np.ascontiguousarray(a).tobytes())
    return h.digest()


def _xorshift():
    import oracle
    return oracle.XorShift()


def int8_ops_cases():
    """The four cases of tests/test_int8_ops.c, in its order, drawing from one
    generator: w = rnd()*0.08, x = rnd()*3, outliers x[m,17] = 20 + rnd(),
    bias = rnd()."""
    g = _xorshift()
    out = []
    for (M, N, K, outlier) in [(7, 32, 64, 0), (23, 96, 128, 1), (112, 160, 1280, 0),
                               (37, 184, 1280, 1)]:
        w = g.rnd(N * K).reshape(N, K) * np.float32(0.08)
        x = g.rnd(M * K).reshape(M, K) * np.float32(3.0)
        if outlier:
            for m in range(M):
                x[m, 17] = np.float32(20.0) + g.rnd(1)[0]
        bias = g.rnd(N)
        out.append((M, N, K, outlier, w.astype(np.float32), x.astype(np.float32),
                    bias.astype(np.float32)))
    return out


def degenerate_rows():
    """tests/test_int8_ops.c:126-134."""
    x = np.zeros((2, 16), np.float32)
    x[1] = 2.5
    return x


def residual_input():
    rng = np.random.default_rng(2024)
    x = (rng.standard_normal((33, 257)) * np.exp(rng.standard_normal((33, 1)))).astype(np.float32)
    x[3] = 0.0
    x[4, 7] = 40.0
    return x


def residual_weight():
    rng = np.random.default_rng(2025)
    return (rng.standard_normal((48, 257)) * 0.02).astype(np.float32)


def conv_cases():
    cases = [dict(T=40, C=32, N=24, kernel=7, stride=1, dilation=1, padding=3, residual=0, bias=1),
             dict(T=40, C=32, N=24, kernel=7, stride=1, dilation=3, padding=9, residual=1, bias=0),
             dict(T=37, C=16, N=8, kernel=7, stride=2, dilation=1, padding=3, residual=0, bias=1),
             dict(T=12, C=32, N=24, kernel=7, stride=1, dilation=9, padding=27, residual=1, bias=1)]
    out = []
    for i, c in enumerate(cases):
        rng = np.random.default_rng(100 + i)
        inp = (rng.standard_normal((c["T"], c["C"])) * 0.5).astype(np.float32)
        inp[min(5, c["T"] - 1)] = 0.0
        w = (rng.standard_normal((c["N"], c["kernel"] * c["C"])) * 0.02).astype(np.float32)
        bias = (rng.standard_normal(c["N"]) * 0.01).astype(np.float32) if c["bias"] else None
        out.append((c, inp, w, bias))
    return out


CONVT_KEYS = ("T", "C_in", "C_out", "kernel", "stride", "padding", "output_padding", "bias")


def convt_cases():
    """Transposed-conv cases: the decoder's geometry (kernel 2*stride,
    padding (stride+1)/2, output_padding stride&1, dacvae.c:150-160) at
    strides 2, 3, 8 and 12, plus one free geometry.  The reference always
    has a bias here (it copies conv->bias into every output row)."""
    cases = []
    for (T, ci, co, s, b) in ((40, 32, 16, 2, 1), (25, 48, 24, 3, 1), (30, 64, 8, 8, 1),
                              (9, 32, 16, 12, 1)):
        cases.append(dict(T=T, C_in=ci, C_out=co, kernel=2 * s, stride=s, padding=(s + 1) // 2,
                          output_padding=s & 1, bias=b))
    cases.append(dict(T=21, C_in=16, C_out=12, kernel=5, stride=2, padding=0, output_padding=2,
                      bias=1))
    out = []
    for i, c in enumerate(cases):
        rng = np.random.default_rng(300 + i)
        inp = (rng.standard_normal((c["T"], c["C_in"])) * 0.5).astype(np.float32)
        inp[min(4, c["T"] - 1)] = 0.0
        w = (rng.standard_normal((c["kernel"] * c["C_out"], c["C_in"])) * 0.05).astype(np.float32)
        bias = (rng.standard_normal(c["C_out"]) * 0.01).astype(np.float32) if c["bias"] else None
        out.append((c, inp, w, bias))
    return out


def conv1_case():
    rng = np.random.default_rng(400)
    rows, C = 70, 48
    hidden = rng.standard_normal((rows, C)).astype(np.float32)
    hidden[3] = 0.0
    skip = (rng.standard_normal((rows, C)) * 0.3).astype(np.float32)
    w = (rng.standard_normal((C, C)) * 0.05).astype(np.float32)
    bias = (rng.standard_normal(C) * 0.01).astype(np.float32)
    return hidden, skip, w, bias


DIT_D, DIT_HEADS, DIT_RANK, DIT_H = 1280, 20, 192, 3680


def dit_block_case(seed, B, S, C, context_batch):
    """Synthetic inputs of one DiT block at the reference's fixed dimensions:
    x [B*S, D], cond [B, 3D], context K/V [context_batch, C, D] with a mask
    [B, C] per batch row that drops some context tokens (the reference reads
    the mask per batch row even for a shared context), AdaLN matrices
    (attention then MLP, each
    in IroAdaLN order), q/k norm weights, and fp32 projection weights
    (wq, wk, wv, gate, wo, w1, w3, w2) to be quantised."""
    D, R, H = DIT_D, DIT_RANK, DIT_H
    rng = np.random.default_rng(seed)
    f = lambda *sh, s=1.0: (rng.standard_normal(sh) * s).astype(np.float32)
    x = f(B * S, D)
    cond = f(B, 3 * D, s=0.5)
    ctx_k, ctx_v = f(context_batch, C, D), f(context_batch, C, D)
    mask = (rng.random((B, C)) < 0.8).astype(np.uint8)
    mask[:, 0] = 1
    adaln = []
    for _ in range(2):
        for _ in range(3):
            adaln += [f(R, D, s=0.03), f(D, R, s=0.03), f(D, s=0.02)]
    q_norm = (1.0 + f(D, s=0.1)).astype(np.float32)
    k_norm = (1.0 + f(D, s=0.1)).astype(np.float32)
    ws = [f(D, D, s=0.03) for _ in range(5)] + [f(H, D, s=0.03), f(H, D, s=0.03), f(D, H, s=0.02)]
    return x, cond, ctx_k, ctx_v, mask, adaln, q_norm, k_norm, ws


DIT_TIMESTEP, DIT_LATENT = 512, 32


def dit_model_case(seed, layers, R, cfg, S, C):
    """Synthetic inputs of whole DiT Euler steps: the latent state
    [R, S, 32], per-layer context K/V [R, C, D] and block parameters (as
    dit_block_case), the CFG mask [R*cfg, C], and the conditioner, input and
    output weights in the reference's layouts (dit.c:488-541, 1070-1090)."""
    D = DIT_D
    rng = np.random.default_rng(seed)
    f = lambda *sh, s=1.0: (rng.standard_normal(sh) * s).astype(np.float32)
    state = f(R, S, DIT_LATENT)
    mask = (rng.random((R * cfg, C)) < 0.75).astype(np.uint8)
    mask[:, 0] = 1
    ctx_k, ctx_v, blocks = [], [], []
    for layer in range(layers):
        ctx_k.append(f(R, C, D))
        ctx_v.append(f(R, C, D))
        _, _, _, _, _, adaln, qn, kn, ws = dit_block_case(seed * 100 + layer, 1, 1, 1, 1)
        blocks.append((adaln, qn, kn, ws))
    head = {"cond_w0": f(D, DIT_TIMESTEP, s=0.04), "cond_w1": f(D, D, s=0.03),
            "cond_w2": f(3 * D, D, s=0.03), "in_w": f(D, DIT_LATENT, s=0.15),
            "in_b": f(D, s=0.02), "out_norm": (1.0 + f(D, s=0.1)).astype(np.float32),
            "out_w": f(DIT_LATENT, D, s=0.03), "out_b": f(DIT_LATENT, s=0.02)}
    return state, ctx_k, ctx_v, mask, blocks, head


def sym_input():
    rng = np.random.default_rng(77)
    x = rng.standard_normal((40, 96)).astype(np.float32)
    x[2] = 0.0
    x[5, 3] = 55.0
    return x


def dit_swiglu_inputs(D, H, rows=3):
    rng = np.random.default_rng(4242)
    x = rng.standard_normal((rows, D)).astype(np.float32)
    w1 = (rng.standard_normal((H, D)) * 0.02).astype(np.float32)
    w3 = (rng.standard_normal((H, D)) * 0.02).astype(np.float32)
    w2 = (rng.standard_normal((D, H)) * 0.02).astype(np.float32)
    return x, w1, w3, w2


def dit_sha(state, ck, cv, mask, blocks, head):
    """SHA-256 over a DiT model case's inputs, in a fixed order."""
    flat = [state, *ck, *cv, mask] + [a for b in blocks for a in (*b[0], b[1], b[2], *b[3])]
    return sha(*flat, *head.values())


# Config-3 row geometry at the reference's own dimensions: 12 layers, 8
# requests x 4 CFG rows x 750 latent frames (24,000 rows per linear), 128
# context tokens.  The reference fixes d_model 1280 / 20 heads / mlp 3680 as
# compile-time constants (dit.c:11-20), so the full-geometry pin runs at
# those dimensions.
CFG3 = dict(seed=2026, layers=12, R=8, cfg=4, S=750, C=128)
CFG3_SAMPLED = (0, 7)            # requests recorded by the fixture
CFG3_SAMPLER = dict(steps=8, init_scale=0.999, cfg_min_t=0.5, cfg_max_t=1.0,
                    scales=(2.0, 1.5, 1.0))  # generate.c:416-422 window


def dit_cfg3_case():
    c = CFG3
    return dit_model_case(c["seed"], c["layers"], c["R"], c["cfg"], c["S"], c["C"])
