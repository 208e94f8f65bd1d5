"""Generate the committed golden fixtures in tests/golden/ from the REFERENCE
itself: oracle/_ref holds irodori-c's ops.c (IEEE build), dacvae.c, dit.c and
the VNNI prototype compiled from their sources (oracle/Makefile `ref`).

    make -C oracle ref REF_DIR=<reference tree>
    python tests/golden/make_golden.py

Inputs are regenerated from seeds by tests/golden/inputs.py (the reference
test's xorshift for the test_int8_ops.c cases, numpy PCG64 elsewhere); each
fixture also records a SHA-256 of its inputs so a generator drift is caught.
Outputs are exactly what the reference code returned.
"""
import ctypes as C
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import oracle  # noqa: E402
import inputs  # noqa: E402


def int8_ops():
    out = {}
    for idx, (M, N, K, outlier, w, x, bias) in enumerate(inputs.int8_ops_cases()):
        W = oracle.ref_weight_quantize(w)
        q, s, z = oracle.ref_quantize_rows(x)
        y, work = oracle.ref_linear_ex(q, s, z, W, bias)
        sub = min(M, 5)
        y_sub, work_sub = oracle.ref_linear_ex(q[M - sub:], s[M - sub:], z[M - sub:], W, bias)
        pre = f"c{idx}_"
        out.update({pre + "shape": np.array([M, N, K, outlier], np.int32),
                    pre + "inputs_sha": np.frombuffer(inputs.sha(w, x, bias), np.uint8),
                    pre + "wdata": W.data, pre + "wscale": W.scale, pre + "wcolsum": W.colsum,
                    pre + "q": q, pre + "s": s, pre + "z": z, pre + "work": work, pre + "y": y,
                    pre + "work_sub": work_sub})
    x = inputs.degenerate_rows()
    q, s, z = oracle.ref_quantize_rows(x)
    out.update({"degen_q": q, "degen_s": s, "degen_z": z})
    L = oracle.ref_lib("ieee")
    out["selfcheck_rc"] = np.array([L.iro_int8_selfcheck()], np.int32)
    return out


def residual():
    x = inputs.residual_input()
    (q1, s1, z1), r, (q2, s2, z2) = oracle.ref_quantize_rows_residual(x)
    acc = {}
    W = oracle.ref_weight_quantize(inputs.residual_weight())
    y1, _ = oracle.ref_linear_ex(q1, s1, z1, W, None)
    y2, _ = oracle.ref_linear_ex(q2, s2, z2, W, None, y=y1, accumulate=True)
    acc.update({"inputs_sha": np.frombuffer(inputs.sha(x), np.uint8), "q1": q1, "s1": s1,
                "z1": z1, "r": r, "q2": q2, "s2": s2, "z2": z2, "y_two_term": y2})
    return acc


def conv7():
    out = {}
    for idx, (case, inp, w, bias) in enumerate(inputs.conv_cases()):
        W = oracle.ref_weight_quantize(w)
        o = oracle.ref_conv1d_int8(inp, W, case["kernel"], case["stride"], case["dilation"],
                                   case["padding"], bias, case["residual"])
        pre = f"c{idx}_"
        out.update({pre + "params": np.array([case[k] for k in inputs.CONV_KEYS], np.int32),
                    pre + "inputs_sha": np.frombuffer(inputs.sha(inp, w, bias), np.uint8),
                    pre + "wdata": W.data, pre + "wscale": W.scale, pre + "wcolsum": W.colsum,
                    pre + "out": o})
    return out


def sym():
    x = inputs.sym_input()
    L = oracle.ref_lib("vnni")
    L.ref_quantize_activation_sym.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int]
    L.ref_quantize_activation_sym.restype = None
    M, K = x.shape
    q = np.empty((M, K), np.uint8)
    s = np.empty(M, np.float32)
    L.ref_quantize_activation_sym(oracle._ptr(x), oracle._ptr(q), oracle._ptr(s), M, K)
    return {"inputs_sha": np.frombuffer(inputs.sha(x), np.uint8), "q": q, "s": s}


def dit_swiglu_child(mode):
    """Runs in a child process so IRO_INT8_RESIDUAL is read fresh (the
    reference caches it in a function-static)."""
    D, H = oracle.ref_dit_dims()
    x, w1, w3, w2 = inputs.dit_swiglu_inputs(D, H)
    W = [oracle.ref_weight_quantize(w) for w in (w1, w3, w2)]
    o = oracle.ref_dit_swiglu(x, *W)
    np.save(os.path.join(HERE, f"_tmp_swiglu_{mode}.npy"), o)


def dit_swiglu():
    out = {}
    for mode, env in (("residual_default", None), ("single_term", "0")):
        e = dict(os.environ)
        e.pop("IRO_INT8_RESIDUAL", None)
        if env is not None:
            e["IRO_INT8_RESIDUAL"] = env
        subprocess.run([sys.executable, __file__, "--swiglu-child", mode], check=True, env=e)
        path = os.path.join(HERE, f"_tmp_swiglu_{mode}.npy")
        out[mode] = np.load(path)
        os.remove(path)
    D, H = oracle.ref_dit_dims()
    x, w1, w3, w2 = inputs.dit_swiglu_inputs(D, H)
    out["dims"] = np.array([D, H], np.int32)
    out["inputs_sha"] = np.frombuffer(inputs.sha(x, w1, w3, w2), np.uint8)
    return out


def convt_child(mode):
    """Child process: the reference's upsample residual policy is read once
    per process from IRO_CODEC_INT8_RESIDUAL (dacvae.c:54-61)."""
    want = mode == "two_term"
    assert oracle.ref_codec_upsample_residual() == want
    res = {}
    for idx, (case, inp, w, bias) in enumerate(inputs.convt_cases()):
        W = oracle.ref_weight_quantize(w)
        res[f"c{idx}"] = oracle.ref_convtranspose1d_int8(
            inp, W, case["C_out"], case["kernel"], case["stride"], case["padding"],
            case["output_padding"], bias)
    np.savez(os.path.join(HERE, f"_tmp_convt_{mode}.npz"), **res)


def convt():
    out = {}
    for mode, env in (("single", "0"), ("two_term", "2")):
        e = dict(os.environ)
        e["IRO_CODEC_INT8_RESIDUAL"] = env
        subprocess.run([sys.executable, __file__, "--convt-child", mode], check=True, env=e)
        path = os.path.join(HERE, f"_tmp_convt_{mode}.npz")
        got = np.load(path)
        for k in got.files:
            out[f"{k}_{mode}"] = got[k]
        os.remove(path)
    for idx, (case, inp, w, bias) in enumerate(inputs.convt_cases()):
        W = oracle.ref_weight_quantize(w)
        pre = f"c{idx}_"
        out.update({pre + "params": np.array([case[k] for k in inputs.CONVT_KEYS], np.int32),
                    pre + "inputs_sha": np.frombuffer(inputs.sha(inp, w, bias), np.uint8),
                    pre + "wdata": W.data, pre + "wscale": W.scale, pre + "wcolsum": W.colsum})
    return out


def conv1():
    """dacvae.c:983-1008 is the skip copy plus these ops.c calls."""
    hidden, skip, w, bias = inputs.conv1_case()
    W = oracle.ref_weight_quantize(w)
    q, s, z = oracle.ref_quantize_rows(hidden)
    y1, _ = oracle.ref_linear_ex(q, s, z, W, bias, y=skip.copy(), accumulate=True)
    (q1, s1, z1), _, (q2, s2, z2) = oracle.ref_quantize_rows_residual(hidden)
    y2, _ = oracle.ref_linear_ex(q1, s1, z1, W, bias, y=skip.copy(), accumulate=True)
    y2, _ = oracle.ref_linear_ex(q2, s2, z2, W, None, y=y2, accumulate=True)
    return {"inputs_sha": np.frombuffer(inputs.sha(hidden, skip, w, bias), np.uint8),
            "wdata": W.data, "wscale": W.scale, "wcolsum": W.colsum,
            "out_single": y1, "out_two_term": y2}


DIT_BLOCK_CASES = [(11, 2, 40, 12, 1), (12, 2, 70, 9, 2)]  # seed, B, S, C, context_batch


def dit_block_child():
    """Child process with IRO_INT8_RESIDUAL unset: the reference's default
    policy (two-term W2, dit.c:429-436)."""
    res = {}
    for i, (seed, B, S, C, cb) in enumerate(DIT_BLOCK_CASES):
        x, cond, ck, cv, mask, adaln, qn, kn, ws = inputs.dit_block_case(seed, B, S, C, cb)
        W = [oracle.ref_weight_quantize(w) for w in ws]
        res[f"c{i}_out"] = oracle.ref_dit_block(x, cond, ck, cv, mask, cb, B, S, C, adaln, qn,
                                                kn, W)
        res[f"c{i}_inputs_sha"] = np.frombuffer(
            inputs.sha(x, cond, ck, cv, mask, *adaln, qn, kn, *ws), np.uint8)
        res[f"c{i}_case"] = np.array([seed, B, S, C, cb], np.int32)
    np.savez(os.path.join(HERE, "_tmp_dit_block.npz"), **res)


DIT_BLOCK_RESID_CASES = [(31, 2, 40, 12, 1, 7), (32, 1, 70, 9, 1, 15), (33, 2, 36, 20, 2, 2)]
# seed, B, S, C, context_batch, IRO_INT8_RESIDUAL


def dit_block_resid_child(idx):
    """Child process with IRO_INT8_RESIDUAL set for one case (the reference
    reads it once per process)."""
    seed, B, S, C, cb, mask = DIT_BLOCK_RESID_CASES[idx]
    x, cond, ck, cv, mask_, adaln, qn, kn, ws = inputs.dit_block_case(seed, B, S, C, cb)
    W = [oracle.ref_weight_quantize(w) for w in ws]
    out = oracle.ref_dit_block(x, cond, ck, cv, mask_, cb, B, S, C, adaln, qn, kn, W)
    np.savez(os.path.join(HERE, f"_tmp_dit_block_resid_{idx}.npz"), out=out,
             case=np.array([seed, B, S, C, cb, mask], np.int32),
             inputs_sha=np.frombuffer(inputs.sha(x, cond, ck, cv, mask_, *adaln, qn, kn, *ws),
                                      np.uint8))


def dit_block_resid():
    res = {}
    for i, case in enumerate(DIT_BLOCK_RESID_CASES):
        e = dict(os.environ)
        e["IRO_INT8_RESIDUAL"] = str(case[5])
        subprocess.run([sys.executable, __file__, "--dit-block-resid-child", str(i)], check=True,
                       env=e)
        path = os.path.join(HERE, f"_tmp_dit_block_resid_{i}.npz")
        g = dict(np.load(path))
        os.remove(path)
        for k, v in g.items():
            res[f"c{i}_{k}"] = v
    return res


# seed, B, S, C, context_batch, IRO_INT8_MASK, IRO_INT8_EMULATE
DIT_BLOCK_DIAG_CASES = [(41, 2, 20, 12, 1, 0, 0), (42, 1, 40, 9, 1, 5, 0),
                        (43, 2, 20, 20, 2, 10, 0), (44, 2, 20, 12, 1, 15, 1),
                        (45, 1, 40, 9, 1, 15, 2), (46, 2, 20, 20, 2, 6, 2)]


def dit_block_diag_child(idx, path):
    """Child process with IRO_INT8_MASK / IRO_INT8_EMULATE set for one case
    (the reference reads both once per process, dit.c:284-304) and
    IRO_INT8_RESIDUAL unset (default two-term W2)."""
    seed, B, S, C, cb, imask, emu = DIT_BLOCK_DIAG_CASES[idx]
    x, cond, ck, cv, mask, adaln, qn, kn, ws = inputs.dit_block_case(seed, B, S, C, cb)
    W = [oracle.ref_weight_quantize(w) for w in ws]
    out = oracle.ref_dit_block(x, cond, ck, cv, mask, cb, B, S, C, adaln, qn, kn, W,
                               fp32_weights=ws)
    np.savez(path, out=out, case=np.array(DIT_BLOCK_DIAG_CASES[idx], np.int32),
             inputs_sha=np.frombuffer(inputs.sha(x, cond, ck, cv, mask, *adaln, qn, kn, *ws),
                                      np.uint8))


def run_dit_block_diag_child(idx, path):
    """Runs dit_block_diag_child(idx) in a fresh interpreter with the case's
    switches in its environment."""
    e = dict(os.environ)
    e.pop("IRO_INT8_RESIDUAL", None)
    e["IRO_INT8_MASK"] = str(DIT_BLOCK_DIAG_CASES[idx][5])
    e["IRO_INT8_EMULATE"] = str(DIT_BLOCK_DIAG_CASES[idx][6])
    subprocess.run([sys.executable, os.path.abspath(__file__), "--dit-block-diag-child", str(idx),
                    path], check=True, env=e)


def dit_block_diag():
    res = {}
    for i in range(len(DIT_BLOCK_DIAG_CASES)):
        path = os.path.join(HERE, f"_tmp_dit_block_diag_{i}.npz")
        run_dit_block_diag_child(i, path)
        g = dict(np.load(path))
        os.remove(path)
        for k, v in g.items():
            res[f"c{i}_{k}"] = v
    return res


def dit_block():
    e = dict(os.environ)
    e.pop("IRO_INT8_RESIDUAL", None)
    subprocess.run([sys.executable, __file__, "--dit-block-child", "x"], check=True, env=e)
    path = os.path.join(HERE, "_tmp_dit_block.npz")
    got = dict(np.load(path))
    os.remove(path)
    return got


# seed, layers, R, cfg, S, C; then the step's t, t_next and CFG scales, and the
# sampler's steps, init_scale, cfg_min_t, cfg_max_t.
DIT_STEP_CASE = (21, 2, 1, 3, 32, 16)
DIT_STEP_T = (1.0, 0.5, (2.0, 1.5))
DIT_SAMPLE = (2, 1.0, 0.6, 1.0)


def dit_step_child():
    seed, layers, R, cfg, S, C = DIT_STEP_CASE
    state, ck, cv, mask, blocks, head = inputs.dit_model_case(*DIT_STEP_CASE)
    bw = [(a, q, k, [oracle.ref_weight_quantize(w) for w in ws]) for a, q, k, ws in blocks]
    t, tn, sc = DIT_STEP_T
    steps, init, lo, hi = DIT_SAMPLE
    flat = [state, *ck, *cv, mask] + [a for b in blocks for a in (*b[0], b[1], b[2], *b[3])]
    res = {"case": np.array(DIT_STEP_CASE, np.int32),
           "step_args": np.array([t, tn, *sc], np.float32),
           "sample_args": np.array([steps, init, lo, hi], np.float32),
           "inputs_sha": np.frombuffer(inputs.sha(*flat, *head.values()), np.uint8),
           "step_out": oracle.ref_dit_euler_step(state, ck, cv, mask, bw, head, R, cfg, S, C, t,
                                                 tn, sc),
           "sample_out": oracle.ref_dit_sample_euler(state, ck, cv, mask, bw, head, R, cfg, S, C,
                                                     steps, init, lo, hi, sc)}
    np.savez(os.path.join(HERE, "_tmp_dit_step.npz"), **res)


def dit_step():
    e = dict(os.environ)
    e.pop("IRO_INT8_RESIDUAL", None)
    subprocess.run([sys.executable, __file__, "--dit-step-child", "x"], check=True, env=e)
    path = os.path.join(HERE, "_tmp_dit_step.npz")
    got = dict(np.load(path))
    os.remove(path)
    return got


def main():
    if len(sys.argv) > 3 and sys.argv[1] == "--dit-block-diag-child":
        dit_block_diag_child(int(sys.argv[2]), sys.argv[3])
        return
    if len(sys.argv) > 2 and sys.argv[1] == "--dit-block-resid-child":
        dit_block_resid_child(int(sys.argv[2]))
        return
    if len(sys.argv) > 2 and sys.argv[1] == "--dit-step-child":
        dit_step_child()
        return
    if len(sys.argv) > 2 and sys.argv[1] == "--dit-block-child":
        dit_block_child()
        return
    if len(sys.argv) > 2 and sys.argv[1] == "--swiglu-child":
        dit_swiglu_child(sys.argv[2])
        return
    if len(sys.argv) > 2 and sys.argv[1] == "--convt-child":
        convt_child(sys.argv[2])
        return
    only = set(sys.argv[1:])
    for name, fn in (("int8_ops", int8_ops), ("residual", residual), ("conv7", conv7),
                     ("sym_quant", sym), ("dit_swiglu", dit_swiglu), ("convt", convt),
                     ("conv1", conv1), ("dit_block", dit_block),
                     ("dit_step", dit_step), ("dit_block_resid", dit_block_resid),
                     ("dit_block_diag", dit_block_diag)):
        if only and name not in only:
            continue
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **fn())
        print("wrote", name)


if __name__ == "__main__":
    main()
