"""Record tests/golden/dit_cfg3.npz: the reference's own 8-step Euler
sampler (sampler.c:241-297, with the CFG window of generate.c:416-422) at
config 3's row geometry -- 12 layers, 8 requests x 4 CFG rows x 750 frames,
128 context tokens -- for the sampled requests inputs.CFG3_SAMPLED, at the
reference's fixed dimensions (1280 / 20 heads / 3680).

    make -C oracle ref REF_DIR=<reference tree>
    python tests/golden/make_dit_cfg3.py

The reference code runs from oracle/_ref/libiro_ref_dit_vec.so: ops.c, dit.c
and the shim at -O3 for this host with IEEE semantics (-ffp-contract=off
-fno-fast-math), bit-identical to the -O2 parity build
(tests/test_oracle.py::test_dit_branch_split_and_vec_build_agree) and about
ten times faster on the integer GEMMs.  Each step's CFG branches run as
independent batch-1 forwards in threads (oracle.ref_dit_branch_velocity;
bit-identical to one batched call).  Stored per sampled request: the guided
velocity of every step (the state update is state += guided * dt in
float32, so the states along the reference's trajectory follow from the
seeded noise) and the final latent.  The inputs are regenerated from seeds;
their SHA-256 is stored.

Also stored: the reference's own rounding envelope on the first sampled
request -- how far its guided velocity at each step moves when that step's
input state is perturbed by one ulp (a random sign per element), and how far
the final latent moves when the sampler starts from one-ulp-perturbed noise.
An implementation that is not bit-identical to the reference (another
summation order, another expf) lands inside an envelope of this size.
"""
import os
import sys
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, HERE)

import oracle  # noqa: E402
import inputs  # noqa: E402


def main():
    c, smp = inputs.CFG3, inputs.CFG3_SAMPLER
    t0 = time.time()
    state, ck, cv, mask, blocks, head = inputs.dit_cfg3_case()
    sha = inputs.dit_sha(state, ck, cv, mask, blocks, head)
    bw = [(a, q, k, [oracle.weight_quantize(w) for w in ws]) for a, q, k, ws in blocks]
    print(f"inputs {time.time() - t0:.1f} s", flush=True)
    cfg, S, C = c["cfg"], c["S"], c["C"]
    pool = ThreadPoolExecutor(max(1, min(os.cpu_count() or 1, cfg * len(inputs.CFG3_SAMPLED))))
    outer = ThreadPoolExecutor(len(inputs.CFG3_SAMPLED) + 1)
    f = np.float32
    rng = np.random.default_rng(11)

    def ulp(x):
        return (x * (1 + rng.choice([-1, 1], x.shape) * 2.0 ** -23)).astype(np.float32)

    def sample(r, st):
        return oracle.ref_dit_sample_request(
            st, [k[r:r + 1] for k in ck], [v[r:r + 1] for v in cv],
            mask[r * cfg:(r + 1) * cfg], bw, head, cfg, S, C, smp["steps"], smp["init_scale"],
            smp["cfg_min_t"], smp["cfg_max_t"], smp["scales"], kind="dit_vec", pool=pool)

    r0 = inputs.CFG3_SAMPLED[0]
    perturbed_noise = ulp(state[r0])
    jobs = [outer.submit(sample, r, state[r]) for r in inputs.CFG3_SAMPLED]
    jobs.append(outer.submit(sample, r0, perturbed_noise))
    res = [j.result() for j in jobs[:-1]]
    fin_p = jobs[-1].result()[0]
    print(f"reference sampler {time.time() - t0:.1f} s; CFG rows per step {res[0][2]}",
          flush=True)

    # The per-step rounding envelope on the first sampled request.
    ck0, cv0 = [k[r0:r0 + 1] for k in ck], [v[r0:r0 + 1] for v in cv]
    m0 = mask[r0 * cfg:(r0 + 1) * cfg]
    vel0 = res[0][1]
    x = state[r0].copy()
    env_max, env_mean = [], []
    for k in range(smp["steps"]):
        t = (f(1) - f(k) / f(smp["steps"])) * f(smp["init_scale"])
        tn = (f(1) - f(k + 1) / f(smp["steps"])) * f(smp["init_scale"])
        nb = res[0][2][k]
        xp = ulp(x)
        v = list(pool.map(lambda b: oracle.ref_dit_branch_velocity(
            xp, ck0, cv0, m0[b], bw, head, S, C, t, kind="dit_vec"), range(nb)))
        d = np.abs(oracle.ref_cfg_guided(np.stack(v), smp["scales"]) - vel0[k])
        env_max.append(float(d.max()))
        env_mean.append(float(d.mean()))
        print(f"envelope step {k}: max {env_max[-1]:.3e} mean {env_mean[-1]:.3e}", flush=True)
        x = x + vel0[k] * f(tn - t)
    d = np.abs(fin_p - res[0][0])
    env_final = [float(d.max()), float(d.mean())]
    print(f"envelope final latent: max {env_final[0]:.3e} mean {env_final[1]:.3e} "
          f"({time.time() - t0:.1f} s)", flush=True)
    np.savez_compressed(
        os.path.join(HERE, "dit_cfg3.npz"),
        case=np.array([c["seed"], c["layers"], c["R"], cfg, S, C], np.int64),
        sampled=np.array(inputs.CFG3_SAMPLED, np.int64),
        sampler=np.array([smp["steps"], smp["init_scale"], smp["cfg_min_t"], smp["cfg_max_t"],
                          *smp["scales"]], np.float64),
        rows_per_step=np.array(res[0][2], np.int64),
        inputs_sha=np.frombuffer(sha, np.uint8),
        velocity=np.stack([r[1] for r in res]).astype(np.float32),
        final=np.stack([r[0] for r in res]).astype(np.float32),
        env_velocity_max=np.array(env_max), env_velocity_mean=np.array(env_mean),
        env_final=np.array(env_final))


if __name__ == "__main__":
    main()
