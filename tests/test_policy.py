"""The int8 policy switches (iro_policy_*, csrc/policy.cu) against the
reference's own readers (dit.c:429-436, dacvae.c:43-71, through
oracle/ref_*_shim.c), one child process per environment setting because the
reference caches each switch per process.  CPU only."""
import json
import os
import subprocess
import sys

import pytest

import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

SETTINGS = [None, "", "0", "15", "0x3", "9", "022", "junk", "255"]

CHILD = r"""
import ctypes, json, os, sys
sys.path[:0] = [os.path.join(sys.argv[1], "irodori-c_b200"), os.path.join(sys.argv[1], "oracle")]
import iro_b200 as iro
import oracle
L = iro.lib()
out = {"dit": L.iro_policy_dit_residual_mask(),
       "dit_diag": [L.iro_policy_dit_fp32_groups(), L.iro_policy_dit_emulate()],
       "codec": [L.iro_policy_codec_int8_mask(), L.iro_policy_codec_residual_mask(),
                 L.iro_policy_codec_residual_stages()],
       "decide": [[L.iro_policy_codec_residual(st, g) for g in (1, 2, 4, 8)] for st in range(4)]}
if oracle.ref_available("dit"):
    R = oracle.ref_lib("dit")
    out["ref_dit"] = R.ref_dit_residual_mask()
    out["ref_dit_diag"] = [15 & ~R.ref_dit_int8_mask(), R.ref_dit_int8_emulate()]
if oracle.ref_available("codec"):
    R = oracle.ref_lib("codec")
    m, r, s = ctypes.c_int(), ctypes.c_int(), ctypes.c_int()
    R.ref_codec_policy(ctypes.byref(m), ctypes.byref(r), ctypes.byref(s))
    out["ref_codec"] = [m.value, r.value, s.value]
print(json.dumps(out))
"""

NAMES = ["IRO_INT8_RESIDUAL", "IRO_CODEC_INT8_MASK", "IRO_CODEC_INT8_RESIDUAL",
         "IRO_CODEC_INT8_RESIDUAL_STAGES", "IRO_INT8_MASK", "IRO_INT8_EMULATE"]


def run_child(value):
    env = dict(os.environ)
    for n in NAMES:
        env.pop(n, None)
        if value is not None:
            env[n] = value
    r = subprocess.run([sys.executable, "-c", CHILD, ROOT], env=env, capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


@pytest.mark.parametrize("value", SETTINGS)
def test_policy_switches_match_reference(value):
    out = run_child(value)
    def c_strtol(v):
        # strtol(v, NULL, 0) for the settings above: 0x hex, leading-zero
        # octal, decimal; no digits parse as 0.
        if v.lower().startswith("0x"):
            return int(v, 16)
        if v.startswith("0") and len(v) > 1:
            return int(v, 8)
        return int(v) if v.isdigit() else 0

    expect = (lambda d: d if value in (None, "") else c_strtol(value) & 15)
    assert out["dit"] == expect(8)
    # IRO_INT8_MASK masked to 4 bits (default 15), complemented into the
    # block's fp32 groups; IRO_INT8_EMULATE unmasked (default 0).
    assert out["dit_diag"] == [15 & ~expect(15),
                               0 if value in (None, "") else c_strtol(value)]
    if "ref_dit_diag" in out:
        assert out["dit_diag"] == out["ref_dit_diag"]
    assert out["codec"] == [expect(15), expect(12), expect(8)]
    if "ref_dit" in out:
        assert out["dit"] == out["ref_dit"]
    if "ref_codec" in out:
        assert out["codec"] == out["ref_codec"]
    resid, stages = out["codec"][1], out["codec"][2]
    for st in range(4):
        for gi, g in enumerate((1, 2, 4, 8)):
            want = bool(resid & g) and (g in (1, 2) or bool((stages >> st) & 1))
            assert out["decide"][st][gi] == int(want), (st, g)
