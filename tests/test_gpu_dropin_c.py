"""The boundary from C: the reference's own test of the int8 API
(tests/test_int8_ops.c), compiled unchanged against the reference's ops.h
and linked with ops.c whose int8 section is renamed away, so every iro_int8_*
call it makes goes to libirodori_b200.so (oracle/Makefile `dropin`, built by
__graft_entry__.build() where the reference tree is present).  It checks the
weight reconstruction bound and colsums, exact integer sums against its own
triple loop, cross-M determinism, the float error against the FP32 oracle,
the selfcheck and the degenerate rows, and prints "int8 ops: PASS"."""
import os
import subprocess

import pytest

import oracle

pytestmark = pytest.mark.gpu

BIN = os.path.join(oracle.REF_DIR, "test_int8_ops_b200")


@pytest.mark.skipif(not os.path.exists(BIN), reason="drop-in test binary not built")
def test_reference_c_test_passes_against_the_b200_library():
    r = subprocess.run([BIN], capture_output=True, text=True, timeout=600)
    print(r.stdout)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "int8 ops: PASS" in r.stdout
    assert "FAIL" not in r.stdout
