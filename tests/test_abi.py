"""CPU checks of the C ABI library: it loads without a GPU, exports every
symbol the public header declares, and fails loudly (no CPU fallback) when
no device is usable."""
import ctypes
import os

import pytest

import iro_b200 as iro


def test_library_exports_every_header_symbol():
    L = ctypes.CDLL(iro.LIB_PATH)
    declared = iro.header_symbols()
    assert len(declared) >= 40
    missing = [s for s in declared if not hasattr(L, s)]
    assert not missing, f"declared but not exported: {missing}"
    # The binding covers the header exactly.
    assert set(declared) == set(iro.SIGNATURES), set(declared) ^ set(iro.SIGNATURES)


def test_no_cpu_fallback_without_device():
    if iro.device_count() > 0:
        pytest.skip("a GPU is present")
    L = iro.lib()
    assert L.iro_int8_fast_available() == 0
    assert L.iro_int8_prepare_backend() is None
    assert L.iro_cuda_init(0) == iro.IRO_ERR_NO_DEVICE
    assert L.iro_int8_selfcheck() == -1
    import numpy as np
    x = np.ones((2, 8), np.float32)
    q = np.full((2, 8), 7, np.uint8)
    s = np.zeros(2, np.float32)
    z = np.zeros(2, np.int32)
    L.iro_cuda_last_error()
    L.iro_int8_quantize_rows(iro._p(x), 2, 8, iro._p(q), iro._p(s), iro._p(z))
    assert L.iro_cuda_last_error() < 0
    assert (q == 7).all(), "outputs must stay untouched without a device"
    w = iro.IroInt8Weight()
    assert L.iro_int8_weight_quantize(ctypes.byref(w), iro._p(x), 2, 8) == -1
    assert not w.data


def test_conv_output_length_matches_reference_rule():
    # dacvae.c:340-348
    assert iro.conv1d_out_len(48000, 7, 1, 1, 3) == 48000
    assert iro.conv1d_out_len(100, 7, 1, 9, 27) == 100
    assert iro.conv1d_out_len(10, 7, 2, 1, 0) == 2
    assert iro.conv1d_out_len(3, 7, 1, 1, 0) < 0


def test_built_for_sm100a():
    """The build recipe compiles and links every object for sm_100a only
    (the flags, not the built bytes, are checked)."""
    mk = open(os.path.join(os.path.dirname(iro.__file__), "Makefile")).read()
    arch = [ln for ln in mk.splitlines() if ln.startswith("ARCH")]
    assert arch and arch[0].split(":=", 1)[1].split() == ["-gencode",
                                                          "arch=compute_100a,code=sm_100a"]
    rules = [ln.strip() for ln in mk.splitlines() if ln.strip().startswith("$(NVCC)")]
    assert len(rules) == 2 and all("$(ARCH)" in r for r in rules)
    assert "-arch" not in mk.replace("ARCH", "")


def test_header_has_reference_citations():
    txt = open(iro.HEADER_PATH).read()
    for cite in ("ops.c:259-293", "ops.c:321-348", "ops.c:450-491", "ops.c:427-442",
                 "ops.c:375-398", "dacvae.c:543-688", "dit.c:785-792", "dit.c:913-969"):
        assert cite in txt, cite


def test_wrappers_do_not_shadow_ctypes():
    """The bindings import ctypes as `C`; a parameter of that name inside a
    function that also calls C.byref/C.c_float breaks only at run time."""
    import ast
    src = open(os.path.join(os.path.dirname(iro.__file__), "iro_b200.py")).read()
    bad = []
    for node in ast.walk(ast.parse(src)):
        if isinstance(node, (ast.FunctionDef, ast.Lambda)):
            a = node.args
            names = {x.arg for x in a.args + a.kwonlyargs + a.posonlyargs}
            if "C" in names and any(isinstance(n, ast.Attribute) and isinstance(n.value, ast.Name)
                                    and n.value.id == "C" for n in ast.walk(node)):
                bad.append(getattr(node, "name", "lambda"))
    assert not bad, bad


def test_c_dropin_binary_binds_the_int8_api_to_this_library():
    """oracle/_ref/test_int8_ops_b200 (the reference's C test): its int8 calls
    are undefined in the executable and its DT_NEEDED names this library;
    ops.c's own int8 definitions are present only under renamed symbols."""
    import oracle
    import subprocess
    binp = os.path.join(oracle.REF_DIR, "test_int8_ops_b200")
    if not os.path.exists(binp):
        pytest.skip("drop-in test binary not built")
    und = subprocess.run(["nm", "-D", "--undefined-only", binp], capture_output=True,
                         text=True).stdout
    for f in ("iro_int8_weight_quantize", "iro_int8_quantize_rows", "iro_int8_linear",
              "iro_int8_selfcheck", "iro_int8_fast_available", "iro_int8_weight_free"):
        assert f" {f}\n" in und, f
    syms = subprocess.run(["nm", binp], capture_output=True, text=True).stdout
    assert "refops_iro_int8_linear_ex" in syms
    dyn = subprocess.run(["readelf", "-d", binp], capture_output=True, text=True).stdout
    assert "libirodori_b200.so" in dyn


def _layout_probe(src, incs, tmp):
    import subprocess
    c = os.path.join(tmp, "probe.c")
    exe = os.path.join(tmp, "probe")
    open(c, "w").write(src)
    subprocess.run(["gcc", "-std=c11", *[f"-I{i}" for i in incs], c, "-o", exe], check=True,
                   capture_output=True)
    return subprocess.run([exe], capture_output=True, text=True, check=True).stdout.split()


def test_int8_container_layouts_match_the_reference(tmp_path):
    """IroDiTInt8HostLayer / IroDACVAEInt8Host have the size and member
    offsets of the reference's IroDiTInt8Layer (dit.h:53-55) and
    IroDACVAEInt8 (dacvae.h:52-67), so an engine passes its own copies."""
    # The reference tree beside this repository (as __graft_entry__ finds it).
    ref = os.environ.get("IRO_REFERENCE_DIR",
                         os.path.join(os.path.dirname(os.path.dirname(iro.HERE)), "reference"))
    if not os.path.isfile(os.path.join(ref, "dit.h")):
        pytest.skip("reference headers not present")
    body = r"""
#include <stddef.h>
#include <stdio.h>
int main(void) {
  printf("%zu %zu %zu %zu ", sizeof(DL), offsetof(DL, gate), offsetof(DL, w2), offsetof(DL, w3));
  printf("%zu %zu %zu %zu\n", sizeof(CQ), offsetof(CQ, stage), offsetof(CQ, stage[1].residual[2].conv1),
         offsetof(CQ, bytes));
  return 0;
}
"""
    theirs = _layout_probe('#include "dit.h"\n#include "dacvae.h"\ntypedef IroDiTInt8Layer DL;\n'
                           'typedef IroDACVAEInt8 CQ;\n' + body, [ref], str(tmp_path))
    inc = os.path.dirname(iro.HEADER_PATH)
    ours = _layout_probe('#include <stdint.h>\n#include "irodori_b200.h"\n'
                         'typedef IroDiTInt8HostLayer DL;\ntypedef IroDACVAEInt8Host CQ;\n' + body,
                         [inc], str(tmp_path))
    assert ours == theirs, (ours, theirs)
