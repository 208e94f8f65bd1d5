"""ctypes/numpy front end of the CPU checker.  TEST INFRASTRUCTURE ONLY.

Two libraries sit behind this module:

* ``liboracle.so`` — the C restatement in ``iro_oracle.c`` (always built);
* ``_ref/libiro_ref_*.so`` — the reference's own ``ops.c`` / ``dacvae.c`` /
  ``dit.c`` compiled from its sources (present where the reference tree was
  available at build time; the GPU box receives the prebuilt files).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU legs import this.
The product library never does.
"""
from __future__ import annotations

import ctypes as C
import os
import platform

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")

_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_vp = C.c_void_p


def _ptr(a):
    return None if a is None else a.ctypes.data_as(C.c_void_p)


_lib = None


def lib():
    """The C restatement (built by ``make -C oracle``)."""
    global _lib
    if _lib is None:
        path = os.path.join(HERE, "liboracle.so")
        if not os.path.exists(path):
            raise RuntimeError("oracle/liboracle.so is not built (make -C oracle)")
        L = C.CDLL(path)
        for name in ("oracle_quantize_rows", "oracle_quantize_rows_sym"):
            getattr(L, name).argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp]
            getattr(L, name).restype = None
        L.oracle_weight_quantize.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp]
        L.oracle_weight_quantize.restype = C.c_int
        L.oracle_weight_quantize_transposed.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp]
        L.oracle_weight_quantize_transposed.restype = C.c_int
        L.oracle_quantize_rows_residual.argtypes = [_vp, C.c_int, C.c_int] + [_vp] * 7
        L.oracle_quantize_rows_residual.restype = None
        L.oracle_gemm_u8s8.argtypes = [_vp, _vp, _vp, C.c_int, C.c_int, C.c_int]
        L.oracle_gemm_u8s8.restype = None
        L.oracle_linear_ex.argtypes = [_vp, _vp, _vp, _vp, _vp, _vp, C.c_int, C.c_int,
                                       _vp, _vp, C.c_int, _vp, C.c_int]
        L.oracle_linear_ex.restype = None
        L.oracle_epilogue.argtypes = [_vp, _vp, _vp, _vp, _vp, C.c_int, _vp, _vp,
                                      C.c_int, C.c_int]
        L.oracle_epilogue.restype = None
        L.oracle_silu_mul.argtypes = [_vp, _vp, C.c_size_t]
        L.oracle_silu_mul.restype = None
        L.oracle_conv1d_out_len.argtypes = [C.c_int] * 5
        L.oracle_conv1d_out_len.restype = C.c_int
        L.oracle_conv1d_int8.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp, C.c_int,
                                         C.c_int, C.c_int, C.c_int, C.c_int, _vp, C.c_int,
                                         _vp, _vp, _vp, _vp]
        L.oracle_conv1d_int8.restype = C.c_int
        L.oracle_swiglu.argtypes = [_vp, C.c_int, C.c_int, C.c_int] + [_vp] * 12 + [
            C.c_int, _vp, _vp]
        L.oracle_swiglu.restype = C.c_int
        L.oracle_selfcheck_case.argtypes = [_vp, _vp, _vp]
        L.oracle_selfcheck_case.restype = None
        L.oracle_convtranspose1d_out_len.argtypes = [C.c_int] * 5
        L.oracle_convtranspose1d_out_len.restype = C.c_int
        L.oracle_convtranspose1d_int8.argtypes = [_vp, C.c_int, C.c_int, C.c_int, _vp, _vp, _vp,
                                                  C.c_int, C.c_int, C.c_int, C.c_int, _vp,
                                                  C.c_int, _vp]
        L.oracle_convtranspose1d_int8.restype = C.c_int
        L.oracle_codec_conv1.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp, _vp, _vp,
                                         C.c_int, _vp]
        L.oracle_codec_conv1.restype = C.c_int
        _lib = L
    return _lib


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


class Weight:
    """Host quantised weight: data int8 [N,K], scale f32 [N], colsum i32 [N]."""

    def __init__(self, data, scale, colsum):
        self.data = _c(data, np.int8)
        self.scale = _c(scale, np.float32)
        self.colsum = _c(colsum, np.int32)
        self.N, self.K = self.data.shape


def weight_quantize(w):
    w = _c(w, np.float32)
    N, K = w.shape
    d = np.empty((N, K), np.int8)
    s = np.empty(N, np.float32)
    c = np.empty(N, np.int32)
    rc = lib().oracle_weight_quantize(_ptr(w), N, K, _ptr(d), _ptr(s), _ptr(c))
    if rc != 0:
        raise ValueError("weight quantize failed")
    return Weight(d, s, c)


def weight_quantize_transposed(w_kn):
    w_kn = _c(w_kn, np.float32)
    K, N = w_kn.shape
    d = np.empty((N, K), np.int8)
    s = np.empty(N, np.float32)
    c = np.empty(N, np.int32)
    rc = lib().oracle_weight_quantize_transposed(_ptr(w_kn), N, K, _ptr(d), _ptr(s), _ptr(c))
    if rc != 0:
        raise ValueError("weight quantize failed")
    return Weight(d, s, c)


def quantize_rows(x, symmetric=False):
    x = _c(x, np.float32)
    M, K = x.shape
    q = np.empty((M, K), np.uint8)
    s = np.empty(M, np.float32)
    z = np.empty(M, np.int32)
    fn = lib().oracle_quantize_rows_sym if symmetric else lib().oracle_quantize_rows
    fn(_ptr(x), M, K, _ptr(q), _ptr(s), _ptr(z))
    return q, s, z


def quantize_rows_residual(x):
    x = _c(x, np.float32)
    M, K = x.shape
    q1 = np.empty((M, K), np.uint8); s1 = np.empty(M, np.float32); z1 = np.empty(M, np.int32)
    r = np.empty((M, K), np.float32)
    q2 = np.empty((M, K), np.uint8); s2 = np.empty(M, np.float32); z2 = np.empty(M, np.int32)
    lib().oracle_quantize_rows_residual(_ptr(x), M, K, _ptr(q1), _ptr(s1), _ptr(z1), _ptr(r),
                                        _ptr(q2), _ptr(s2), _ptr(z2))
    return (q1, s1, z1), r, (q2, s2, z2)


def gemm_u8s8(a, b):
    a = _c(a, np.uint8); b = _c(b, np.int8)
    M, K = a.shape
    N = b.shape[0]
    c = np.empty((M, N), np.int32)
    lib().oracle_gemm_u8s8(_ptr(a), _ptr(b), _ptr(c), M, N, K)
    return c


def linear_ex(q, scale, zero, w: Weight, bias=None, y=None, accumulate=False):
    q = _c(q, np.uint8); scale = _c(scale, np.float32); zero = _c(zero, np.int32)
    M = q.shape[0]
    if y is None:
        y = np.zeros((M, w.N), np.float32)
    else:
        y = _c(y, np.float32).copy()
    work = np.empty((M, w.N), np.int32)
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_linear_ex(_ptr(q), _ptr(scale), _ptr(zero), _ptr(w.data), _ptr(w.scale),
                           _ptr(w.colsum), w.N, w.K, _ptr(b), _ptr(y), M, _ptr(work),
                           int(bool(accumulate)))
    return y, work


def epilogue(work, scale, zero, w: Weight, bias=None, y=None, accumulate=False):
    work = _c(work, np.int32)
    M, N = work.shape
    y = np.zeros((M, N), np.float32) if y is None else _c(y, np.float32).copy()
    b = None if bias is None else _c(bias, np.float32)
    lib().oracle_epilogue(_ptr(work), _ptr(_c(scale, np.float32)), _ptr(_c(zero, np.int32)),
                          _ptr(w.scale), _ptr(w.colsum), N, _ptr(b), _ptr(y), M,
                          int(bool(accumulate)))
    return y


def silu_mul(x, gate):
    x = _c(x, np.float32).copy(); gate = _c(gate, np.float32)
    lib().oracle_silu_mul(_ptr(x), _ptr(gate), x.size)
    return x


def conv1d_out_len(T_in, kernel, stride=1, dilation=1, padding=0):
    return lib().oracle_conv1d_out_len(T_in, kernel, stride, dilation, padding)


def conv1d_int8(inp, w: Weight, kernel, stride=1, dilation=1, padding=0, bias=None,
                residual=False, want_cols=False):
    """inp: time-major [T_in, C]; w: [N, kernel*C].  Returns out [T_out, N]
    (and the first-term im2col codes and row parameters with want_cols)."""
    inp = _c(inp, np.float32)
    T_in, Cin = inp.shape
    T_out = conv1d_out_len(T_in, kernel, stride, dilation, padding)
    if T_out <= 0:
        raise ValueError("empty convolution output")
    out = np.empty((T_out, w.N), np.float32)
    cols = np.empty((T_out, kernel * Cin), np.uint8) if want_cols else None
    sc = np.empty(T_out, np.float32) if want_cols else None
    zr = np.empty(T_out, np.int32) if want_cols else None
    b = None if bias is None else _c(bias, np.float32)
    rc = lib().oracle_conv1d_int8(_ptr(inp), T_in, Cin, _ptr(w.data), _ptr(w.scale),
                                  _ptr(w.colsum), w.N, kernel, stride, dilation, padding,
                                  _ptr(b), int(bool(residual)), _ptr(out), _ptr(cols),
                                  _ptr(sc), _ptr(zr))
    if rc != T_out:
        raise RuntimeError("oracle conv failed")
    if want_cols:
        return out, cols, sc, zr
    return out


def swiglu(x, w1: Weight, w3: Weight, w2: Weight, b1=None, b3=None, b2=None,
           residual_w2=False, want_hidden=False):
    x = _c(x, np.float32)
    M, D = x.shape
    H = w1.N
    out = np.empty((M, w2.N), np.float32)
    hid = np.empty((M, H), np.float32) if want_hidden else None
    bs = [None if b is None else _c(b, np.float32) for b in (b1, b3, b2)]
    rc = lib().oracle_swiglu(_ptr(x), M, D, H,
                             _ptr(w1.data), _ptr(w1.scale), _ptr(w1.colsum), _ptr(bs[0]),
                             _ptr(w3.data), _ptr(w3.scale), _ptr(w3.colsum), _ptr(bs[1]),
                             _ptr(w2.data), _ptr(w2.scale), _ptr(w2.colsum), _ptr(bs[2]),
                             int(bool(residual_w2)), _ptr(out), _ptr(hid))
    if rc != 0:
        raise RuntimeError("oracle swiglu failed")
    return (out, hid) if want_hidden else out


def selfcheck_case():
    a = np.empty(3 * 64, np.uint8); b = np.empty(5 * 64, np.int8); want = np.empty(15, np.int32)
    lib().oracle_selfcheck_case(_ptr(a), _ptr(b), _ptr(want))
    return a.reshape(3, 64), b.reshape(5, 64), want.reshape(3, 5)


# ---------------------------------------------------------------------------
# The reference's own code, compiled from its sources into _ref/.


class _IroInt8Weight(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scale", C.c_void_p), ("colsum", C.c_void_p),
                ("N", C.c_int), ("K", C.c_int)]


def ref_available(kind="ieee"):
    return os.path.exists(os.path.join(REF_DIR, f"libiro_ref_{kind}.so"))


_ref_libs = {}


def _bind_ops(L):
    L.iro_int8_weight_quantize.argtypes = [C.POINTER(_IroInt8Weight), _vp, C.c_int, C.c_int]
    L.iro_int8_weight_quantize.restype = C.c_int
    L.iro_int8_weight_quantize_transposed.argtypes = [C.POINTER(_IroInt8Weight), _vp,
                                                      C.c_int, C.c_int]
    L.iro_int8_weight_quantize_transposed.restype = C.c_int
    L.iro_int8_weight_free.argtypes = [C.POINTER(_IroInt8Weight)]
    L.iro_int8_weight_free.restype = None
    L.iro_int8_quantize_rows.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp]
    L.iro_int8_quantize_rows.restype = None
    L.iro_int8_quantize_rows_residual.argtypes = [_vp, C.c_int, C.c_int] + [_vp] * 7
    L.iro_int8_quantize_rows_residual.restype = None
    L.iro_int8_linear_ex.argtypes = [_vp, _vp, _vp, C.POINTER(_IroInt8Weight), _vp, _vp,
                                     C.c_int, _vp, C.c_int]
    L.iro_int8_linear_ex.restype = None
    L.iro_int8_selfcheck.argtypes = []
    L.iro_int8_selfcheck.restype = C.c_int
    L.iro_silu_mul_inplace.argtypes = [_vp, _vp, C.c_size_t]
    L.iro_silu_mul_inplace.restype = None
    return L


def convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding=0):
    return lib().oracle_convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding)


def convtranspose1d_int8(inp, w: Weight, C_out, kernel, stride, padding, output_padding=0,
                         bias=None, residual=False):
    """inp: time-major [T_in, C_in]; w: [kernel*C_out, C_in].  Returns [T_out, C_out]."""
    inp = _c(inp, np.float32)
    T_in, Cin = inp.shape
    T_out = convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding)
    if T_out <= 0 or w.N != kernel * C_out or w.K != Cin:
        raise ValueError("bad transposed-convolution shape")
    out = np.empty((T_out, C_out), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    rc = lib().oracle_convtranspose1d_int8(_ptr(inp), T_in, Cin, C_out, _ptr(w.data),
                                           _ptr(w.scale), _ptr(w.colsum), kernel, stride,
                                           padding, output_padding, _ptr(b),
                                           int(bool(residual)), _ptr(out))
    if rc != T_out:
        raise RuntimeError("oracle transposed conv failed")
    return out


def codec_conv1(hidden, w: Weight, bias, skip, residual=False):
    """Residual unit's skip + 1x1 projection: skip + linear(quant(hidden))."""
    hidden = _c(hidden, np.float32)
    skip = _c(skip, np.float32)
    rows, Cc = hidden.shape
    if w.N != Cc or w.K != Cc or skip.shape != hidden.shape:
        raise ValueError("bad conv1 shape")
    out = np.empty_like(hidden)
    b = None if bias is None else _c(bias, np.float32)
    rc = lib().oracle_codec_conv1(_ptr(hidden), rows, Cc, _ptr(w.data), _ptr(w.scale),
                                  _ptr(w.colsum), _ptr(b), _ptr(skip), int(bool(residual)),
                                  _ptr(out))
    if rc != 0:
        raise RuntimeError("oracle conv1 failed")
    return out


def ref_lib(kind="ieee"):
    """kind: "ieee" (parity build), "codec", "dit", "vnni", "fast" (product flags,
    variant chosen for this host's ISA), "dit_fast" / "codec_fast" (the DiT /
    codec builds with the product flags, likewise) or "dit_vec" (the DiT build
    with IEEE semantics at -O3 for the build host, fixture recording only)."""
    if kind in ("fast", "dit_fast", "codec_fast"):
        kind = kind + "_" + _host_isa_variant()
    if kind not in _ref_libs:
        path = os.path.join(REF_DIR, f"libiro_ref_{kind}.so")
        if not os.path.exists(path):
            raise RuntimeError(f"reference build {path} is missing")
        L = C.CDLL(path) if kind == "vnni" else _bind_ops(C.CDLL(path))
        if kind.startswith("codec"):
            L.ref_conv1d_int8_forward.argtypes = [_vp, C.c_int, C.c_int, _vp, _vp, _vp, C.c_int,
                                                  C.c_int, C.c_int, C.c_int, C.c_int, _vp,
                                                  C.c_int, _vp]
            L.ref_conv1d_int8_forward.restype = C.c_int
            L.ref_conv1d_output_length.argtypes = [C.c_int] * 5
            L.ref_conv1d_output_length.restype = C.c_int
            L.ref_convtranspose1d_int8_forward.argtypes = [_vp, C.c_int, C.c_int, C.c_int, _vp,
                                                           _vp, _vp, C.c_int, C.c_int, C.c_int,
                                                           C.c_int, _vp, _vp]
            L.ref_convtranspose1d_int8_forward.restype = C.c_int
            L.ref_convtranspose1d_output_length.argtypes = [C.c_int] * 5
            L.ref_convtranspose1d_output_length.restype = C.c_int
            L.ref_codec_upsample_residual.argtypes = []
            L.ref_codec_upsample_residual.restype = C.c_int
        if kind.startswith("dit"):
            L.ref_dit_swiglu_int8.argtypes = [_vp, C.c_int] + [_vp] * 10
            L.ref_dit_swiglu_int8.restype = C.c_int
            L.ref_dit_block_int8.argtypes = [_vp] * 5 + [C.c_int] * 4 + [_vp] * 6
            L.ref_dit_block_int8.restype = C.c_int
            L.ref_dit_block_w.argtypes = [_vp] * 5 + [C.c_int] * 4 + [_vp] * 7
            L.ref_dit_block_w.restype = C.c_int
            L.ref_dit_block_dims.argtypes = [C.POINTER(C.c_int)] * 4
            L.ref_dit_block_dims.restype = C.c_int
            L.ref_dit_condition_w.argtypes = [_vp] * 4 + [C.c_int, _vp]
            L.ref_dit_condition_w.restype = C.c_int
            L.ref_dit_input_w.argtypes = [_vp] * 3 + [C.c_int, C.c_int, _vp]
            L.ref_dit_input_w.restype = C.c_int
            L.ref_dit_output_w.argtypes = [_vp] * 4 + [C.c_int, C.c_int, _vp]
            L.ref_dit_output_w.restype = C.c_int
            L.ref_dit_dims.argtypes = [C.POINTER(C.c_int), C.POINTER(C.c_int)]
            L.ref_dit_dims.restype = C.c_int
        _ref_libs[kind] = L
    return _ref_libs[kind]


def _host_isa_variant():
    flags = set()
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    flags = set(line.split(":", 1)[1].split())
                    break
    except OSError:
        pass
    if platform.machine() not in ("x86_64", "AMD64"):
        raise RuntimeError("reference fast builds are x86-64 only")
    v4 = {"avx512f", "avx512bw", "avx512cd", "avx512dq", "avx512vl", "avx512_vnni"}
    v3 = {"avx2", "fma", "bmi1", "bmi2", "movbe", "f16c"}
    if v4 <= flags and v3 <= flags:
        return "v4vnni"
    if v3 <= flags:
        return "v3"
    return "v2"


def ref_weight_quantize(w, kind="ieee"):
    L = ref_lib(kind)
    w = _c(w, np.float32)
    N, K = w.shape
    st = _IroInt8Weight()
    if L.iro_int8_weight_quantize(C.byref(st), _ptr(w), N, K) != 0:
        raise RuntimeError("reference weight quantize failed")
    d = np.ctypeslib.as_array(C.cast(st.data, C.POINTER(C.c_int8)), shape=(N * K,)).copy()
    s = np.ctypeslib.as_array(C.cast(st.scale, C.POINTER(C.c_float)), shape=(N,)).copy()
    c = np.ctypeslib.as_array(C.cast(st.colsum, C.POINTER(C.c_int32)), shape=(N,)).copy()
    L.iro_int8_weight_free(C.byref(st))
    return Weight(d.reshape(N, K), s, c)


def ref_weight_quantize_transposed(w_kn, kind="ieee"):
    L = ref_lib(kind)
    w_kn = _c(w_kn, np.float32)
    K, N = w_kn.shape
    st = _IroInt8Weight()
    if L.iro_int8_weight_quantize_transposed(C.byref(st), _ptr(w_kn), N, K) != 0:
        raise RuntimeError("reference weight quantize failed")
    d = np.ctypeslib.as_array(C.cast(st.data, C.POINTER(C.c_int8)), shape=(N * K,)).copy()
    s = np.ctypeslib.as_array(C.cast(st.scale, C.POINTER(C.c_float)), shape=(N,)).copy()
    c = np.ctypeslib.as_array(C.cast(st.colsum, C.POINTER(C.c_int32)), shape=(N,)).copy()
    L.iro_int8_weight_free(C.byref(st))
    return Weight(d.reshape(N, K), s, c)


def _ref_struct(w: Weight):
    return _IroInt8Weight(_ptr(w.data).value, _ptr(w.scale).value, _ptr(w.colsum).value,
                          w.N, w.K)


def ref_quantize_rows(x, kind="ieee"):
    x = _c(x, np.float32)
    M, K = x.shape
    q = np.empty((M, K), np.uint8); s = np.empty(M, np.float32); z = np.empty(M, np.int32)
    ref_lib(kind).iro_int8_quantize_rows(_ptr(x), M, K, _ptr(q), _ptr(s), _ptr(z))
    return q, s, z


def ref_quantize_rows_residual(x, kind="ieee"):
    x = _c(x, np.float32)
    M, K = x.shape
    q1 = np.empty((M, K), np.uint8); s1 = np.empty(M, np.float32); z1 = np.empty(M, np.int32)
    r = np.empty((M, K), np.float32)
    q2 = np.empty((M, K), np.uint8); s2 = np.empty(M, np.float32); z2 = np.empty(M, np.int32)
    ref_lib(kind).iro_int8_quantize_rows_residual(_ptr(x), M, K, _ptr(q1), _ptr(s1), _ptr(z1),
                                                  _ptr(r), _ptr(q2), _ptr(s2), _ptr(z2))
    return (q1, s1, z1), r, (q2, s2, z2)


def ref_linear_ex(q, scale, zero, w: Weight, bias=None, y=None, accumulate=False,
                  kind="ieee"):
    q = _c(q, np.uint8); scale = _c(scale, np.float32); zero = _c(zero, np.int32)
    M = q.shape[0]
    y = np.zeros((M, w.N), np.float32) if y is None else _c(y, np.float32).copy()
    work = np.empty((M, w.N), np.int32)
    b = None if bias is None else _c(bias, np.float32)
    st = _ref_struct(w)
    ref_lib(kind).iro_int8_linear_ex(_ptr(q), _ptr(scale), _ptr(zero), C.byref(st), _ptr(b),
                                     _ptr(y), M, _ptr(work), int(bool(accumulate)))
    return y, work


def ref_silu_mul(x, gate, kind="ieee"):
    x = _c(x, np.float32).copy(); gate = _c(gate, np.float32)
    ref_lib(kind).iro_silu_mul_inplace(_ptr(x), _ptr(gate), x.size)
    return x


def ref_selfcheck(kind="ieee"):
    return ref_lib(kind).iro_int8_selfcheck()


def ref_conv1d_int8(inp, w: Weight, kernel, stride=1, dilation=1, padding=0, bias=None,
                    residual=False, kind="codec"):
    L = ref_lib(kind)
    inp = _c(inp, np.float32)
    T_in, Cin = inp.shape
    T_out = L.ref_conv1d_output_length(T_in, kernel, stride, dilation, padding)
    out = np.empty((T_out, w.N), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    rc = L.ref_conv1d_int8_forward(_ptr(inp), T_in, Cin, _ptr(w.data), _ptr(w.scale),
                                   _ptr(w.colsum), w.N, kernel, stride, dilation, padding,
                                   _ptr(b), int(bool(residual)), _ptr(out))
    if rc != 0:
        raise RuntimeError("reference conv failed")
    return out


def ref_convtranspose1d_int8(inp, w: Weight, C_out, kernel, stride, padding, output_padding=0,
                             bias=None):
    """The reference's own transposed conv (dacvae.c:696-790).  Whether it adds
    the second term is the reference's process-wide policy: see
    ref_codec_upsample_residual()."""
    L = ref_lib("codec")
    inp = _c(inp, np.float32)
    T_in, Cin = inp.shape
    T_out = L.ref_convtranspose1d_output_length(T_in, kernel, stride, padding, output_padding)
    out = np.empty((T_out, C_out), np.float32)
    b = None if bias is None else _c(bias, np.float32)
    rc = L.ref_convtranspose1d_int8_forward(_ptr(inp), T_in, Cin, C_out, _ptr(w.data),
                                            _ptr(w.scale), _ptr(w.colsum), kernel, stride,
                                            padding, output_padding, _ptr(b), _ptr(out))
    if rc != 0:
        raise RuntimeError("reference transposed conv failed")
    return out


def ref_codec_upsample_residual():
    return bool(ref_lib("codec").ref_codec_upsample_residual())


def ref_dit_block(x, cond, ctx_k, ctx_v, mask, context_batch, B, S, C_ctx, adaln, q_norm,
                  k_norm, weights, kind="dit", fp32_weights=None):
    """The reference's dit_block (dit.c:983-1051) at layer 0 with int8
    projections.  weights: Weight objects wq, wk, wv, gate, wo, w1, w3, w2.
    fp32_weights: the fp32 projections in the same order, which the
    reference's diagnostic switches IRO_INT8_MASK / IRO_INT8_EMULATE read
    (dit.c:273-335; the reference takes both from this process's
    environment, once).  Returns the updated x [B*S, D]."""
    L = ref_lib(kind)
    x = _c(x, np.float32).copy()
    keep = [_c(a, np.float32) for a in adaln]
    ada = (_vp * 18)(*[a.ctypes.data for a in keep])
    wd = (_vp * 8)(*[w.data.ctypes.data for w in weights])
    wsc = (_vp * 8)(*[w.scale.ctypes.data for w in weights])
    wcs = (_vp * 8)(*[w.colsum.ctypes.data for w in weights])
    f32 = [_c(w, np.float32) for w in fp32_weights] if fp32_weights is not None else None
    wf = (_vp * 8)(*[w.ctypes.data for w in f32]) if f32 is not None else None
    cond = _c(cond, np.float32); ctx_k = _c(ctx_k, np.float32); ctx_v = _c(ctx_v, np.float32)
    mask = _c(mask, np.uint8); q_norm = _c(q_norm, np.float32); k_norm = _c(k_norm, np.float32)
    rc = L.ref_dit_block_w(_ptr(x), _ptr(cond), _ptr(ctx_k), _ptr(ctx_v), _ptr(mask),
                           context_batch, B, S, C_ctx, ada, _ptr(q_norm), _ptr(k_norm),
                           wd, wsc, wcs, wf)
    if rc != 0:
        raise RuntimeError("reference dit_block failed")
    return x


def ref_dit_condition(w0, w1, w2, t, kind="dit"):
    """dit.c:502-530 for timesteps t [B] -> cond [B, 3*1280]."""
    t = _c(np.atleast_1d(t), np.float32)
    out = np.empty((t.size, w2.shape[0]), np.float32)
    ws = [_c(w, np.float32) for w in (w0, w1, w2)]
    if ref_lib(kind).ref_dit_condition_w(*[_ptr(w) for w in ws], _ptr(t), t.size, _ptr(out)):
        raise RuntimeError("reference conditioner failed")
    return out


def ref_dit_input(in_w, in_b, x, B, S, kind="dit"):
    """dit.c:532-541: x [B*S, 32] -> [B*S, 1280]."""
    x = _c(x, np.float32)
    out = np.empty((B * S, in_w.shape[0]), np.float32)
    if ref_lib(kind).ref_dit_input_w(_ptr(_c(in_w, np.float32)), _ptr(_c(in_b, np.float32)),
                                      _ptr(x), B, S, _ptr(out)):
        raise RuntimeError("reference input projection failed")
    return out


def ref_dit_output(out_norm, out_w, out_b, x, B, S, kind="dit"):
    """dit.c:1070-1090: RMSNorm + linear -> velocity [B*S, 32]."""
    x = _c(x, np.float32)
    out = np.empty((B * S, out_w.shape[0]), np.float32)
    if ref_lib(kind).ref_dit_output_w(_ptr(_c(out_norm, np.float32)), _ptr(_c(out_w, np.float32)),
                                       _ptr(_c(out_b, np.float32)), _ptr(x), B, S, _ptr(out)):
        raise RuntimeError("reference output head failed")
    return out


def ref_dit_euler_step(state, ctx_k, ctx_v, mask, blocks, head, R, cfg, S, C, t, t_next,
                       scales):
    """One Euler step of R independent requests composed from the
    reference's own pieces, per request as sampler.c:241-297 runs it:
    conditioner once (B=1) broadcast to the cfg rows, input projection
    broadcast likewise, each layer's block with the request's shared context
    (context_batch 1), the output head, then guided = v0 + sum_i s_i (v0 -
    v_i) in row order and state += guided * dt in float32.

    blocks: per layer (adaln, q_norm, k_norm, [8 Weight]).  Returns the new
    state [R, S, 32]."""
    D = head["in_w"].shape[0]
    out = np.array(state, np.float32, copy=True)
    for r in range(R):
        cond = ref_dit_condition(head["cond_w0"], head["cond_w1"], head["cond_w2"],
                                 np.float32(t))
        proj = ref_dit_input(head["in_w"], head["in_b"], out[r], 1, S)
        x = np.tile(proj, (cfg, 1))
        cond_b = np.tile(cond, (cfg, 1))
        m = mask[r * cfg:(r + 1) * cfg]
        for l, (adaln, qn, kn, W) in enumerate(blocks):
            x = ref_dit_block(x, cond_b, ctx_k[l][r:r + 1], ctx_v[l][r:r + 1], m, 1, cfg, S, C,
                              adaln, qn, kn, W)
        v = ref_dit_output(head["out_norm"], head["out_w"], head["out_b"], x, cfg, S)
        v = v.reshape(cfg, S, -1)
        g = v[0].copy()
        for i in range(1, cfg):
            g = g + np.float32(scales[i - 1]) * (v[0] - v[i])
        dt = np.float32(np.float32(t_next) - np.float32(t))
        out[r] = out[r] + g * dt
    del D
    return out


def ref_dit_sample_euler(state, ctx_k, ctx_v, mask, blocks, head, R, cfg, S, C, steps,
                         init_scale, cfg_min_t, cfg_max_t, scales):
    """sampler.c:241-297's loop: the timestep schedule in float32 and the
    conditional row alone outside [cfg_min_t, cfg_max_t]."""
    f = np.float32
    cond_rows = mask.reshape(R, cfg, C)[:, 0]
    for step in range(steps):
        u, un = f(step) / f(steps), f(step + 1) / f(steps)
        t, tn = (f(1) - u) * f(init_scale), (f(1) - un) * f(init_scale)
        use = cfg > 1 and f(cfg_min_t) <= t <= f(cfg_max_t)
        state = ref_dit_euler_step(state, ctx_k, ctx_v, mask if use else cond_rows, blocks, head,
                                   R, cfg if use else 1, S, C, t, tn, scales)
    return state


def ref_dit_branch_velocity(state_r, ctx_k_r, ctx_v_r, mask_row, blocks, head, S, C, t,
                            kind="dit"):
    """The velocity of ONE CFG branch of one request at timestep t: the
    conditioner (B=1), the input projection of the request's state
    [S, 32], every layer's dit_block with batch 1 over that branch's
    context mask row [C] (ctx_k_r / ctx_v_r: per layer [1, C, D]), then
    the output head.  dit_block mixes rows only inside one batch row
    (attention, dit.c:809-868) and applies its AdaLN per batch row, so a
    batch of cfg branches equals cfg batch-1 calls
    (tests/test_oracle.py checks this bit for bit).  Returns [S, 32]."""
    cond = ref_dit_condition(head["cond_w0"], head["cond_w1"], head["cond_w2"], np.float32(t),
                             kind=kind)
    x = ref_dit_input(head["in_w"], head["in_b"], state_r, 1, S, kind=kind)
    m = np.ascontiguousarray(mask_row, np.uint8).reshape(1, C)
    for l, (adaln, qn, kn, W) in enumerate(blocks):
        x = ref_dit_block(x, cond, ctx_k_r[l], ctx_v_r[l], m, 1, 1, S, C, adaln, qn, kn, W,
                          kind=kind)
    return ref_dit_output(head["out_norm"], head["out_w"], head["out_b"], x, 1, S, kind=kind)


def ref_cfg_guided(v, scales):
    """sampler.c:283-297: guided = v0, then += s_i * (v0 - v_i) for the
    uncond rows in order, all in float32.  v: [cfg, S, 32]."""
    g = v[0].copy()
    for i in range(1, v.shape[0]):
        g = g + np.float32(scales[i - 1]) * (v[0] - v[i])
    return g


def ref_dit_sample_request(state_r, ctx_k_r, ctx_v_r, mask_r, blocks, head, cfg, S, C, steps,
                           init_scale, cfg_min_t, cfg_max_t, scales, kind="dit", pool=None):
    """sampler.c:241-297 for one request, its CFG branches evaluated as
    independent batch-1 forwards (in `pool`, a thread pool, when given: the
    reference calls release the GIL).  Returns (final state [S, 32],
    guided velocity per step [steps, S, 32], CFG rows used per step)."""
    f = np.float32
    state = np.array(state_r, np.float32, copy=True)
    vels, rows = [], []
    for step in range(steps):
        u, un = f(step) / f(steps), f(step + 1) / f(steps)
        t, tn = (f(1) - u) * f(init_scale), (f(1) - un) * f(init_scale)
        use = cfg > 1 and f(cfg_min_t) <= t <= f(cfg_max_t)
        nb = cfg if use else 1
        run = lambda b, st=state, tt=t: ref_dit_branch_velocity(  # noqa: E731
            st, ctx_k_r, ctx_v_r, mask_r[b], blocks, head, S, C, tt, kind=kind)
        v = list(pool.map(run, range(nb))) if pool is not None else [run(b) for b in range(nb)]
        g = ref_cfg_guided(np.stack(v), scales)
        dt = f(tn - t)
        state = state + g * dt
        vels.append(g)
        rows.append(nb)
    return state, np.stack(vels), rows


def ref_dit_block_dims():
    L = ref_lib("dit")
    v = [C.c_int() for _ in range(4)]
    L.ref_dit_block_dims(*[C.byref(i) for i in v])
    return tuple(i.value for i in v)


def ref_dit_dims():
    L = ref_lib("dit")
    d = C.c_int(); h = C.c_int()
    L.ref_dit_dims(C.byref(d), C.byref(h))
    return d.value, h.value


def ref_dit_swiglu(x, w1: Weight, w3: Weight, w2: Weight):
    """The reference's dit_swiglu (IRO_INT8_RESIDUAL of this process applies)."""
    L = ref_lib("dit")
    x = _c(x, np.float32)
    M = x.shape[0]
    out = np.empty((M, w2.N), np.float32)
    rc = L.ref_dit_swiglu_int8(_ptr(x), M, _ptr(w1.data), _ptr(w1.scale), _ptr(w1.colsum),
                               _ptr(w3.data), _ptr(w3.scale), _ptr(w3.colsum),
                               _ptr(w2.data), _ptr(w2.scale), _ptr(w2.colsum), _ptr(out))
    if rc != 0:
        raise RuntimeError("reference dit_swiglu failed")
    return out


# ---------------------------------------------------------------------------
# The reference test's deterministic generator (tests/test_int8_ops.c:12-16).


class XorShift:
    """xorshift64 seeded 0x9E3779B97F4A7C15; rnd() in [-0.5, 0.5) as float32."""

    def __init__(self, seed=0x9E3779B97F4A7C15):
        self.s = seed & 0xFFFFFFFFFFFFFFFF

    def rnd(self, n):
        out = np.empty(n, np.float32)
        s = self.s
        M = 0xFFFFFFFFFFFFFFFF
        for i in range(n):
            s ^= (s << 13) & M
            s ^= s >> 7
            s ^= (s << 17) & M
            out[i] = np.float32((s >> 40) & 0xFFFFFF) / np.float32(16777216.0) - np.float32(0.5)
        self.s = s
        return out
