"""Python ctypes binding of libirodori_b200.so (the C ABI in
include/irodori_b200.h).

The library is the product; this module only marshals numpy arrays and
device buffers into its C entry points for tests, the smoke check and the
benchmark.  Importing it loads the in-tree shared library and fails loudly
when it is missing: there is no Python or CPU implementation behind it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libirodori_b200.so")
HEADER_PATH = os.path.join(os.path.dirname(HERE), "include", "irodori_b200.h")

IRO_OK = 0
IRO_ERR_INVALID = -1
IRO_ERR_NO_DEVICE = -2
IRO_ERR_CUDA = -3
IRO_ERR_OOM = -4
IRO_ERR_DEVICE_TIMEOUT = -5
IRO_ERR_UNSUPPORTED = -6
IRO_ERR_SELFCHECK = -7
IRO_ERR_RANGE = -8
LAYOUT_PLAIN = 0
LAYOUT_GATED_PAIR = 1


class IroError(RuntimeError):
    def __init__(self, code, what=""):
        self.code = code
        msg = lib().iro_cuda_error_string(code).decode() if _lib else str(code)
        super().__init__(f"{what}: {msg} ({code})")


class IroInt8Weight(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scale", C.c_void_p), ("colsum", C.c_void_p),
                ("N", C.c_int), ("K", C.c_int)]


class IroInt8DevWeight(C.Structure):
    _fields_ = [("data", C.c_void_p), ("scale", C.c_void_p), ("colsum", C.c_void_p),
                ("bias", C.c_void_p), ("N", C.c_int), ("K", C.c_int), ("ld", C.c_int),
                ("layout", C.c_int), ("pair", C.c_int), ("hidden", C.c_int),
                ("device", C.c_int), ("priv", C.c_void_p)]


class IroDiTBlockDev(C.Structure):
    _fields_ = [("adaln", (C.c_void_p * 9) * 2), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("qkvg", IroInt8DevWeight), ("wo", IroInt8DevWeight), ("w13", IroInt8DevWeight),
                ("w2", IroInt8DevWeight), ("model_dim", C.c_int), ("heads", C.c_int),
                ("head_dim", C.c_int), ("adaln_rank", C.c_int), ("mlp_dim", C.c_int),
                ("norm_eps", C.c_float), ("residual_mask", C.c_int),
                ("fp32_groups", C.c_int), ("emulate", C.c_int), ("w_fp32", C.c_void_p * 8)]


class IroDiTInt8HostLayer(C.Structure):
    _fields_ = [(n, IroInt8Weight) for n in ("wq", "wk", "wv", "gate", "wo", "w1", "w2", "w3")]


class IroDiTInt8DevLayer(C.Structure):
    _fields_ = [(n, IroInt8DevWeight) for n in ("qkvg", "wo", "w13", "w2")]


class IroDiTInt8Dev(C.Structure):
    _fields_ = [("layer", IroDiTInt8DevLayer * 16), ("layers", C.c_int), ("bytes", C.c_size_t)]


class IroDACVAEInt8HostResidual(C.Structure):
    _fields_ = [("conv0", IroInt8Weight), ("conv1", IroInt8Weight)]


class IroDACVAEInt8HostStage(C.Structure):
    _fields_ = [("upsample", IroInt8Weight), ("residual", IroDACVAEInt8HostResidual * 3)]


class IroDACVAEInt8Host(C.Structure):
    _fields_ = [("initial", IroInt8Weight), ("stage", IroDACVAEInt8HostStage * 4),
                ("bytes", C.c_size_t)]


class IroDACVAEInt8DevResidual(C.Structure):
    _fields_ = [("conv0", IroInt8DevWeight), ("conv1", IroInt8DevWeight)]


class IroDACVAEInt8DevStage(C.Structure):
    _fields_ = [("upsample", IroInt8DevWeight), ("residual", IroDACVAEInt8DevResidual * 3)]


class IroDACVAEInt8Dev(C.Structure):
    _fields_ = [("initial", IroInt8DevWeight), ("stage", IroDACVAEInt8DevStage * 4),
                ("bytes", C.c_size_t)]


_vp, _i, _sz, _u64 = C.c_void_p, C.c_int, C.c_size_t, C.c_uint64
_W = C.POINTER(IroInt8Weight)
_DW = C.POINTER(IroInt8DevWeight)
_DB = C.POINTER(IroDiTBlockDev)

# name -> (restype, argtypes); every symbol declared in the public header.
SIGNATURES = {
    "iro_int8_weight_quantize": (_i, [_W, _vp, _i, _i]),
    "iro_int8_weight_quantize_transposed": (_i, [_W, _vp, _i, _i]),
    "iro_int8_weight_free": (None, [_W]),
    "iro_int8_weight_bytes": (_sz, [_W]),
    "iro_int8_quantize_rows": (None, [_vp, _i, _i, _vp, _vp, _vp]),
    "iro_int8_linear": (None, [_vp, _vp, _vp, _W, _vp, _vp, _i, _vp]),
    "iro_int8_linear_ex": (None, [_vp, _vp, _vp, _W, _vp, _vp, _i, _vp, _i]),
    "iro_int8_quantize_rows_residual": (None, [_vp, _i, _i] + [_vp] * 7),
    "iro_int8_fast_available": (_i, []),
    "iro_int8_prepare_backend": (C.c_char_p, []),
    "iro_int8_selfcheck": (_i, []),
    "iro_ops_backend_name": (C.c_char_p, []),
    "iro_cuda_init": (_i, [_i]),
    "iro_cuda_last_error": (_i, []),
    "iro_cuda_error_string": (C.c_char_p, [_i]),
    "iro_cuda_device_count": (_i, []),
    "iro_cuda_stream": (_vp, []),
    "iro_cuda_synchronize": (_i, [_vp]),
    "iro_int8_dev_weight_bytes": (_sz, [_DW]),
    "iro_dit_int8_dev_upload": (_i, [C.POINTER(IroDiTInt8Dev), C.POINTER(IroDiTInt8HostLayer),
                                     _i]),
    "iro_dit_int8_dev_free": (None, [C.POINTER(IroDiTInt8Dev)]),
    "iro_dacvae_int8_dev_upload": (_i, [C.POINTER(IroDACVAEInt8Dev),
                                        C.POINTER(IroDACVAEInt8Host)]),
    "iro_dacvae_int8_dev_free": (None, [C.POINTER(IroDACVAEInt8Dev)]),
    "iro_dit_velocity_dev": (_i, [C.c_void_p, _vp, _i, _i, _i, C.c_float, _vp, _vp, _vp, _i,
                                  _vp, _vp, _vp]),
    "iro_dit_cfg_update_dev": (_i, [C.c_void_p, _vp, _vp, _i, _i, _i, C.c_float, C.c_float,
                                    _vp, _vp]),
    "iro_cuda_gemm_profile_enabled": (_i, []),
    "iro_cuda_gemm_profile_reset": (None, []),
    "iro_cuda_gemm_profile_emit_json": (None, [C.c_char_p, _i, _i, _i]),
    "iro_dev_malloc": (_vp, [_sz]),
    "iro_dev_free": (None, [_vp]),
    "iro_memcpy_htod": (_i, [_vp, _vp, _sz, _vp]),
    "iro_memcpy_dtoh": (_i, [_vp, _vp, _sz, _vp]),
    "iro_memcpy_dtod": (_i, [_vp, _vp, _sz, _vp]),
    "iro_memset_dev": (_i, [_vp, _i, _sz, _vp]),
    "iro_host_alloc_pinned": (_vp, [_sz]),
    "iro_host_free_pinned": (None, [_vp]),
    "iro_int8_dev_weight_upload": (_i, [_DW, _W, _vp]),
    "iro_int8_dev_weight_quantize": (_i, [_DW, _vp, _i, _i, _vp, _vp]),
    "iro_int8_dev_weight_concat": (_i, [_DW, C.POINTER(_W), C.POINTER(_vp), _i]),
    "iro_int8_dev_weight_gated_pair": (_i, [_DW, _W, _W, _vp, _vp]),
    "iro_int8_dev_weight_free": (None, [_DW]),
    "iro_int8_quantize_rows_dev": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "iro_int8_quantize_rows_sym_dev": (_i, [_vp, _i, _i, _vp, _vp, _vp, _vp]),
    "iro_int8_quantize_rows_residual_dev": (_i, [_vp, _i, _i] + [_vp] * 7 + [_vp]),
    "iro_int8_linear_dev": (_i, [_vp, _vp, _vp, _DW, _vp, _vp, _i, _vp, _i, _vp]),
    "iro_int8_linear2_dev": (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _DW, _vp, _vp, _i, _vp]),
    "iro_int8_linear_split_dev": (_i, [_vp, _vp, _vp, _DW, C.POINTER(_vp), _i, _i, _i, _vp]),
    "iro_int8_gated_dev": (_i, [_vp, _vp, _vp, _DW, _vp, _i, _vp]),
    "iro_int8_swiglu_workspace_bytes": (_sz, [_i, _i, _i, _i]),
    "iro_int8_swiglu_dev": (_i, [_vp, _i, _DW, _DW, _vp, _vp, _i, _vp, _vp]),
    "iro_int8_swiglu": (_i, [_vp, _i, _DW, _DW, _vp, _vp, _i]),
    "iro_int8_swiglu_noalloc_dev": (_i, [_vp, _i, _DW, _DW, _vp, _vp, _i, _vp]),
    "iro_int8_swiglu_plan": (_i, [C.POINTER(_vp), _vp, _i, _DW, _DW, _vp, _vp, _i]),
    "iro_plan_launch": (_i, [_vp, _vp]),
    "iro_plan_free": (None, [_vp]),
    "iro_int8_swiglu_pipe_create": (_i, [C.POINTER(_vp), _i, _DW, _DW, _vp, _i, _i]),
    "iro_int8_swiglu_pipe_submit": (_i, [_vp, _vp, _vp]),
    "iro_int8_swiglu_pipe_wait": (_i, [_vp]),
    "iro_int8_swiglu_pipe_free": (None, [_vp]),
    "iro_conv1d_out_len": (_i, [_i, _i, _i, _i, _i]),
    "iro_int8_conv1d_dev": (_i, [_vp, _i, _i, _i, _DW, _i, _i, _i, _i, _vp, _i, _vp, _vp]),
    "iro_convtranspose1d_out_len": (_i, [_i, _i, _i, _i, _i]),
    "iro_int8_convtranspose1d_dev": (_i, [_vp, _i, _i, _i, _DW, _i, _i, _i, _i, _i, _vp, _i,
                                          _vp, _vp]),
    "iro_int8_codec_conv1_dev": (_i, [_vp, _i, _DW, _vp, _vp, _i, _vp, _vp]),
    "iro_st_file_open": (_i, [_vp, C.c_char_p]),
    "iro_st_file_close": (None, [_vp]),
    "iro_st_file_count": (_i, [_vp]),
    "iro_st_file_name": (C.c_char_p, [_vp, _i]),
    "iro_st_file_tensor": (_i, [_vp, C.c_char_p, _vp, _vp, _vp, _vp]),
    "iro_st_file_data": (_vp, [_vp, C.c_char_p]),
    "iro_st_file_drop_prefix": (_u64, [_vp, C.c_char_p]),
    "iro_int8_dev_weight_from_st": (_i, [_DW, _vp, C.c_char_p, _i, C.c_char_p]),
    "iro_dit_rope_table": (_i, [_vp, _vp, _i, _i]),
    "iro_dit_block_workspace_bytes": (_sz, [_DB, _i, _i, _i, _i]),
    "iro_dit_block_dev": (_i, [_DB, _vp, _vp, _i, _vp, _vp, _vp, _i, _i, _i, _i, _vp, _vp, _vp,
                               _vp]),
    "iro_dit_step_workspace_bytes": (_sz, [_vp, _i, _i, _i, _i]),
    "iro_dit_euler_step_dev": (_i, [_vp, _vp, _i, _i, _i, C.c_float, C.c_float, _vp, _vp, _vp,
                                    _vp, _i, _vp, _vp]),
    "iro_dit_stage_workspace_bytes": (_sz, [_vp, _i]),
    "iro_policy_dit_residual_mask": (_i, []),
    "iro_policy_dit_fp32_groups": (_i, []),
    "iro_policy_dit_emulate": (_i, []),
    "iro_dit_stats_read": (_i, [_i, _i, C.POINTER(C.c_double), C.POINTER(C.c_double), _vp, _i]),
    "iro_dit_stats_reset": (None, []),
    "iro_dit_stats_report": (None, []),
    "iro_policy_codec_int8_mask": (_i, []),
    "iro_policy_codec_residual_mask": (_i, []),
    "iro_policy_codec_residual_stages": (_i, []),
    "iro_policy_codec_residual": (_i, [_i, _i]),
    "iro_dit_sample_workspace_bytes": (_sz, [_vp, _i, _i, _i, _i, _i]),
    "iro_dit_condition_dev": (_i, [_vp, _vp, _i, _vp, _vp, _vp]),
    "iro_dit_input_dev": (_i, [_vp, _vp, _i, _i, _vp, _vp]),
    "iro_dit_output_dev": (_i, [_vp, _vp, _i, _i, _vp, _vp, _vp]),
    "iro_dit_sample_euler_dev": (_i, [_vp, _vp, _i, _i, _i, _i, C.c_float, C.c_float, C.c_float,
                                      _vp, _vp, _vp, _vp, _i, _vp, _vp]),
    "iro_debug_bounded_wait_probe": (_i, [_u64]),
}

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is not built: run `make -C irodori-c_b200` (or "
                "__graft_entry__.build()); there is no fallback implementation")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(code, what="irodori_b200"):
    if code != IRO_OK:
        raise IroError(code, what)


def check_last(what):
    code = lib().iro_cuda_last_error()
    if code != IRO_OK:
        raise IroError(code, what)


def init(device=0):
    check(lib().iro_cuda_init(device), f"iro_cuda_init({device})")


def device_count():
    return lib().iro_cuda_device_count()


def _p(a):
    if a is None:
        return None
    if isinstance(a, DevBuf):
        return C.c_void_p(a.ptr)
    if isinstance(a, int):
        return C.c_void_p(a)
    if hasattr(a, "data_ptr"):
        return C.c_void_p(a.data_ptr())
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dt):
    return np.ascontiguousarray(a, dtype=dt)


# ----------------------------------------------------------------------------
# Device buffers owned through the library's own allocator.


class DevBuf:
    """A device allocation of `shape` x `dtype` (iro_dev_malloc)."""

    def __init__(self, shape, dtype):
        self.shape = tuple(int(s) for s in (shape if isinstance(shape, (tuple, list)) else (shape,)))
        self.dtype = np.dtype(dtype)
        self.nbytes = int(np.prod(self.shape, dtype=np.int64)) * self.dtype.itemsize
        self.ptr = lib().iro_dev_malloc(max(self.nbytes, 1))
        if not self.ptr:
            raise IroError(IRO_ERR_OOM, "iro_dev_malloc")

    @classmethod
    def from_host(cls, a, dtype=None):
        a = np.ascontiguousarray(a, dtype=dtype or a.dtype)
        b = cls(a.shape, a.dtype)
        b.upload(a)
        return b

    def upload(self, a, stream=None):
        a = np.ascontiguousarray(a, dtype=self.dtype)
        assert a.nbytes == self.nbytes
        check(lib().iro_memcpy_htod(C.c_void_p(self.ptr), _p(a), self.nbytes, stream), "htod")

    def zero(self):
        check(lib().iro_memset_dev(C.c_void_p(self.ptr), 0, self.nbytes, None), "memset")

    def fill_byte(self, v):
        check(lib().iro_memset_dev(C.c_void_p(self.ptr), int(v), self.nbytes, None), "memset")

    def get(self):
        out = np.empty(self.shape, self.dtype)
        check(lib().iro_memcpy_dtoh(_p(out), C.c_void_p(self.ptr), self.nbytes, None), "dtoh")
        return out

    def free(self):
        if self.ptr:
            lib().iro_dev_free(C.c_void_p(self.ptr))
            self.ptr = 0

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def synchronize(stream=None):
    check(lib().iro_cuda_synchronize(stream), "synchronize")


# ----------------------------------------------------------------------------
# Part 1: the ops.h-compatible host API.


class HostWeight:
    """An IroInt8Weight quantised by iro_int8_weight_quantize (GPU)."""

    def __init__(self, w=None, transposed=False, N=None, K=None):
        self.st = IroInt8Weight()
        if w is not None:
            w = _c(w, np.float32)
            if transposed:
                K_, N_ = w.shape
                rc = lib().iro_int8_weight_quantize_transposed(C.byref(self.st), _p(w), N_, K_)
            else:
                N_, K_ = w.shape
                rc = lib().iro_int8_weight_quantize(C.byref(self.st), _p(w), N_, K_)
            if rc != 0:
                raise IroError(lib().iro_cuda_last_error() or IRO_ERR_INVALID,
                               "iro_int8_weight_quantize")

    @classmethod
    def from_arrays(cls, data, scale, colsum):
        """Wrap caller-owned arrays (kept alive by this object)."""
        self = cls()
        self._keep = (_c(data, np.int8), _c(scale, np.float32), _c(colsum, np.int32))
        d, s, c = self._keep
        self.st = IroInt8Weight(_p(d).value, _p(s).value, _p(c).value, d.shape[0], d.shape[1])
        self._borrowed = True
        return self

    @property
    def N(self):
        return self.st.N

    @property
    def K(self):
        return self.st.K

    @property
    def data(self):
        return np.ctypeslib.as_array(C.cast(self.st.data, C.POINTER(C.c_int8)),
                                     shape=(self.N, self.K)).copy()

    @property
    def scale(self):
        return np.ctypeslib.as_array(C.cast(self.st.scale, C.POINTER(C.c_float)),
                                     shape=(self.N,)).copy()

    @property
    def colsum(self):
        return np.ctypeslib.as_array(C.cast(self.st.colsum, C.POINTER(C.c_int32)),
                                     shape=(self.N,)).copy()

    def nbytes(self):
        return lib().iro_int8_weight_bytes(C.byref(self.st))

    def free(self):
        if getattr(self, "_borrowed", False):
            self.st = IroInt8Weight()
            self._keep = None
            return
        lib().iro_int8_weight_free(C.byref(self.st))

    def __del__(self):
        try:
            if self.st.data:
                self.free()
        except Exception:
            pass


def quantize_rows(x):
    x = _c(x, np.float32)
    M, K = x.shape
    q = np.empty((M, K), np.uint8)
    s = np.empty(M, np.float32)
    z = np.empty(M, np.int32)
    lib().iro_int8_quantize_rows(_p(x), M, K, _p(q), _p(s), _p(z))
    check_last("iro_int8_quantize_rows")
    return q, s, z


def quantize_rows_residual(x):
    x = _c(x, np.float32)
    M, K = x.shape
    q1 = np.empty((M, K), np.uint8); s1 = np.empty(M, np.float32); z1 = np.empty(M, np.int32)
    r = np.empty((M, K), np.float32)
    q2 = np.empty((M, K), np.uint8); s2 = np.empty(M, np.float32); z2 = np.empty(M, np.int32)
    lib().iro_int8_quantize_rows_residual(_p(x), M, K, _p(q1), _p(s1), _p(z1), _p(r),
                                          _p(q2), _p(s2), _p(z2))
    check_last("iro_int8_quantize_rows_residual")
    return (q1, s1, z1), r, (q2, s2, z2)


def linear_ex(q, scale, zero, w: HostWeight, bias=None, y=None, accumulate=False):
    q = _c(q, np.uint8); scale = _c(scale, np.float32); zero = _c(zero, np.int32)
    M = q.shape[0]
    y = np.zeros((M, w.N), np.float32) if y is None else _c(y, np.float32).copy()
    work = np.empty((M, w.N), np.int32)
    b = None if bias is None else _c(bias, np.float32)
    lib().iro_int8_linear_ex(_p(q), _p(scale), _p(zero), C.byref(w.st), _p(b), _p(y), M,
                             _p(work), int(bool(accumulate)))
    check_last("iro_int8_linear_ex")
    return y, work


def selfcheck():
    return lib().iro_int8_selfcheck()


# ----------------------------------------------------------------------------
# Part 2: device weights and device-pointer operations.


class DevWeight:
    """An IroInt8DevWeight owned by the library."""

    def __init__(self):
        self.st = IroInt8DevWeight()

    @classmethod
    def upload(cls, w, bias=None):
        """w: HostWeight or an (data, scale, colsum) triple."""
        self = cls()
        hw = w if isinstance(w, HostWeight) else HostWeight.from_arrays(*w)
        b = None if bias is None else _c(bias, np.float32)
        check(lib().iro_int8_dev_weight_upload(C.byref(self.st), C.byref(hw.st), _p(b)),
              "dev_weight_upload")
        return self

    @classmethod
    def quantize(cls, w_dev, N, K, bias_dev=None):
        self = cls()
        check(lib().iro_int8_dev_weight_quantize(C.byref(self.st), _p(w_dev), N, K,
                                                 _p(bias_dev), None), "dev_weight_quantize")
        return self

    @classmethod
    def concat(cls, parts, biases=None):
        self = cls()
        hws = [p if isinstance(p, HostWeight) else HostWeight.from_arrays(*p) for p in parts]
        arr = (_W * len(hws))(*[C.pointer(h.st) for h in hws])
        bl = [None if (biases is None or b is None) else _c(b, np.float32) for b in
              (biases or [None] * len(hws))]
        barr = (_vp * len(hws))(*[(_p(b).value if b is not None else None) for b in bl])
        check(lib().iro_int8_dev_weight_concat(C.byref(self.st), arr, barr, len(hws)),
              "dev_weight_concat")
        self._keep = (hws, bl)
        return self

    @classmethod
    def gated_pair(cls, w1, w3, b1=None, b3=None):
        self = cls()
        h1 = w1 if isinstance(w1, HostWeight) else HostWeight.from_arrays(*w1)
        h3 = w3 if isinstance(w3, HostWeight) else HostWeight.from_arrays(*w3)
        b1 = None if b1 is None else _c(b1, np.float32)
        b3 = None if b3 is None else _c(b3, np.float32)
        check(lib().iro_int8_dev_weight_gated_pair(C.byref(self.st), C.byref(h1.st),
                                                   C.byref(h3.st), _p(b1), _p(b3)),
              "dev_weight_gated_pair")
        return self

    @property
    def N(self):
        return self.st.N

    @property
    def K(self):
        return self.st.K

    def free(self):
        lib().iro_int8_dev_weight_free(C.byref(self.st))

    def __del__(self):
        try:
            if self.st.data:
                self.free()
        except Exception:
            pass


def quantize_rows_dev(x, M, K, q, s, z, symmetric=False, stream=None):
    fn = lib().iro_int8_quantize_rows_sym_dev if symmetric else lib().iro_int8_quantize_rows_dev
    check(fn(_p(x), M, K, _p(q), _p(s), _p(z), stream), "quantize_rows_dev")


def quantize_rows_residual_dev(x, M, K, q1, s1, z1, r, q2, s2, z2, stream=None):
    check(lib().iro_int8_quantize_rows_residual_dev(_p(x), M, K, _p(q1), _p(s1), _p(z1), _p(r),
                                                    _p(q2), _p(s2), _p(z2), stream),
          "quantize_rows_residual_dev")


def linear_dev(q, s, z, w: DevWeight, bias, y, M, work=None, accumulate=False, stream=None):
    check(lib().iro_int8_linear_dev(_p(q), _p(s), _p(z), C.byref(w.st), _p(bias), _p(y), M,
                                    _p(work), int(bool(accumulate)), stream), "linear_dev")


def linear2_dev(q1, s1, z1, q2, s2, z2, w: DevWeight, bias, y, M, stream=None):
    check(lib().iro_int8_linear2_dev(_p(q1), _p(s1), _p(z1), _p(q2), _p(s2), _p(z2),
                                     C.byref(w.st), _p(bias), _p(y), M, stream), "linear2_dev")


def linear_split_dev(q, s, z, w: DevWeight, outs, seg, M, stream=None):
    arr = (_vp * len(outs))(*[_p(o).value for o in outs])
    check(lib().iro_int8_linear_split_dev(_p(q), _p(s), _p(z), C.byref(w.st), arr, len(outs),
                                          seg, M, stream), "linear_split_dev")


def gated_dev(q, s, z, w13: DevWeight, hidden, M, stream=None):
    check(lib().iro_int8_gated_dev(_p(q), _p(s), _p(z), C.byref(w13.st), _p(hidden), M, stream),
          "gated_dev")


def swiglu_workspace_bytes(M, D, H, residual_w2=False):
    return lib().iro_int8_swiglu_workspace_bytes(M, D, H, int(bool(residual_w2)))


def swiglu_dev(x, M, w13: DevWeight, w2: DevWeight, b2, out, residual_w2=False, workspace=None,
               stream=None):
    check(lib().iro_int8_swiglu_dev(_p(x), M, C.byref(w13.st), C.byref(w2.st), _p(b2), _p(out),
                                    int(bool(residual_w2)), _p(workspace), stream), "swiglu_dev")


def swiglu_host(x, w13: DevWeight, w2: DevWeight, out=None, residual_w2=False, b2_dev=None):
    x = _c(x, np.float32)
    M = x.shape[0]
    if out is None:
        out = np.empty((M, w2.N), np.float32)
    check(lib().iro_int8_swiglu(_p(x), M, C.byref(w13.st), C.byref(w2.st), _p(b2_dev), _p(out),
                                int(bool(residual_w2))), "iro_int8_swiglu")
    return out


def swiglu_noalloc_dev(x, M, w13: DevWeight, w2: DevWeight, b2, out, residual_w2=False,
                      stream=None):
    """The SwiGLU block on the library's built-in scratch (no allocation)."""
    return lib().iro_int8_swiglu_noalloc_dev(_p(x), M, C.byref(w13.st), C.byref(w2.st), _p(b2),
                                             _p(out), int(bool(residual_w2)), stream)


class Plan:
    """A recorded SwiGLU block (CUDA graph) with fixed device buffers."""

    def __init__(self, x, M, w13: DevWeight, w2: DevWeight, b2, out, residual_w2=False):
        self.h = C.c_void_p()
        check(lib().iro_int8_swiglu_plan(C.byref(self.h), _p(x), M, C.byref(w13.st),
                                         C.byref(w2.st), _p(b2), _p(out),
                                         int(bool(residual_w2))), "iro_int8_swiglu_plan")
        self._keep = (x, w13, w2, b2, out)

    def launch(self, stream=None):
        check(lib().iro_plan_launch(self.h, stream), "iro_plan_launch")

    def free(self):
        if self.h:
            lib().iro_plan_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


class SwigluPipe:
    """Asynchronous host-buffer pipeline of the SwiGLU block."""

    def __init__(self, M, w13: DevWeight, w2: DevWeight, b2=None, residual_w2=False, depth=3):
        self.h = C.c_void_p()
        check(lib().iro_int8_swiglu_pipe_create(C.byref(self.h), M, C.byref(w13.st),
                                                C.byref(w2.st), _p(b2), int(bool(residual_w2)),
                                                depth), "iro_int8_swiglu_pipe_create")
        self._keep = (w13, w2, b2)

    def submit(self, x_host, out_host):
        check(lib().iro_int8_swiglu_pipe_submit(self.h, _p(x_host), _p(out_host)),
              "iro_int8_swiglu_pipe_submit")

    def wait(self):
        check(lib().iro_int8_swiglu_pipe_wait(self.h), "iro_int8_swiglu_pipe_wait")

    def free(self):
        if self.h:
            lib().iro_int8_swiglu_pipe_free(self.h)
            self.h = C.c_void_p()

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def conv1d_out_len(T_in, kernel, stride=1, dilation=1, padding=0):
    return lib().iro_conv1d_out_len(T_in, kernel, stride, dilation, padding)


def conv1d_dev(inp, batch, T_in, Cin, w: DevWeight, kernel, stride, dilation, padding, bias,
               residual, out, stream=None):
    rc = lib().iro_int8_conv1d_dev(_p(inp), batch, T_in, Cin, C.byref(w.st), kernel, stride,
                                   dilation, padding, _p(bias), int(bool(residual)), _p(out), stream)
    if rc < 0:
        raise IroError(rc, "conv1d_dev")
    return rc


def convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding=0):
    return lib().iro_convtranspose1d_out_len(T_in, kernel, stride, padding, output_padding)


def convtranspose1d_dev(inp, batch, T_in, Cin, w: DevWeight, C_out, kernel, stride, padding,
                        output_padding, bias, residual, out, stream=None):
    rc = lib().iro_int8_convtranspose1d_dev(_p(inp), batch, T_in, Cin, C.byref(w.st), C_out,
                                            kernel, stride, padding, output_padding, _p(bias),
                                            int(bool(residual)), _p(out), stream)
    if rc < 0:
        raise IroError(rc, "convtranspose1d_dev")
    return rc


def codec_conv1_dev(hidden, rows, w: DevWeight, bias, skip, residual, out, stream=None):
    check(lib().iro_int8_codec_conv1_dev(_p(hidden), rows, C.byref(w.st), _p(bias), _p(skip),
                                          int(bool(residual)), _p(out), stream),
           "codec_conv1_dev")


def dit_rope_table(S, head_dim=64):
    """dit.c:644-705 RoPE tables as host arrays [S, head_dim/2]."""
    c = np.empty((S, head_dim // 2), np.float32)
    sn = np.empty((S, head_dim // 2), np.float32)
    check(lib().iro_dit_rope_table(_p(c), _p(sn), S, head_dim), "dit_rope_table")
    return c, sn


class DiTBlock:
    """One DiT block's device weights (IroDiTBlockDev), built from host fp32
    AdaLN/norm arrays and int8 weights (HostWeight or (data, scale, colsum))."""

    def __init__(self, adaln, q_norm, k_norm, wq, wk, wv, wg, wo, w1, w3, w2, model_dim=1280,
                 heads=20, rank=192, mlp_dim=3680, eps=1e-5, residual_mask=8, fp32_weights=None,
                 fp32_groups=0, emulate=0):
        """fp32_weights: host fp32 arrays (wq, wk, wv, gate, wo, w1, w3, w2), uploaded
        for the diagnostic modes fp32_groups / emulate (the reference's
        15 & ~IRO_INT8_MASK and IRO_INT8_EMULATE, dit.c:273-335)."""
        self.bufs = [DevBuf.from_host(np.ascontiguousarray(a, np.float32)) for a in adaln]
        self.qn = DevBuf.from_host(np.ascontiguousarray(q_norm, np.float32))
        self.kn = DevBuf.from_host(np.ascontiguousarray(k_norm, np.float32))
        self.qkvg = DevWeight.concat([wq, wk, wv, wg])
        self.wo = DevWeight.upload(wo)
        self.w13 = DevWeight.gated_pair(w1, w3)
        self.w2 = DevWeight.upload(w2)
        st = IroDiTBlockDev()
        for i in range(2):
            for j in range(9):
                st.adaln[i][j] = self.bufs[9 * i + j].ptr
        st.q_norm, st.k_norm = self.qn.ptr, self.kn.ptr
        st.qkvg, st.wo, st.w13, st.w2 = self.qkvg.st, self.wo.st, self.w13.st, self.w2.st
        st.model_dim, st.heads, st.head_dim, st.adaln_rank, st.mlp_dim = (model_dim, heads, 64,
                                                                          rank, mlp_dim)
        st.norm_eps, st.residual_mask = eps, residual_mask
        self.fp32 = [DevBuf.from_host(np.ascontiguousarray(a, np.float32))
                     for a in (fp32_weights or [])]
        for i, b in enumerate(self.fp32):
            st.w_fp32[i] = b.ptr
        st.fp32_groups, st.emulate = fp32_groups, emulate
        self.st = st

    def run(self, x, cond, ctx_k, ctx_v, mask, context_batch, B, S, n_ctx, rope_cos, rope_sin,
            cond_rows=None, workspace=None, stream=None):
        check(lib().iro_dit_block_dev(C.byref(self.st), _p(x), _p(cond),
                                      B if cond_rows is None else cond_rows, _p(ctx_k), _p(ctx_v),
                                      _p(mask), context_batch, B, S, n_ctx, _p(rope_cos),
                                      _p(rope_sin), _p(workspace), stream), "dit_block_dev")


class IroDiTModelDev(C.Structure):
    _fields_ = [("block", IroDiTBlockDev * 16), ("layers", C.c_int),
                ("cond_w0", C.c_void_p), ("cond_w1", C.c_void_p), ("cond_w2", C.c_void_p),
                ("in_w", C.c_void_p), ("in_b", C.c_void_p), ("out_norm", C.c_void_p),
                ("out_w", C.c_void_p), ("out_b", C.c_void_p), ("timestep_dim", C.c_int),
                ("latent_dim", C.c_int), ("norm_eps", C.c_float)]


class DiTModel:
    """The whole DiT on the device: blocks (DiTBlock) plus the conditioner,
    input and output fp32 layers (host arrays, uploaded)."""

    def __init__(self, blocks, cond_w0, cond_w1, cond_w2, in_w, in_b, out_norm, out_w, out_b,
                 eps=1e-5):
        self.blocks = list(blocks)
        self.bufs = [DevBuf.from_host(np.ascontiguousarray(a, np.float32))
                     for a in (cond_w0, cond_w1, cond_w2, in_w, in_b, out_norm, out_w, out_b)]
        st = IroDiTModelDev()
        for i, b in enumerate(self.blocks):
            st.block[i] = b.st
        st.layers = len(self.blocks)
        (st.cond_w0, st.cond_w1, st.cond_w2, st.in_w, st.in_b, st.out_norm, st.out_w,
         st.out_b) = [b.ptr for b in self.bufs]
        st.timestep_dim = cond_w0.shape[1]
        st.latent_dim = in_w.shape[1]
        st.norm_eps = eps
        self.st = st

    def euler_step(self, state, R, cfg, S, t, t_next, cfg_scales, ctx_k, ctx_v, mask, n_ctx,
                   workspace=None, stream=None):
        """ctx_k/ctx_v: per layer DevBuf [R, C, D]; mask DevBuf [R*cfg, C]."""
        ks = (_vp * len(ctx_k))(*[k.ptr for k in ctx_k])
        vs = (_vp * len(ctx_v))(*[v.ptr for v in ctx_v])
        sc = (C.c_float * 3)(*(list(cfg_scales) + [0.0] * (3 - len(cfg_scales))))
        check(lib().iro_dit_euler_step_dev(C.byref(self.st), _p(state), R, cfg, S, t, t_next, sc,
                                           ks, vs, _p(mask), n_ctx, _p(workspace), stream),
              "dit_euler_step_dev")

    def sample_euler(self, state, R, cfg, S, steps, init_scale, cfg_min_t, cfg_max_t,
                     cfg_scales, ctx_k, ctx_v, mask, n_ctx, workspace=None, stream=None):
        ks = (_vp * len(ctx_k))(*[k.ptr for k in ctx_k])
        vs = (_vp * len(ctx_v))(*[v.ptr for v in ctx_v])
        sc = (C.c_float * 3)(*(list(cfg_scales) + [0.0] * (3 - len(cfg_scales))))
        check(lib().iro_dit_sample_euler_dev(C.byref(self.st), _p(state), R, cfg, S, steps,
                                             init_scale, cfg_min_t, cfg_max_t, sc, ks, vs,
                                             _p(mask), n_ctx, _p(workspace), stream),
              "dit_sample_euler_dev")

    def velocity(self, state, R, cfg, S, t, ctx_k, ctx_v, mask, n_ctx, velocity, workspace=None,
                 stream=None):
        """Per-row velocities [R*cfg, S, 32] of one model forward (no update)."""
        ks = (_vp * len(ctx_k))(*[k.ptr for k in ctx_k])
        vs = (_vp * len(ctx_v))(*[v.ptr for v in ctx_v])
        check(lib().iro_dit_velocity_dev(C.byref(self.st), _p(state), R, cfg, S, t, ks, vs,
                                         _p(mask), n_ctx, _p(velocity), _p(workspace), stream),
              "dit_velocity_dev")

    def cfg_update(self, state, velocity, R, cfg, S, t, t_next, cfg_scales, stream=None):
        sc = (C.c_float * 3)(*(list(cfg_scales) + [0.0] * (3 - len(cfg_scales))))
        check(lib().iro_dit_cfg_update_dev(C.byref(self.st), _p(state), _p(velocity), R, cfg, S,
                                           t, t_next, sc, stream), "dit_cfg_update_dev")

    def condition(self, t, cond):
        t = np.ascontiguousarray(np.atleast_1d(t), np.float32)
        check(lib().iro_dit_condition_dev(C.byref(self.st), _p(t), t.size, _p(cond), None, None),
              "dit_condition_dev")

    def input(self, x, B, S, projected):
        check(lib().iro_dit_input_dev(C.byref(self.st), _p(x), B, S, _p(projected), None),
              "dit_input_dev")

    def output(self, x, B, S, velocity):
        check(lib().iro_dit_output_dev(C.byref(self.st), _p(x), B, S, _p(velocity), None, None),
              "dit_output_dev")

    def workspace_bytes(self, R, cfg, S, n_ctx, steps=None):
        """Workspace of one euler_step, or of sample_euler over `steps`."""
        if steps is None:
            return lib().iro_dit_step_workspace_bytes(C.byref(self.st), R, cfg, S, n_ctx)
        return lib().iro_dit_sample_workspace_bytes(C.byref(self.st), R, cfg, S, n_ctx, steps)


DIT_STAT_GROUPS = ("qkvg", "wo", "w13", "w2")


def dit_stats(layer, group, channels=8192):
    """IRO_INT8_STATS cell of (layer, group): rows, sum of max|x|/rms(x) over
    rows, and the histogram of each row's first max-|x| channel (dit.c:340-400)."""
    rows, ratio = C.c_double(), C.c_double()
    hist = np.zeros(channels, np.uint32)
    check(lib().iro_dit_stats_read(layer, group, C.byref(rows), C.byref(ratio), _p(hist),
                                   channels), "iro_dit_stats_read")
    return rows.value, ratio.value, hist


def dit_stats_reset():
    lib().iro_dit_stats_reset()


def dit_stats_report():
    """Print the reference's int8-stats summary lines to stderr."""
    lib().iro_dit_stats_report()


class StFile:
    """A .safetensors checkpoint mapped read-only (iro_st_file_*)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().iro_st_file_open(C.byref(h), os.fsencode(path)), "st_file_open")
        self.h = h

    def close(self):
        if self.h:
            lib().iro_st_file_close(self.h)
            self.h = None

    def names(self):
        return [lib().iro_st_file_name(self.h, i).decode() for i in range(lib().iro_st_file_count(self.h))]

    def tensor(self, name):
        dt, nd = C.c_int(), C.c_int()
        shape = (C.c_uint64 * 8)()
        nb = C.c_uint64()
        check(lib().iro_st_file_tensor(self.h, name.encode(), C.byref(dt), C.byref(nd), shape,
                                       C.byref(nb)), "st_file_tensor")
        return dt.value, tuple(shape[i] for i in range(nd.value)), nb.value

    def drop_prefix(self, prefix):
        return lib().iro_st_file_drop_prefix(self.h, prefix.encode())

    def weight(self, name, transposed=False, bias_name=None):
        """Device int8 weight quantised on the GPU from the file's fp32 tensor."""
        w = DevWeight()
        check(lib().iro_int8_dev_weight_from_st(C.byref(w.st), self.h, name.encode(),
                                                int(bool(transposed)),
                                                bias_name.encode() if bias_name else None),
              "dev_weight_from_st")
        return w


def header_symbols(path=HEADER_PATH):
    """Function names declared in the public header."""
    import re
    txt = open(path).read()
    txt = re.sub(r"/\*.*?\*/", "", txt, flags=re.S)
    return sorted(set(re.findall(r"\b(iro_[a-z0-9_]+)\s*\(", txt)))
