"""Checkpoint loading (iro_st_file_*): header parsing and page dropping
against the reference's own loader (safetensors.c via oracle/_ref), on CPU;
device quantisation straight from the mapping against the host quantiser,
bit-exact, on the GPU."""
import ctypes as C
import json
import os

import numpy as np
import pytest

import iro_b200 as iro
import oracle


def write_safetensors(path, tensors, metadata=None):
    """tensors: list of (name, float32/other numpy array)."""
    header, blobs, off = {}, [], 0
    dt = {np.dtype(np.float32): "F32", np.dtype(np.int8): "I8", np.dtype(np.int32): "I32"}
    for name, a in tensors:
        a = np.ascontiguousarray(a)
        header[name] = {"dtype": dt[a.dtype], "shape": list(a.shape),
                        "data_offsets": [off, off + a.nbytes]}
        blobs.append(a.tobytes())
        off += a.nbytes
    if metadata:
        header["__metadata__"] = metadata
    hj = json.dumps(header).encode()
    hj += b" " * ((8 - len(hj) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(hj).to_bytes(8, "little"))
        f.write(hj)
        for b in blobs:
            f.write(b)


def checkpoint(tmp_path, seed=0):
    rng = np.random.default_rng(seed)
    ts = [("blocks.0.attention.wq.weight", rng.standard_normal((96, 128)).astype(np.float32) * 0.02),
          ("blocks.0.mlp.w1.weight", rng.standard_normal((200, 128)).astype(np.float32) * 0.02),
          ("blocks.0.mlp.w1.bias", rng.standard_normal(200).astype(np.float32) * 0.01),
          ("blocks.0.mlp.w2.weight", rng.standard_normal((128, 3000)).astype(np.float32)),
          ("blocks.1.attention.wq.weight", rng.standard_normal((128, 64)).astype(np.float32)),
          ("step", np.arange(7, dtype=np.int32)),
          ("codes", rng.integers(-128, 127, (5, 9), dtype=np.int8))]
    ts[3][1][3, 17] = 40.0  # an outlier channel
    path = str(tmp_path / "model.safetensors")
    write_safetensors(path, ts, {"format": "pt", "config_json": "{\"a\": [1, 2]}"})
    return path, dict(ts)


def test_header_and_data(tmp_path):
    path, ts = checkpoint(tmp_path)
    f = iro.StFile(path)
    assert sorted(f.names()) == sorted(ts)
    for name, a in ts.items():
        dtype, shape, nbytes = f.tensor(name)
        assert shape == a.shape and nbytes == a.nbytes
        assert dtype == {np.dtype(np.float32): 0, np.dtype(np.int32): 4, np.dtype(np.int8): 6}[a.dtype]
        ptr = iro.lib().iro_st_file_data(f.h, name.encode())
        got = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(a.nbytes,))
        assert bytes(got) == a.tobytes()
    f.close()


def test_malformed_files_are_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    h = json.dumps({"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 32]}}).encode()
    p.write_bytes(len(h).to_bytes(8, "little") + h + b"\0" * 16)  # data shorter than claimed
    with pytest.raises(iro.IroError):
        iro.StFile(str(p))
    p.write_bytes((1 << 40).to_bytes(8, "little") + b"{}")  # header longer than the file
    with pytest.raises(iro.IroError):
        iro.StFile(str(p))
    h = json.dumps({"x": {"dtype": "F32", "shape": [3], "data_offsets": [0, 16]}}).encode()
    p.write_bytes(len(h).to_bytes(8, "little") + h + b"\0" * 16)  # size != shape x dtype
    with pytest.raises(iro.IroError):
        iro.StFile(str(p))


class _RefSafetensors(C.Structure):
    # irodori.h: IroSafetensors
    _fields_ = [("fd", C.c_int), ("map_size", C.c_uint64), ("map", C.c_void_p),
                ("header", C.c_char_p), ("tensors", C.c_void_p), ("n_tensors", C.c_int),
                ("meta_keys", C.c_void_p), ("meta_values", C.c_void_p), ("n_meta", C.c_int)]


@pytest.mark.skipif(not os.path.exists(os.path.join(oracle.REF_DIR, "libiro_ref_codec.so")),
                    reason="reference build absent")
def test_drop_prefix_matches_reference(tmp_path):
    path, ts = checkpoint(tmp_path)
    L = oracle.ref_lib("codec")
    L.iro_st_load.argtypes = [C.c_char_p, C.POINTER(_RefSafetensors)]
    L.iro_st_load.restype = C.c_int
    L.iro_st_drop_prefix.argtypes = [C.POINTER(_RefSafetensors), C.c_char_p]
    L.iro_st_drop_prefix.restype = C.c_uint64
    L.iro_st_free.argtypes = [C.POINTER(_RefSafetensors)]
    L.iro_st_free.restype = None
    ref = _RefSafetensors()
    assert L.iro_st_load(path.encode(), C.byref(ref)) == 0
    assert ref.n_tensors == len(ts)
    f = iro.StFile(path)
    for prefix in ("blocks.0.mlp.", "blocks.0.", "blocks.1.attention.wq.", "step", "nothing."):
        want = L.iro_st_drop_prefix(C.byref(ref), prefix.encode())
        assert f.drop_prefix(prefix) == want, prefix
    # Pointers stay valid: the pages fault back in with the file's bytes.
    for name, a in ts.items():
        ptr = iro.lib().iro_st_file_data(f.h, name.encode())
        got = np.ctypeslib.as_array(C.cast(ptr, C.POINTER(C.c_uint8)), shape=(a.nbytes,))
        assert bytes(got) == a.tobytes()
    f.close()
    L.iro_st_free(C.byref(ref))


def _dev_weight_arrays(w):
    N, K, ld = w.st.N, w.st.K, w.st.ld
    data = np.empty((N, ld), np.int8)
    scale = np.empty(N, np.float32)
    colsum = np.empty(N, np.int32)
    for dst, src in ((data, w.st.data), (scale, w.st.scale), (colsum, w.st.colsum)):
        iro.check(iro.lib().iro_memcpy_dtoh(dst.ctypes.data_as(C.c_void_p), C.c_void_p(src),
                                            dst.nbytes, None), "dtoh")
    return data[:, :K], scale, colsum


@pytest.mark.gpu
@pytest.mark.parametrize("name,transposed,bias", [
    ("blocks.0.attention.wq.weight", False, None),
    ("blocks.0.mlp.w1.weight", False, "blocks.0.mlp.w1.bias"),
    ("blocks.0.mlp.w2.weight", False, None),
    ("blocks.0.mlp.w2.weight", True, None),
    ("blocks.1.attention.wq.weight", True, None)])
def test_device_quantisation_from_checkpoint(tmp_path, name, transposed, bias):
    iro.init(0)
    path, ts = checkpoint(tmp_path, seed=3)
    f = iro.StFile(path)
    w = f.weight(name, transposed=transposed, bias_name=bias)
    src = ts[name].T if transposed else ts[name]
    want = oracle.weight_quantize(np.ascontiguousarray(src))
    data, scale, colsum = _dev_weight_arrays(w)
    assert (data == want.data).all()
    assert (scale.view(np.uint32) == want.scale.view(np.uint32)).all()
    assert (colsum == want.colsum).all()
    if bias:
        b = np.empty(w.st.N, np.float32)
        iro.check(iro.lib().iro_memcpy_dtoh(b.ctypes.data_as(C.c_void_p), C.c_void_p(w.st.bias),
                                            b.nbytes, None), "dtoh")
        assert (b == ts[bias]).all()
    # The fp32 pages can go once quantised (generate.c:543-556).
    assert f.drop_prefix(name) > 0
    w.free()
    f.close()


@pytest.mark.gpu
def test_checkpoint_rejects_non_f32_and_missing(tmp_path):
    iro.init(0)
    path, _ = checkpoint(tmp_path)
    f = iro.StFile(path)
    for name in ("codes", "step", "missing.weight"):
        with pytest.raises(iro.IroError):
            f.weight(name)
    f.close()
