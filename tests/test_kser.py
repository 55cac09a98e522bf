"""The .ser format (include/kser.h, csrc/kser.cpp) against the reference's own
libkser (libs/kser/src/*.c, compiled in place into oracle/_ref): the same
bytes written for the same content, each reader opening the other's files,
the same quantised / dequantised values, and the SHA-256 against hashlib.
CPU only: the format code is host code."""
import ctypes as C
import hashlib
import os

import numpy as np
import pytest

import bissimamba_b200 as kmb
from oracle import pyoracle as po


class KSerConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_uint32), ("dim", C.c_uint32), ("state_size", C.c_uint32),
                ("n_layers", C.c_uint32), ("seq_len", C.c_uint32), ("d_conv", C.c_uint32),
                ("expand_factor", C.c_float), ("dtype", C.c_uint8), ("_pad", C.c_uint8 * 3),
                ("model_name", C.c_char * 64)]


class KSerTensorEntry(C.Structure):
    _fields_ = [("name", C.c_char * 32), ("shape", C.c_uint32 * 4), ("dtype", C.c_uint8), ("_pad", C.c_uint8 * 7),
                ("offset", C.c_uint64), ("size_bytes", C.c_uint64)]


def _bind(L):
    vp = C.c_void_p
    for fn in ("kser_writer_create", "kser_reader_open", "kser_reader_config", "kser_reader_load_tensor",
               "kser_reader_get_tensor_info"):
        getattr(L, fn).restype = vp
    L.kser_writer_create.argtypes = [C.c_char_p, vp]
    L.kser_writer_add_vocab.argtypes = [vp, C.c_uint32, C.c_char_p, C.c_uint16]
    L.kser_writer_add_tensor.argtypes = [vp, C.c_char_p, vp, vp, C.c_int, C.c_int]
    L.kser_writer_finalize.argtypes = [vp]
    L.kser_writer_free.argtypes = [vp]
    L.kser_writer_free.restype = None
    L.kser_reader_open.argtypes = [C.c_char_p]
    L.kser_reader_config.argtypes = [vp]
    L.kser_reader_is_valid.argtypes = [vp]
    L.kser_reader_load_tensor.argtypes = [vp, C.c_char_p]
    L.kser_reader_count_tensors.argtypes = [vp]
    L.kser_reader_count_tensors.restype = C.c_uint64
    L.kser_reader_get_tensor_info.argtypes = [vp, C.c_uint64]
    L.kser_reader_close.argtypes = [vp]
    L.kser_reader_close.restype = None
    L.kser_quantize.argtypes = [vp, vp, C.c_uint64, C.c_int]
    L.kser_dequantize.argtypes = [vp, vp, C.c_uint64, C.c_int]
    return L


@pytest.fixture(scope="module")
def libs():
    if not po.have_ref():
        pytest.skip("reference build unavailable")
    ref = _bind(C.CDLL(po.REF_SO))
    return _bind(kmb.lib()), ref


libc = C.CDLL(None)
libc.free.argtypes = [C.c_void_p]

FP32, FP16, BF16, INT8 = 0, 1, 2, 3


def _write(L, path, cfg, vocab, tensors):
    w = L.kser_writer_create(path.encode(), C.byref(cfg))
    assert w
    for i, tok in vocab:
        assert L.kser_writer_add_vocab(w, i, tok, len(tok)) == 0
    for name, arr, shape, sdt in tensors:
        sh = (C.c_uint32 * 4)(*shape)
        assert L.kser_writer_add_tensor(w, name.encode(), arr.ctypes.data, sh, FP32, sdt) == 0
    assert L.kser_writer_finalize(w) == 0
    L.kser_writer_free(w)


def _content(seed=0):
    rng = np.random.default_rng(seed)
    cfg = KSerConfig(vocab_size=300, dim=24, state_size=8, n_layers=2, seq_len=30, d_conv=4, expand_factor=2.0,
                     dtype=BF16, model_name=b"kmamba-test")
    vocab = [(i, f"tok{i}é".encode()) for i in range(0, 300, 7)]
    special = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -3e-38, 65504.0, 70000.0, 6e-8, 1.0 + 2 ** -11],
                       np.float32)
    tensors = [("embedding", rng.standard_normal((300, 24)).astype(np.float32), (300, 24, 0, 0), FP32),
               ("layers.0.W_B", rng.standard_normal((16, 24)).astype(np.float32), (16, 24, 0, 0), BF16),
               ("layers.0.theta", rng.uniform(0, 1, 4).astype(np.float32), (4, 0, 0, 0), FP16),
               ("layers.1.W_C", (rng.standard_normal(384) * 3).astype(np.float32), (16, 24, 0, 0), INT8),
               ("special16", special, (special.size, 0, 0, 0), FP16),
               ("specialbf", special, (special.size, 0, 0, 0), BF16),
               ("head", rng.standard_normal((24, 300)).astype(np.float32), (24, 300, 0, 0), FP32)]
    return cfg, vocab, tensors


def test_sha256_matches_hashlib(libs):
    ours, _ = libs
    rng = np.random.default_rng(1)
    for n in (0, 1, 3, 55, 56, 57, 63, 64, 65, 127, 128, 1000, 100003):
        data = rng.integers(0, 256, n, dtype=np.uint8)
        out = (C.c_uint8 * 32)()
        ours.kser_sha256(data.ctypes.data, n, out)
        assert bytes(out) == hashlib.sha256(data.tobytes()).digest(), n


@pytest.mark.parametrize("dtype", [FP32, FP16, BF16, INT8])
def test_quantize_matches_reference(libs, dtype):
    ours, ref = libs
    rng = np.random.default_rng(dtype)
    x = np.concatenate([rng.standard_normal(1000) * 10, rng.standard_normal(1000) * 1e-5,
                        np.array([0.0, -0.0, 65504.0, 65519.0, 1e6, -1e-7, 5.9e-8, 3e-45])]).astype(np.float32)
    if dtype != INT8:
        x = np.concatenate([x, np.array([np.inf, -np.inf, np.nan], np.float32)])
    nb = x.size * (4 if dtype == FP32 else 2 if dtype in (FP16, BF16) else 1) + (8 if dtype == INT8 else 0)
    qa, qb = np.zeros(nb, np.uint8), np.zeros(nb, np.uint8)
    assert ours.kser_quantize(x.ctypes.data, qa.ctypes.data, x.size, dtype) == 0
    assert ref.kser_quantize(x.ctypes.data, qb.ctypes.data, x.size, dtype) == 0
    assert np.array_equal(qa, qb)
    da, db = np.zeros(x.size, np.float32), np.zeros(x.size, np.float32)
    assert ours.kser_dequantize(qa.ctypes.data, da.ctypes.data, x.size, dtype) == 0
    assert ref.kser_dequantize(qb.ctypes.data, db.ctypes.data, x.size, dtype) == 0
    assert np.array_equal(da.view(np.uint32), db.view(np.uint32))


def test_writer_bytes_equal_reference(libs, tmp_path):
    ours, ref = libs
    cfg, vocab, tensors = _content()
    a, b = str(tmp_path / "ours.ser"), str(tmp_path / "ref.ser")
    _write(ours, a, cfg, vocab, tensors)
    _write(ref, b, cfg, vocab, tensors)
    assert open(a, "rb").read() == open(b, "rb").read()
    assert not os.path.exists(a + ".tmp")


def _read_all(L, path):
    r = L.kser_reader_open(path.encode())
    assert r
    cfg = KSerConfig.from_address(L.kser_reader_config(r))
    out = {"cfg": bytes(cfg), "valid": L.kser_reader_is_valid(r), "tensors": {}}
    for i in range(L.kser_reader_count_tensors(r)):
        e = KSerTensorEntry.from_address(L.kser_reader_get_tensor_info(r, i))
        n = int(np.prod([s for s in e.shape if s > 0]))
        p = L.kser_reader_load_tensor(r, e.name)
        arr = np.ctypeslib.as_array((C.c_float * n).from_address(p)).copy()
        libc.free(p)
        out["tensors"][e.name.decode()] = (tuple(e.shape), e.dtype, e.offset, e.size_bytes, arr)
    L.kser_reader_close(r)
    return out


def test_readers_open_each_others_files(libs, tmp_path):
    ours, ref = libs
    cfg, vocab, tensors = _content(seed=5)
    a, b = str(tmp_path / "ours.ser"), str(tmp_path / "ref.ser")
    _write(ours, a, cfg, vocab, tensors)
    _write(ref, b, cfg, vocab, tensors)
    for path in (a, b):
        x, y = _read_all(ours, path), _read_all(ref, path)
        assert x["cfg"] == y["cfg"] and x["valid"] == 1
        assert x["tensors"].keys() == y["tensors"].keys() == {t[0] for t in tensors}
        for k in x["tensors"]:
            assert x["tensors"][k][:4] == y["tensors"][k][:4]
            assert np.array_equal(x["tensors"][k][4].view(np.uint32), y["tensors"][k][4].view(np.uint32)), k
    # a flipped data byte is caught by the checksum (the file still opens)
    raw = bytearray(open(a, "rb").read())
    raw[200] ^= 1
    bad = str(tmp_path / "bad.ser")
    open(bad, "wb").write(bytes(raw))
    assert _read_all(ours, bad)["valid"] == 0
    # not a .ser file
    open(bad, "wb").write(b"x" * 400)
    assert not ours.kser_reader_open(bad.encode())
