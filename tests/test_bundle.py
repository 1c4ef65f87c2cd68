"""TCM1LE bundles (include/tcm_bundle.h, cmachine_b200/host/bundle.c) on the CPU.

1. tcm_sha256 against Python's hashlib on the FIPS 180-4 test messages and
   random buffers of every tail length.
2. tcm_load against the reference's own loader (src/model.c, built from the
   reference sources into oracle/_ref/libref_bundle.so): on a valid bundle and
   on a set of damaged ones, both accept or refuse with the same message, and
   an accepted bundle gives the same digest, header and tensor table.
3. qwen_model_init refuses what the reference refuses (src/qwen.c:27-31).
"""
import ctypes
import hashlib
import struct
from ctypes import POINTER, Structure, c_char, c_size_t, c_uint32, c_uint64, c_void_p

import numpy as np
import pytest

import cmachine_b200 as cm
from checkers import ROOT

REF_BUNDLE = ROOT / "oracle" / "_ref" / "libref_bundle.so"
HOST_CPU = ROOT / "oracle" / "_ref" / "libqwen_host_cpu.so"


class Tensor(Structure):
    _fields_ = [("name", c_char * 65), ("rank", c_uint32), ("dtype", c_uint32), ("dim", c_uint64 * 4),
                ("bytes", c_uint64), ("data", c_void_p)]


class Bundle(Structure):
    _fields_ = [("architecture", c_uint32), ("count", c_uint32), ("config", c_uint32 * 16), ("identity", c_char * 65),
                ("digest", c_char * 65), ("tensor", POINTER(Tensor)), ("mapping", c_void_p), ("mapping_bytes", c_size_t)]


def loader(path):
    L = ctypes.CDLL(str(path))
    L.tcm_load.argtypes = [POINTER(Bundle), ctypes.c_char_p, ctypes.c_char_p, c_size_t]
    L.tcm_load.restype = ctypes.c_int
    L.tcm_unload.argtypes = [POINTER(Bundle)]
    L.tcm_sha256.argtypes = [c_void_p, c_size_t, c_void_p]
    return L


@pytest.fixture(scope="module")
def ours():
    return loader(cm.LIB_PATH)


def write_bundle(path, architecture, identity, config, tensors, pad=8):
    """The TCM1LE layout: header, 120-byte records in name order, payloads each
    aligned to `pad` bytes (tools/bundle.py's layout, restated)."""
    names = sorted(tensors)
    offset = 176 + 120 * len(names)
    records, blocks = [], []
    for name in names:
        dtype, shape, raw = tensors[name]
        gap = (-offset) % pad
        blocks.append(b"\0" * gap)
        offset += gap
        records.append(struct.pack("<64sII4QQQ", name.encode(), len(shape), dtype, *(list(shape) + [0] * (4 - len(shape))),
                                   offset, len(raw)))
        blocks.append(raw)
        offset += len(raw)
    body = struct.pack("<II16I64s", architecture, len(names), *(list(config) + [0] * (16 - len(config))),
                       identity.encode()) + b"".join(records) + b"".join(blocks)
    path.write_bytes(b"TCM1LE\0\0" + hashlib.sha256(body).digest() + body)
    return path


def sample_tensors():
    rng = np.random.default_rng(5)
    return {
        "a.weight": (1, (3, 4), rng.standard_normal((3, 4)).astype(np.float32).tobytes()),
        "b.bias": (2, (5,), rng.integers(0, 65535, 5, dtype=np.uint16).tobytes()),
        "c.table": (3, (2, 1, 3), rng.standard_normal(6).tobytes()),
    }


def resign(data: bytearray) -> bytes:
    data[8:40] = hashlib.sha256(bytes(data[40:])).digest()
    return bytes(data)


def damaged_variants(good: bytes):
    n = struct.unpack_from("<I", good, 44)[0]
    rec0 = 176
    off0 = struct.unpack_from("<Q", good, rec0 + 104)[0]
    v = {}
    v["magic"] = b"TCM2LE\0\0" + good[8:]
    v["digest"] = good[:8] + bytes(32) + good[40:]
    v["truncated"] = good[:100]
    d = bytearray(good); d[112] = ord("G"); v["identity"] = resign(d)
    d = bytearray(good); struct.pack_into("<I", d, 44, 0); v["count0"] = resign(d)
    d = bytearray(good); struct.pack_into("<I", d, 44, 5000); v["count_big"] = resign(d)
    d = bytearray(good); struct.pack_into("<I", d, 44, n + 40); v["table_past_end"] = resign(d)
    d = bytearray(good); struct.pack_into("<I", d, rec0 + 68, 7); v["dtype"] = resign(d)
    d = bytearray(good); struct.pack_into("<I", d, rec0 + 64, 5); v["rank"] = resign(d)
    d = bytearray(good); struct.pack_into("<Q", d, rec0 + 72, 0); v["zero_dim"] = resign(d)
    d = bytearray(good); struct.pack_into("<Q", d, rec0 + 104, off0 + 2); v["misaligned"] = resign(d)
    d = bytearray(good); struct.pack_into("<Q", d, rec0 + 112, 44); v["size"] = resign(d)
    d = bytearray(good); d[rec0 + 120:rec0 + 128] = d[rec0:rec0 + 8]; v["duplicate"] = resign(d)
    d = bytearray(good); d[rec0:rec0 + 64] = b"x" * 64; v["unterminated"] = resign(d)
    d = bytearray(good); d[rec0] = 0; v["empty_name"] = resign(d)
    v["trailing"] = resign(bytearray(good + b"\0" * 8))
    return v


def load(L, path):
    b = Bundle()
    err = ctypes.create_string_buffer(256)
    status = L.tcm_load(ctypes.byref(b), str(path).encode(), err, 256)
    out = None
    if status == 0:
        out = dict(architecture=b.architecture, count=b.count, config=list(b.config), identity=b.identity,
                   digest=b.digest,
                   tensors=[(b.tensor[i].name, b.tensor[i].rank, b.tensor[i].dtype, list(b.tensor[i].dim),
                             b.tensor[i].bytes, ctypes.string_at(b.tensor[i].data, b.tensor[i].bytes))
                            for i in range(b.count)])
        L.tcm_unload(ctypes.byref(b))
    return status, err.value.decode(), out


@pytest.mark.parametrize("message", [b"", b"abc", b"abcdbcdecdefdefgefghfghighijhijkijkljklmklmnlmnomnopnopq",
                                     b"a" * 1000000])
def test_sha256_known_answers(ours, message):
    buf = ctypes.create_string_buffer(message, len(message) + 1)
    out = ctypes.create_string_buffer(32)
    ours.tcm_sha256(buf, len(message), out)
    assert out.raw == hashlib.sha256(message).digest()


def test_sha256_every_tail_length(ours):
    rng = np.random.default_rng(9)
    for n in range(0, 300):
        data = rng.integers(0, 256, n, dtype=np.uint8).tobytes()
        buf = ctypes.create_string_buffer(data, n + 1)
        out = ctypes.create_string_buffer(32)
        ours.tcm_sha256(buf, n, out)
        assert out.raw == hashlib.sha256(data).digest(), n


@pytest.mark.skipif(not REF_BUNDLE.exists(), reason="reference sources not built here")
def test_loader_matches_reference_loader(ours, tmp_path):
    ref = loader(REF_BUNDLE)
    good = write_bundle(tmp_path / "good.tcm", 2, "ab" * 32, [1536, 28, 7], sample_tensors()).read_bytes()
    cases = {"good": good, **damaged_variants(good)}
    accepted = 0
    for name, data in cases.items():
        p = tmp_path / f"{name}.tcm"
        p.write_bytes(data)
        a, b = load(ours, p), load(ref, p)
        assert a[0] == b[0] and a[1] == b[1], (name, a[:2], b[:2])
        assert a[2] == b[2], name
        accepted += a[0] == 0
    assert accepted == 1  # only the good bundle
    status, _, info = load(ours, tmp_path / "good.tcm")
    assert info["digest"].decode() == hashlib.sha256(good[40:]).hexdigest()
    assert [t[0].decode() for t in info["tensors"]] == ["a.weight", "b.bias", "c.table"]
    assert load(ours, tmp_path / "missing.tcm")[1] == "cannot open model bundle"


@pytest.mark.skipif(not HOST_CPU.exists(), reason="reference sources not built here")
def test_model_init_refuses_other_profiles(tmp_path):
    L = cm.load_library(HOST_CPU)
    L.tcm_load.argtypes = [POINTER(Bundle), ctypes.c_char_p, ctypes.c_char_p, c_size_t]
    L.qwen_model_init.argtypes = [c_void_p, POINTER(Bundle), ctypes.c_char_p, c_size_t]
    L.tcm_unload.argtypes = [POINTER(Bundle)]
    path = write_bundle(tmp_path / "small.tcm", 2, "cd" * 32, [1536, 28, 12, 2, 128, 8960, 151936, 0, 0, 0, 4096],
                        sample_tensors())
    b = Bundle()
    err = ctypes.create_string_buffer(256)
    assert L.tcm_load(ctypes.byref(b), str(path).encode(), err, 256) == 0
    model = ctypes.create_string_buffer(L.qwen_b200_model_size())
    assert L.qwen_model_init(model, ctypes.byref(b), err, 256) == -1
    assert err.value == b"unsupported Qwen2.5-1.5B profile"
    L.tcm_unload(ctypes.byref(b))
