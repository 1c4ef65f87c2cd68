"""Test-side loaders for the CPU checkers under oracle/ (test infrastructure).

liboracle.so is this repository's C restatement of the reference CPU path;
_ref/libref_cpu.so is the reference's own CPU path built from its sources;
_ref/libref_gpuhost.so is the reference's unchanged C host linked against
libcmachine_b200.so. All three export the orc_* ABI of oracle/oracle_api.h.
"""
from __future__ import annotations

import ctypes
from ctypes import POINTER, c_float, c_int, c_uint32, c_uint64, c_void_p
from pathlib import Path

import numpy as np

from cmachine_b200 import FillLaw, Shape, Top2

ROOT = Path(__file__).resolve().parent.parent
ORACLE = ROOT / "oracle" / "liboracle.so"
REF_CPU = ROOT / "oracle" / "_ref" / "libref_cpu.so"
REF_GPUHOST = ROOT / "oracle" / "_ref" / "libref_gpuhost.so"


def load(path: Path):
    if not path.exists():
        raise FileNotFoundError(f"{path} missing: run __graft_entry__.build()")
    L = ctypes.CDLL(str(path))
    L.orc_model_create.restype = c_void_p
    L.orc_model_create.argtypes = [POINTER(Shape), c_uint64, POINTER(FillLaw), c_int]
    L.orc_model_free.argtypes = [c_void_p]
    L.orc_session_create.restype = c_void_p
    L.orc_session_create.argtypes = [c_void_p, c_int]
    L.orc_session_free.argtypes = [c_void_p]
    L.orc_push.argtypes = [c_void_p, c_int, c_void_p, c_void_p]
    L.orc_position.argtypes = [c_void_p]
    L.orc_read_kv.argtypes = [c_void_p, c_int, c_int, c_void_p]
    L.orc_read_hidden.argtypes = [c_void_p, c_void_p]
    L.orc_weight_value.restype = c_float
    L.orc_weight_value.argtypes = [c_void_p, c_uint32, c_uint64]
    L.orc_write_kv.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
    L.orc_set_cursor.argtypes = [c_void_p, c_int]
    if hasattr(L, "orc_stack_push"):  # the reference drivers only
        L.orc_stack_push.argtypes = [c_void_p, POINTER(c_uint64)]
        L.orc_stack_rollback.argtypes = [c_void_p, c_uint64]
    return L


class CpuDecoder:
    """One CPU model + session of a checker library."""

    def __init__(self, path: Path, shape: Shape, seed: int, law: FillLaw, bf16: bool, capacity: int):
        self.L = load(path)
        self.shape = shape
        self.model = self.L.orc_model_create(ctypes.byref(shape), seed, ctypes.byref(law), int(bf16))
        self.session = self.L.orc_session_create(self.model, capacity)
        assert self.session, "checker refused the session"

    def push(self, token: int, readout: bool = True, logits: bool = True):
        if not readout:
            assert self.L.orc_push(self.session, token, None, None) == 0
            return None, None
        top = Top2()
        out = np.empty(self.shape.vocab, np.float32) if logits else None
        assert self.L.orc_push(self.session, token, ctypes.byref(top),
                               c_void_p(out.ctypes.data) if logits else None) == 0
        return top.tuple(), out

    def kv(self, layer: int, kind: int) -> np.ndarray:
        pos = self.L.orc_position(self.session)
        out = np.empty((self.shape.kvheads, pos, self.shape.head), np.float32)
        self.L.orc_read_kv(self.session, layer, kind, c_void_p(out.ctypes.data))
        return out

    def write_kv(self, layer: int, kind: int, rows: np.ndarray):
        """K (kind 0) or V (kind 1) rows 0..n-1 of one layer from [kvheads][n][head]."""
        rows = np.ascontiguousarray(rows, np.float32)
        self.L.orc_write_kv(self.session, layer, kind, rows.shape[1], c_void_p(rows.ctypes.data))

    def set_cursor(self, position: int):
        assert self.L.orc_set_cursor(self.session, position) == 0

    def hidden(self) -> np.ndarray:
        out = np.empty(self.shape.hidden, np.float32)
        self.L.orc_read_hidden(self.session, c_void_p(out.ctypes.data))
        return out

    def weight(self, tensor: int, index: int) -> float:
        return self.L.orc_weight_value(self.model, tensor, index)

    def close(self):
        self.L.orc_session_free(self.session)
        self.L.orc_model_free(self.model)


class OrcRingView(ctypes.Structure):
    _fields_ = [("cursor", c_int), ("population", c_uint64), ("rng", c_uint64)] + [
        (n, c_int) for n in ("write_slot", "sample_slot", "active", "rows")]


class OracleRing(CpuDecoder):
    """The oracle's bounded byte-codec session (liboracle.so only)."""

    def __init__(self, shape: Shape, seed: int, law: FillLaw, bf16: bool, logical: int, anchors: int, recent: int,
                 sample: int):
        self.L = load(ORACLE)
        self.L.orc_ring_session_create.restype = c_void_p
        self.L.orc_ring_session_create.argtypes = [c_void_p, c_int, c_int, c_int, c_int]
        self.L.orc_ring_read.argtypes = [c_void_p, POINTER(OrcRingView), c_void_p, c_void_p, c_void_p, c_void_p]
        self.shape = shape
        self.model = self.L.orc_model_create(ctypes.byref(shape), seed, ctypes.byref(law), int(bf16))
        self.session = self.L.orc_ring_session_create(self.model, logical, anchors, recent, sample)
        assert self.session, "oracle refused the ring"
        self.rows = anchors + recent + sample

    def state(self):
        v = OrcRingView()
        pos = np.empty(self.rows, np.int32)
        order = np.empty(self.rows, np.int32)
        weights = np.empty(self.rows, np.float32)
        arena = np.empty(self.shape.layers * self.rows * 528, np.uint8)
        self.L.orc_ring_read(self.session, ctypes.byref(v), c_void_p(pos.ctypes.data), c_void_p(order.ctypes.data),
                             c_void_p(weights.ctypes.data), c_void_p(arena.ctypes.data))
        return dict(view=(v.cursor, v.population, v.rng), slots=(v.write_slot, v.sample_slot), active=v.active,
                    positions=pos, order=order[:v.active], weights=weights[:v.active], arena=arena)


def codec_rows(x: np.ndarray):
    """The oracle's byte codec (src/byte_codec.h:5-9) over rows of 128: codes, scales."""
    L = load(ORACLE)
    L.orc_codec.argtypes = [c_void_p, c_void_p, c_void_p]
    x = np.ascontiguousarray(x, np.float32).reshape(-1, 128)
    codes = np.empty(x.shape, np.int8)
    scales = np.empty(x.shape[0], np.float32)
    for i in range(x.shape[0]):
        assert L.orc_codec(c_void_p(x[i].ctypes.data), c_void_p(codes[i].ctypes.data),
                           c_void_p(scales[i:].ctypes.data)) == 0
    return codes, scales


def seeded_context(shape, seed: int, rows: int, scale: float = 0.8):
    """Synthetic cached K/V rows for long-context parity: per layer and kind an
    array [kvheads][rows][head] of N(0, scale) values (scale 0.8 is the spread of
    the decoder's own K/V rows under N(0, 0.02) weights), plus every 97th row
    scaled up 4x so the softmax has sharp peaks to place exactly."""
    rng = np.random.default_rng(seed)
    out = []
    for _ in range(shape.layers):
        pair = []
        for _ in range(2):
            a = rng.standard_normal((shape.kvheads, rows, shape.head), dtype=np.float32) * np.float32(scale)
            a[:, ::97, :] *= np.float32(4.0)
            pair.append(a)
        out.append(pair)
    return out
